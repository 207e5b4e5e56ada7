/*
 * lancius_threadpool.h -- worker pool. Same types and entry points as the
 * reference's bleeding/v11A1/include/lancius/lancius_threadpool.h:10-24, so programs
 * that create a pool for lancius_schedule_execute_parallel link unchanged. The GPU
 * executors do not submit to it (a wave's nodes run concurrently on the device);
 * it remains a working pthread pool for the caller's own tasks.
 */
#ifndef LANCIUS_THREADPOOL_H
#define LANCIUS_THREADPOOL_H
#include <stdbool.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef void (*lancius_task_fn)(void*);

typedef struct {
    lancius_task_fn fn;
    void* arg;
} lancius_task;

typedef struct lancius_pool lancius_pool;

lancius_pool* lancius_pool_create(int num_threads);
void lancius_pool_submit(lancius_pool* pool, lancius_task_fn fn, void* arg);
void lancius_pool_wait(lancius_pool* pool);
void lancius_pool_destroy(lancius_pool* pool);

#ifdef __cplusplus
}
#endif
#endif
