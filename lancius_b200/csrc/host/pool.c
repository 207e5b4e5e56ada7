/* Worker pool with the reference's interface (bleeding/v11A1/include/lancius/
 * lancius_threadpool.h:10-24): a FIFO of tasks under one mutex, `num_threads`
 * pthreads, lancius_pool_wait returns once every submitted task has finished.
 * The GPU executors do not use it; it exists so that programs written against the
 * reference (which create one for lancius_schedule_execute_parallel) link and run. */
#define _POSIX_C_SOURCE 200809L
#include "lancius/lancius_threadpool.h"
#include "lancius/lancius_error.h"

#include <pthread.h>
#include <stdlib.h>

struct lancius_pool {
    pthread_mutex_t mu;
    pthread_cond_t has_work, idle;
    lancius_task* q;
    size_t head, count, cap;
    size_t running;       /* tasks taken off the queue and not yet finished */
    int stop, nthreads;
    pthread_t* threads;
};

static void* worker(void* arg) {
    lancius_pool* p = (lancius_pool*)arg;
    pthread_mutex_lock(&p->mu);
    for (;;) {
        while (!p->stop && p->count == 0) pthread_cond_wait(&p->has_work, &p->mu);
        if (p->count == 0 && p->stop) break;
        lancius_task t = p->q[p->head];
        p->head = (p->head + 1) % p->cap;
        p->count--;
        p->running++;
        pthread_mutex_unlock(&p->mu);
        t.fn(t.arg);
        pthread_mutex_lock(&p->mu);
        p->running--;
        if (p->count == 0 && p->running == 0) pthread_cond_broadcast(&p->idle);
    }
    pthread_mutex_unlock(&p->mu);
    return NULL;
}

lancius_pool* lancius_pool_create(int num_threads) {
    if (num_threads < 1) num_threads = 1;
    lancius_pool* p = (lancius_pool*)calloc(1, sizeof(*p));
    if (!p) { lancius_set_error(LANCIUS_ERROR_OOM); return NULL; }
    p->cap = 64;
    p->q = (lancius_task*)malloc(p->cap * sizeof(lancius_task));
    p->threads = (pthread_t*)calloc((size_t)num_threads, sizeof(pthread_t));
    if (!p->q || !p->threads) { free(p->q); free(p->threads); free(p); lancius_set_error(LANCIUS_ERROR_OOM); return NULL; }
    pthread_mutex_init(&p->mu, NULL);
    pthread_cond_init(&p->has_work, NULL);
    pthread_cond_init(&p->idle, NULL);
    for (int i = 0; i < num_threads; i++) {
        if (pthread_create(&p->threads[i], NULL, worker, p) != 0) break;
        p->nthreads++;
    }
    if (p->nthreads == 0) { lancius_pool_destroy(p); lancius_set_error(LANCIUS_ERROR_INTERNAL); return NULL; }
    return p;
}

void lancius_pool_submit(lancius_pool* p, lancius_task_fn fn, void* arg) {
    if (!p || !fn) { lancius_set_error(LANCIUS_ERROR_NULL_PTR); return; }
    pthread_mutex_lock(&p->mu);
    if (p->count == p->cap) {   /* grow, unrolling the ring */
        size_t ncap = p->cap * 2;
        lancius_task* nq = (lancius_task*)malloc(ncap * sizeof(lancius_task));
        if (!nq) {
            pthread_mutex_unlock(&p->mu);
            fn(arg);               /* no room: run it on the caller's thread */
            return;
        }
        for (size_t i = 0; i < p->count; i++) nq[i] = p->q[(p->head + i) % p->cap];
        free(p->q);
        p->q = nq; p->head = 0; p->cap = ncap;
    }
    p->q[(p->head + p->count) % p->cap] = (lancius_task){fn, arg};
    p->count++;
    pthread_cond_signal(&p->has_work);
    pthread_mutex_unlock(&p->mu);
}

void lancius_pool_wait(lancius_pool* p) {
    if (!p) return;
    pthread_mutex_lock(&p->mu);
    while (p->count || p->running) pthread_cond_wait(&p->idle, &p->mu);
    pthread_mutex_unlock(&p->mu);
}

void lancius_pool_destroy(lancius_pool* p) {
    if (!p) return;
    pthread_mutex_lock(&p->mu);
    p->stop = 1;
    pthread_cond_broadcast(&p->has_work);
    pthread_mutex_unlock(&p->mu);
    for (int i = 0; i < p->nthreads; i++) pthread_join(p->threads[i], NULL);
    pthread_mutex_destroy(&p->mu);
    pthread_cond_destroy(&p->has_work);
    pthread_cond_destroy(&p->idle);
    free(p->q);
    free(p->threads);
    free(p);
}
