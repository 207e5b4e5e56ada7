/*
 * lancius_arena.h -- chained bump allocator for IR nodes and host scratch.
 * Same entry points as the reference's lancius_arena.h:12-15.
 */
#ifndef LANCIUS_ARENA_H
#define LANCIUS_ARENA_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct lancius_arena lancius_arena;

lancius_arena* lancius_arena_create(size_t block_size);
void* lancius_arena_alloc(lancius_arena* arena, size_t size, size_t alignment);
void lancius_arena_reset(lancius_arena* arena);
void lancius_arena_destroy(lancius_arena* arena);

#ifdef __cplusplus
}
#endif
#endif
