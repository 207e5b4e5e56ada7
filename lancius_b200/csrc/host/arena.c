/* Chained bump allocator (reference contract: bleeding/v11A1/src/core/lancius_arena.c:30-100).
 * Every allocation is rounded up to a 32-byte footprint; a request larger than the
 * block size gets a dedicated block; reset keeps only the first block. */
#include "lancius/lancius_arena.h"
#include <stdlib.h>

typedef struct chunk { struct chunk* next; size_t cap, used; unsigned char* mem; } chunk;
struct lancius_arena { chunk* head; chunk* cur; size_t block; };

static chunk* chunk_new(size_t cap) {
    chunk* c = (chunk*)malloc(sizeof(chunk));
    if (!c) return NULL;
    c->mem = (unsigned char*)malloc(cap);
    if (!c->mem) { free(c); return NULL; }
    c->cap = cap; c->used = 0; c->next = NULL;
    return c;
}

lancius_arena* lancius_arena_create(size_t block_size) {
    lancius_arena* a = (lancius_arena*)calloc(1, sizeof(*a));
    if (!a) return NULL;
    a->block = block_size ? block_size : ((size_t)16 << 20);
    a->head = a->cur = chunk_new(a->block);
    if (!a->head) { free(a); return NULL; }
    return a;
}

void* lancius_arena_alloc(lancius_arena* a, size_t size, size_t alignment) {
    if (!a) return NULL;
    if (alignment == 0) alignment = 32;
    if (alignment & (alignment - 1)) return NULL;
    if (size == 0) size = 1;
    if (size > SIZE_MAX - 64 - alignment) return NULL;
    size = (size + 31) & ~(size_t)31;
    chunk* c = a->cur;
    uintptr_t base = (uintptr_t)(c->mem + c->used);
    size_t pad = (size_t)(((base + alignment - 1) & ~(uintptr_t)(alignment - 1)) - base);
    if (pad + size > c->cap - c->used) {
        size_t cap = size + alignment > a->block ? size + alignment : a->block;
        chunk* n = chunk_new(cap);
        if (!n) return NULL;
        c->next = n; a->cur = c = n;
        base = (uintptr_t)c->mem;
        pad = (size_t)(((base + alignment - 1) & ~(uintptr_t)(alignment - 1)) - base);
    }
    c->used += pad + size;
    return (void*)(base + pad);
}

void lancius_arena_reset(lancius_arena* a) {
    if (!a) return;
    chunk* c = a->head->next;
    while (c) { chunk* n = c->next; free(c->mem); free(c); c = n; }
    a->head->next = NULL; a->head->used = 0; a->cur = a->head;
}

void lancius_arena_destroy(lancius_arena* a) {
    if (!a) return;
    chunk* c = a->head;
    while (c) { chunk* n = c->next; free(c->mem); free(c); c = n; }
    free(a);
}
