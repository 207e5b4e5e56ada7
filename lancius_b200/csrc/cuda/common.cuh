// Shared helpers for the sm_100a kernels and their launchers.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>
#include <stddef.h>
#include "lancius_cuda.h"

#define LCU_SMS 148   // B200: 2 dies x 74 SMs

static inline cudaStream_t lcu_as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// Map a CUDA status onto the Lancius thread-local error and return it.
extern "C" void lcu_note_cuda_error(int e);
static inline lancius_error lcu_check_cuda(cudaError_t e) {
    if (e == cudaSuccess) return LANCIUS_ERROR_OK;
    lcu_note_cuda_error((int)e);
    lancius_error le = (e == cudaErrorMemoryAllocation) ? LANCIUS_ERROR_OOM : LANCIUS_ERROR_INTERNAL;
    lancius_set_error(le);
    return le;
}
// After a launch: configuration errors only (no device sync).
static inline lancius_error lcu_launch_status() { return lcu_check_cuda(cudaGetLastError()); }

static inline unsigned lcu_blocks(size_t n, unsigned per_block, unsigned cap = 148u * 16u) {
    size_t b = (n + per_block - 1) / per_block;
    if (b == 0) b = 1;
    return (unsigned)(b < cap ? b : cap);
}

__device__ __forceinline__ float lcu_gelu_f(float x) {
    // tanh-form GELU with the reference's clamp to [-100, 100] (lancius_kernels.c:238-246)
    x = fminf(fmaxf(x, -100.f), 100.f);
    const float c = 0.7978845608028654f;
    return 0.5f * x * (1.f + tanhf(c * (x + 0.044715f * x * x * x)));
}

__device__ __forceinline__ float lcu_apply_epi(float v, int epi) {
    if (epi == LCU_EPI_RELU) return v > 0.f ? v : 0.f;
    if (epi == LCU_EPI_GELU) return lcu_gelu_f(v);
    return v;
}

// Launch-count bookkeeping used by the executor and the per-op API.
extern "C" void lcu_note_launch(void);
