// lcu_matmul_noalloc: the tensor-core GEMM (3xTF32 / TF32, see gemm_tc.cu) with
// its scratch taken from a fixed array compiled into this library instead of
// from cudaMalloc.
//
// Who needs it: callers that must not allocate device memory after start-up --
// a serving process whose device memory is owned and budgeted by another
// allocator (a framework arena, a memory-capped inference server), or a
// deployment that, like Lancius' static flat-buffer executor, fixes its memory
// footprint up front. lcu_matmul grows a cached cudaMalloc'd buffer on demand;
// this entry point never allocates or frees anything.
//
// Limits and sharing rules:
//   * scratch is LCU_NOALLOC_SCRATCH_BYTES (64 MiB) per GPU, held until process
//     exit. When the GPU reserves it depends on CUDA's module loading: eagerly
//     (CUDA_MODULE_LOADING=EAGER) every GPU that loads the library pays it at
//     context creation; lazily (the default) it is reserved by the first
//     lcu_noalloc_prepare / lcu_matmul_noalloc call on that GPU, which can then
//     fail with LANCIUS_ERROR_OOM in a memory-capped process. Call
//     lcu_noalloc_prepare() once per GPU at start-up to settle it there. The need is lcu_gemm_tc_scratch_bytes(...) + 256
//     (about 16*(M*K + K*N) bytes in FP32-exact mode, plus split-K partials when
//     K > 8192); larger problems are rejected with LANCIUS_ERROR_OVERFLOW.
//   * every call on a device uses the same array: calls whose work overlaps on
//     the GPU (other streams, other host threads) race on it. Serialize them.
//   * nothing in the array has to start at zero (every byte a call reads, that
//     call wrote first), so the array is never cleared.
//   * the first call on each device looks up the array's device address
//     (cudaGetSymbolAddress, with that device current); make that first call
//     (or lcu_noalloc_prepare) before any stream capture.
#include "lcu_internal.h"
#include <cstdio>
#include <mutex>

#define LCU_NOALLOC_SCRATCH_BYTES (64u << 20)

static __device__ __align__(256) unsigned char g_noalloc_scratch[LCU_NOALLOC_SCRATCH_BYTES];

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_addr[kMaxDevices] = {};

// Device address of the array on the current device (looked up once per device);
// NULL with the Lancius error set (OOM when the module load could not reserve it).
void* scratch_address(int dev) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_addr[dev]) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) {
            fprintf(stderr, "[LANCIUS CUDA] lcu_matmul_noalloc: cudaGetSymbolAddress failed on device %d: %s\n", dev,
                    cudaGetErrorString(e));
            cudaGetLastError();
            lcu_check_cuda(e);
            return nullptr;
        }
        g_addr[dev] = p;
    }
    return g_addr[dev];
}

lancius_error current_scratch(char** out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        cudaGetLastError();
        lancius_set_error(LANCIUS_ERROR_INTERNAL);
        return LANCIUS_ERROR_INTERNAL;
    }
    *out = static_cast<char*>(scratch_address(dev));
    return *out ? LANCIUS_ERROR_OK : lancius_get_error();
}
}  // namespace

extern "C" size_t lcu_noalloc_scratch_capacity(void) { return LCU_NOALLOC_SCRATCH_BYTES; }

extern "C" lancius_error lcu_noalloc_prepare(void) {
    char* scratch = nullptr;
    return current_scratch(&scratch);
}

extern "C" lancius_error lcu_matmul_noalloc(float* out, const float* a, const float* b, size_t M, size_t K, size_t N,
                                            const float* bias, int epilogue, int mode, void* stream) {
    if (!out || !a || !b) { lancius_set_error(LANCIUS_ERROR_NULL_PTR); return LANCIUS_ERROR_NULL_PTR; }
    if (epilogue < LCU_EPI_NONE || epilogue > LCU_EPI_GELU) { lancius_set_error(LANCIUS_ERROR_UNSUPPORTED_OP); return LANCIUS_ERROR_UNSUPPORTED_OP; }
    if (mode != LCU_MODE_FP32_EXACT && mode != LCU_MODE_TF32) { lancius_set_error(LANCIUS_ERROR_UNSUPPORTED_DTYPE); return LANCIUS_ERROR_UNSUPPORTED_DTYPE; }
    if (M == 0 || N == 0 || K == 0) { lancius_set_error(LANCIUS_ERROR_SHAPE_MISMATCH); return LANCIUS_ERROR_SHAPE_MISMATCH; }
    // Every scratch term is a multiple of M*K, K*N or M*N times at least 4 bytes, so a
    // problem past these bounds cannot fit; checking them first keeps the size
    // arithmetic below far from wrapping.
    const size_t cap_elems = LCU_NOALLOC_SCRATCH_BYTES / 4;
    if (M > cap_elems || N > cap_elems || K > cap_elems || M * K > cap_elems || K * N > cap_elems || M * N > cap_elems) {
        fprintf(stderr, "[LANCIUS CUDA] lcu_matmul_noalloc: %zux%zux%zu exceeds the fixed %u-byte scratch array\n", M, K, N,
                LCU_NOALLOC_SCRATCH_BYTES);
        lancius_set_error(LANCIUS_ERROR_OVERFLOW);
        return LANCIUS_ERROR_OVERFLOW;
    }
    const int passes = mode == LCU_MODE_TF32 ? 1 : 3;
    const size_t need = lcu_gemm_tc_scratch_bytes(M, N, K, 1, 1, 1, passes) + 256;
    if (need > LCU_NOALLOC_SCRATCH_BYTES) {
        fprintf(stderr, "[LANCIUS CUDA] lcu_matmul_noalloc: %zux%zux%zu needs %zu scratch bytes, the fixed array holds %u\n",
                M, K, N, need, LCU_NOALLOC_SCRATCH_BYTES);
        lancius_set_error(LANCIUS_ERROR_OVERFLOW);
        return LANCIUS_ERROR_OVERFLOW;
    }
    char* scratch = nullptr;
    lancius_error se0 = current_scratch(&scratch);
    if (se0 != LANCIUS_ERROR_OK) return se0;
    // the one-entry group record sits in the last 256 bytes of this call's region
    LcuGemmGroup* d_group = reinterpret_cast<LcuGemmGroup*>(scratch + need - 256);
    LcuGemmGroup h{a, b, out, bias, nullptr};
    cudaStream_t st = lcu_as_stream(stream);
    cudaError_t ce = cudaMemcpyAsync(d_group, &h, sizeof(h), cudaMemcpyHostToDevice, st);
    if (ce != cudaSuccess) return lcu_check_cuda(ce);
    LcuTcGemmPlan p;
    lancius_error e = lcu_gemm_tc_prepare(&p, scratch, M, N, K, 1, 1, 1, passes);
    if (e == LANCIUS_ERROR_OK) e = lcu_gemm_tc_run(&p, d_group, epilogue, stream);
    // `h` lives on this stack frame: wait until the copy (and the GEMM) ran
    lancius_error se = lcu_check_stream(st);
    return e != LANCIUS_ERROR_OK ? e : se;
}
