// Column-split GEMM across the GPUs of one box (the one path with a real exchange):
// rank r of g holds A [M, K] and its column slab B_r [K, N/g] (contiguous), computes
// C_r = A * B_r on its tensor cores, then ncclAllGather collects the g blocks
// [g][M][N/g] in every rank's memory and a repack kernel writes row-major C [M, N].
// The remote blocks cross NVLink once, through NCCL, into local memory; no kernel
// reads another GPU's memory.
//
// NCCL is opened with dlopen at the first lcu_comm_* call, so the library has no
// link-time NCCL dependency and shares the process's NCCL if one is loaded.
#include "lcu_internal.h"
#include <dlfcn.h>
#include <nccl.h>
#include <cstdio>
#include <cstring>
#include <mutex>

namespace {

struct NcclApi {
    ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
    ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
    ncclResult_t (*comm_abort)(ncclComm_t) = nullptr;
    ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    const char* (*error_string)(ncclResult_t) = nullptr;
    bool ok = false;
};

NcclApi& nccl() {
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, [] {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL | RTLD_NOLOAD);
        if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) { fprintf(stderr, "[LANCIUS CUDA] libnccl.so.2 not found: %s\n", dlerror()); return; }
        api.get_unique_id = (decltype(api.get_unique_id))dlsym(h, "ncclGetUniqueId");
        api.comm_init_rank = (decltype(api.comm_init_rank))dlsym(h, "ncclCommInitRank");
        api.comm_destroy = (decltype(api.comm_destroy))dlsym(h, "ncclCommDestroy");
        api.comm_abort = (decltype(api.comm_abort))dlsym(h, "ncclCommAbort");
        api.all_gather = (decltype(api.all_gather))dlsym(h, "ncclAllGather");
        api.error_string = (decltype(api.error_string))dlsym(h, "ncclGetErrorString");
        api.ok = api.get_unique_id && api.comm_init_rank && api.comm_destroy && api.comm_abort && api.all_gather;
    });
    return api;
}

lancius_error nccl_fail(ncclResult_t r, const char* what) {
    NcclApi& n = nccl();
    fprintf(stderr, "[LANCIUS CUDA] %s: %s\n", what, n.error_string ? n.error_string(r) : "nccl error");
    lancius_set_error(LANCIUS_ERROR_INTERNAL);
    return LANCIUS_ERROR_INTERNAL;
}

// gathered [g][M][ns] -> C [M][g*ns]
__global__ void k_repack(float* __restrict__ c, const float* __restrict__ gathered, int g, size_t M, size_t ns) {
    const size_t N = (size_t)g * ns, total = M * N;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        size_t m = i / N, col = i % N, r = col / ns, cc = col % ns;
        c[i] = gathered[(r * M + m) * ns + cc];
    }
}
__global__ void k_repack_v4(float4* __restrict__ c, const float4* __restrict__ gathered, int g, size_t M, size_t ns4) {
    const size_t N4 = (size_t)g * ns4, total = M * N4;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        size_t m = i / N4, col = i % N4, r = col / ns4, cc = col % ns4;
        c[i] = gathered[(r * M + m) * ns4 + cc];
    }
}

}  // namespace

struct lcu_comm {
    ncclComm_t comm;
    int nranks, rank, device;
};

extern "C" lancius_error lcu_comm_unique_id(void* out, size_t bytes) {
    if (!out || bytes < NCCL_UNIQUE_ID_BYTES) { lancius_set_error(LANCIUS_ERROR_NULL_PTR); return LANCIUS_ERROR_NULL_PTR; }
    if (!nccl().ok) { lancius_set_error(LANCIUS_ERROR_UNSUPPORTED_OP); return LANCIUS_ERROR_UNSUPPORTED_OP; }
    ncclUniqueId id;
    ncclResult_t r = nccl().get_unique_id(&id);
    if (r != ncclSuccess) return nccl_fail(r, "ncclGetUniqueId");
    memcpy(out, &id, NCCL_UNIQUE_ID_BYTES);
    return LANCIUS_ERROR_OK;
}

extern "C" lcu_comm* lcu_comm_create(int nranks, int rank, const void* unique_id, int device) {
    if (!unique_id || nranks <= 0 || rank < 0 || rank >= nranks) { lancius_set_error(LANCIUS_ERROR_NULL_PTR); return nullptr; }
    if (!nccl().ok) { lancius_set_error(LANCIUS_ERROR_UNSUPPORTED_OP); return nullptr; }
    if (cudaSetDevice(device) != cudaSuccess) { cudaGetLastError(); lancius_set_error(LANCIUS_ERROR_INTERNAL); return nullptr; }
    lcu_comm* c = new (std::nothrow) lcu_comm();
    if (!c) { lancius_set_error(LANCIUS_ERROR_OOM); return nullptr; }
    ncclUniqueId id;
    memcpy(&id, unique_id, NCCL_UNIQUE_ID_BYTES);
    ncclResult_t r = nccl().comm_init_rank(&c->comm, nranks, id, rank);
    if (r != ncclSuccess) { nccl_fail(r, "ncclCommInitRank"); delete c; return nullptr; }
    c->nranks = nranks; c->rank = rank; c->device = device;
    return c;
}

extern "C" void lcu_comm_destroy(lcu_comm* c) {
    if (!c) return;
    nccl().comm_destroy(c->comm);
    delete c;
}

// Ends a communicator whose peers may be gone (failure path): in-flight collectives
// return with an error instead of waiting forever.
extern "C" void lcu_comm_abort(lcu_comm* c) {
    if (!c) return;
    nccl().comm_abort(c->comm);
    delete c;
}

extern "C" int lcu_comm_size(const lcu_comm* c) { return c ? c->nranks : 0; }

// C [M, N] (row-major, every rank) = A [M, K] * B, B split by columns: this rank
// passes its slab b_slab [K, N / nranks] (row-major). N % nranks == 0.
extern "C" lancius_error lcu_gemm_colsplit(lcu_comm* comm, float* c, const float* a, const float* b_slab, size_t M,
                                          size_t K, size_t N, int mode, void* stream) {
    if (!comm || !c || !a || !b_slab) { lancius_set_error(LANCIUS_ERROR_NULL_PTR); return LANCIUS_ERROR_NULL_PTR; }
    const int g = comm->nranks;
    if (N % (size_t)g) { lancius_set_error(LANCIUS_ERROR_SHAPE_MISMATCH); return LANCIUS_ERROR_SHAPE_MISMATCH; }
    const size_t ns = N / g;
    // local block and gathered blocks live in the per-device scratch cache: [g][M][ns]
    float* gathered = static_cast<float*>(lcu_scratch_acquire_gather((size_t)g * M * ns * sizeof(float)));
    if (!gathered) { lancius_set_error(LANCIUS_ERROR_OOM); return LANCIUS_ERROR_OOM; }
    float* mine = gathered + (size_t)comm->rank * M * ns;
    lancius_error e = lcu_matmul(mine, a, b_slab, M, K, ns, nullptr, LCU_EPI_NONE, mode, stream);
    if (e != LANCIUS_ERROR_OK) return e;
    cudaStream_t st = lcu_as_stream(stream);
    if (g > 1) {
        ncclResult_t r = nccl().all_gather(mine, gathered, M * ns, ncclFloat32, comm->comm, st);
        if (r != ncclSuccess) return nccl_fail(r, "ncclAllGather");
    }
    if (ns % 4 == 0 && ((uintptr_t)c & 15) == 0)
        k_repack_v4<<<lcu_blocks(M * N / 4, 256 * 4), 256, 0, st>>>((float4*)c, (const float4*)gathered, g, M, ns / 4);
    else
        k_repack<<<lcu_blocks(M * N, 256 * 4), 256, 0, st>>>(c, gathered, g, M, ns);
    lcu_note_launch();
    return lcu_launch_status();
}
