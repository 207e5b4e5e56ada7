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
    // fused path: every rank's C, opened through CUDA IPC for the C pointer last used
    float* c_key = nullptr;             // this rank's C those pointers belong to
    size_t c_bytes = 0;
    float* peer_c[8] = {};              // peer_c[r] = rank r's C (this rank's own at [rank])
    void* peer_base[8] = {};            // IPC mappings to close
    void* dev_buf = nullptr;            // small device buffer for handle exchange and the barrier
    unsigned char opened[8 * 128] = {}; // the gathered C records the peer mappings were opened from
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

static void close_peers(lcu_comm* c) {
    for (int r = 0; r < 8; r++) {
        if (c->peer_base[r]) cudaIpcCloseMemHandle(c->peer_base[r]);
        c->peer_base[r] = nullptr;
        c->peer_c[r] = nullptr;
    }
    c->c_key = nullptr;
    c->c_bytes = 0;
    memset(c->opened, 0, sizeof(c->opened));
}

extern "C" void lcu_comm_destroy(lcu_comm* c) {
    if (!c) return;
    cudaSetDevice(c->device);
    close_peers(c);
    if (c->dev_buf) cudaFree(c->dev_buf);
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

// ---------------------------------------------------------------------------
// Fused variant: the GEMM's epilogue stores each finished tile of this rank's column
// slab straight into every rank's row-major C over NVLink (peer pointers opened with
// CUDA IPC once per C buffer), so there is no NCCL data movement and no repack; one
// 4-byte ncclAllGather afterwards is the barrier that tells each rank its C is complete.

namespace {
typedef CUresult (*GetRangeFn)(CUdeviceptr*, size_t*, CUdeviceptr);
GetRangeFn get_range_fn() {
    static GetRangeFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<GetRangeFn>(p);
    });
    return fn;
}
struct PeerRecord {               // what each rank publishes about its C, every call
    cudaIpcMemHandle_t handle;    // of the allocation that contains C
    uint64_t offset;              // C - allocation base
    uint64_t usable;              // allocation bytes from C on
    uint64_t c;                   // C's address in the publishing process
    uint64_t bytes;               // bytes this call writes into every C
    uint64_t pad[4];
};
static_assert(sizeof(PeerRecord) % 16 == 0 && sizeof(PeerRecord) <= 128, "record size (lcu_comm::opened)");
}  // namespace

// Makes every rank's C reachable for this call. Collective on every call: each rank
// publishes its C's IPC handle, offset and size, the records are all-gathered, and
// every rank reopens its peer mappings when ANY rank's record differs from the one
// it last opened -- all ranks see the same gathered records, so all take the same
// branch, and a buffer freed and reallocated (a new IPC handle) is never used through
// a stale mapping. The all-gather also orders the call: no rank's GEMM (queued after
// it on the stream) starts before every rank's stream has reached this point, so the
// peer stores cannot overtake work queued earlier on the ranks' streams (e.g. a
// kernel still reading C from the previous call).
static lancius_error open_peers(lcu_comm* comm, float* c, size_t bytes, cudaStream_t st) {
    GetRangeFn range = get_range_fn();
    if (!range) { lancius_set_error(LANCIUS_ERROR_UNSUPPORTED_OP); return LANCIUS_ERROR_UNSUPPORTED_OP; }
    const int g = comm->nranks;
    if (!comm->dev_buf && cudaMalloc(&comm->dev_buf, 8 * sizeof(PeerRecord) + 256) != cudaSuccess) {
        cudaGetLastError(); lancius_set_error(LANCIUS_ERROR_OOM); return LANCIUS_ERROR_OOM;
    }
    CUdeviceptr base = 0;
    size_t size = 0;
    if (range(&base, &size, (CUdeviceptr)c) != CUDA_SUCCESS) { lancius_set_error(LANCIUS_ERROR_INTERNAL); return LANCIUS_ERROR_INTERNAL; }
    PeerRecord mine{};
    if (cudaIpcGetMemHandle(&mine.handle, (void*)base) != cudaSuccess) { cudaGetLastError(); lancius_set_error(LANCIUS_ERROR_INTERNAL); return LANCIUS_ERROR_INTERNAL; }
    mine.offset = (uint64_t)((CUdeviceptr)c - base);
    mine.usable = (uint64_t)(size - mine.offset);
    mine.c = (uint64_t)(uintptr_t)c;
    mine.bytes = bytes;
    PeerRecord all[8];
    char* d = static_cast<char*>(comm->dev_buf);
    if (cudaMemcpyAsync(d + comm->rank * sizeof(PeerRecord), &mine, sizeof(PeerRecord), cudaMemcpyHostToDevice, st) != cudaSuccess)
        return lcu_check_cuda(cudaGetLastError());
    ncclResult_t r = nccl().all_gather(d + comm->rank * sizeof(PeerRecord), d, sizeof(PeerRecord), ncclInt8, comm->comm, st);
    if (r != ncclSuccess) return nccl_fail(r, "ncclAllGather (C records)");
    if (cudaMemcpyAsync(all, d, g * sizeof(PeerRecord), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess)
        return lcu_check_cuda(cudaGetLastError());
    for (int k = 0; k < g; k++)
        if (all[k].usable < bytes || all[k].bytes != bytes) {   // every rank fails the same way
            close_peers(comm); lancius_set_error(LANCIUS_ERROR_SHAPE_MISMATCH); return LANCIUS_ERROR_SHAPE_MISMATCH;
        }
    if (comm->c_key == c && memcmp(comm->opened, all, g * sizeof(PeerRecord)) == 0) return LANCIUS_ERROR_OK;
    close_peers(comm);
    for (int k = 0; k < g; k++) {
        if (k == comm->rank) { comm->peer_c[k] = c; continue; }
        void* p = nullptr;
        if (cudaIpcOpenMemHandle(&p, all[k].handle, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
            cudaGetLastError(); close_peers(comm); lancius_set_error(LANCIUS_ERROR_INTERNAL); return LANCIUS_ERROR_INTERNAL;
        }
        comm->peer_base[k] = p;
        comm->peer_c[k] = reinterpret_cast<float*>(static_cast<char*>(p) + all[k].offset);
    }
    memcpy(comm->opened, all, g * sizeof(PeerRecord));
    comm->c_key = c;
    comm->c_bytes = bytes;
    return LANCIUS_ERROR_OK;
}

extern "C" lancius_error lcu_gemm_colsplit_fused(lcu_comm* comm, float* c, const float* a, const float* b_slab, size_t M,
                                                size_t K, size_t N, int mode, void* stream) {
    if (!comm || !c || !a || !b_slab) { lancius_set_error(LANCIUS_ERROR_NULL_PTR); return LANCIUS_ERROR_NULL_PTR; }
    const int g = comm->nranks;
    if (g > 8 || N % (size_t)g || M == 0 || K == 0 || ((uintptr_t)c & 15)) {
        lancius_set_error(LANCIUS_ERROR_SHAPE_MISMATCH); return LANCIUS_ERROR_SHAPE_MISMATCH;
    }
    if (mode != LCU_MODE_FP32_EXACT && mode != LCU_MODE_TF32) { lancius_set_error(LANCIUS_ERROR_UNSUPPORTED_DTYPE); return LANCIUS_ERROR_UNSUPPORTED_DTYPE; }
    const size_t ns = N / g;
    cudaStream_t st = lcu_as_stream(stream);
    lancius_error e = open_peers(comm, c, M * N * sizeof(float), st);
    if (e != LANCIUS_ERROR_OK) return e;
    const int passes = mode == LCU_MODE_TF32 ? 1 : 3;
    const size_t need = lcu_gemm_tc_scratch_bytes(M, ns, K, 1, 1, 1, passes) + 256;
    char* scratch = static_cast<char*>(lcu_scratch_acquire(need));
    if (!scratch) { lancius_set_error(LANCIUS_ERROR_OOM); return LANCIUS_ERROR_OOM; }
    LcuGemmGroup* d_group = reinterpret_cast<LcuGemmGroup*>(scratch + need - 256);
    LcuGemmGroup h{a, b_slab, comm->peer_c[comm->rank], nullptr, nullptr};
    cudaError_t ce = cudaMemcpyAsync(d_group, &h, sizeof(h), cudaMemcpyHostToDevice, st);
    if (ce != cudaSuccess) return lcu_check_cuda(ce);
    LcuTcGemmPlan p;
    e = lcu_gemm_tc_prepare(&p, scratch, M, ns, K, 1, 1, 1, passes);
    if (e != LANCIUS_ERROR_OK) return e;
    LcuColDest dst{};
    for (int k = 0; k < g; k++) dst.ptr[k] = comm->peer_c[k];
    dst.n_dst = g;
    dst.ldc = N;
    dst.col_off = (size_t)comm->rank * ns;
    e = lcu_gemm_tc_run_dst(&p, d_group, LCU_EPI_NONE, dst, stream);
    if (e != LANCIUS_ERROR_OK) return e;
    if (g > 1) {   // barrier: completes once every rank's kernels (and their peer stores) are done
        char* d = static_cast<char*>(comm->dev_buf) + 8 * sizeof(PeerRecord);
        ncclResult_t r = nccl().all_gather(d + comm->rank * 4, d, 4, ncclInt8, comm->comm, st);
        if (r != ncclSuccess) return nccl_fail(r, "ncclAllGather (barrier)");
    }
    // the host record of the group table must stay valid until the copy ran
    return lcu_check_stream(st);
}
