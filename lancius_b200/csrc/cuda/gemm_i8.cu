// INT8 mixed-precision MATMUL / CONV2D on the tcgen05 tensor cores (kind::i8).
// Restates the reference's dynamic-quantisation path (lancius_scheduler.c:195-220,
// lancius_vision_ops.c:16-57): scale_a = max|a| / 127 (1e-8 when a == 0), a_q =
// (int8)round(a / scale_a), int8 x int8 products summed exactly in int32, result =
// (double)sum * scale_a * scale_w. Integer accumulation is exact, so this path and
// the CUDA-core one give bit-identical results; the dispatcher picks by size.
//
//   1. max |a| over the activation (grid-stride, atomicMax on the float bits)
//   2. quantise a into K-major int8 rows with a 16-byte pitch (MATMUL: [M][Kp];
//      CONV: the im2col matrix [N*Ho*Wo][Kp]); MATMUL weights [K][N] are transposed
//      to [N][Kp], CONV weights [Co][K] are used as they are (or re-pitched)
//   3. D[M][N] = A[M][Kp] . B[N][Kp]^T: TMA (128-byte swizzle) -> 4-stage ring ->
//      tcgen05.mma kind::i8 (M=128, N=256, K=32 per instruction) into two int32 TMEM
//      accumulators (256 x 256 CTA tile: the B tile is read once for both row halves); warp 0 lane 0 loads, warp 1 lane 0 issues, all four warps run
//      the epilogue (tcgen05.ld -> scale -> ReLU -> row-major or NCHW store).
// Every mbarrier wait is bounded; a timeout sets the watchdog word and unwinds.
#include "tc_common.cuh"
#include <mutex>
#include <vector>

namespace {

constexpr int BM = 256, BN = 256, BK = 128, STAGES = 3, THREADS = 128;
constexpr int A_TILE = BM * BK;                    // 32 KB (two 128-row halves)
constexpr int B_TILE = BN * BK;                    // 32 KB
constexpr int STAGE_BYTES = A_TILE + B_TILE;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 + 256;
constexpr uint32_t TMEM_COLS = 2 * BN;             // two 128 x 256 int32 accumulators (rows 0-127, 128-255)

__device__ int g_i8_watchdog = 0;

struct Smem {
    uint64_t full[STAGES], empty[STAGES], accum, drain;
    uint32_t tmem;
    int abort, consumed;
};

__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(acc)
        : "memory");
}
// instruction descriptor: D = S32, A = B = signed 8-bit, both K-major
__host__ __device__ constexpr uint32_t idesc_s8(int M, int N) {
    return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ double act_scale(const float* amax, double scale_w) {
    const double sa = amax[0] > 0.f ? (double)amax[0] / 127.0 : 1e-8;
    return sa * scale_w;
}

__global__ void __launch_bounds__(THREADS, 1)
k_gemm_i8(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tb, float* __restrict__ out,
          const float* __restrict__ amax, double scale_w, int M, int N, int Kp, int relu, int conv_hw) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* tiles = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    Smem* sm = reinterpret_cast<Smem*>(tiles + STAGES * STAGE_BYTES);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
    const int KT = (Kp + BK - 1) / BK;
    volatile int* abort = &sm->abort;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) { tc::mbar_init(&sm->full[s], 1); tc::mbar_init(&sm->empty[s], 1); }
        tc::mbar_init(&sm->accum, 1);
        tc::mbar_init(&sm->drain, 1);
        sm->abort = 0;
        sm->consumed = 0;
        tc::fence_barrier_init();
        tc::prefetch_tmap(&ta); tc::prefetch_tmap(&tb);
    }
    if (warp == 1) tc::tmem_alloc(&sm->tmem, TMEM_COLS);
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = sm->tmem;
    int issued = 0;

    if (warp == 0 && lane == 0) {
        for (int kt = 0; kt < KT; kt++) {
            const int s = kt % STAGES;
            if (kt >= STAGES && !tc::mbar_wait(&sm->empty[s], ((kt / STAGES) - 1) & 1, abort, &g_i8_watchdog, 1)) break;
            uint8_t* st = tiles + s * STAGE_BYTES;
            tc::mbar_expect_tx(&sm->full[s], STAGE_BYTES);
            tc::tma_load_3d(st, &ta, &sm->full[s], kt * BK, m0, 0);
            tc::tma_load_3d(st + A_TILE, &tb, &sm->full[s], kt * BK, n0, 0);
            issued = kt + 1;
        }
    } else if (warp == 1 && lane == 0) {
        constexpr uint32_t idesc = idesc_s8(128, BN);
        bool ok = true;
        for (int kt = 0; kt < KT; kt++) {
            const int s = kt % STAGES;
            if (!tc::mbar_wait(&sm->full[s], (kt / STAGES) & 1, abort, &g_i8_watchdog, 2)) { ok = false; break; }
            tc::tc_fence_after();
            const uint32_t a = tc::smem_u32(tiles + s * STAGE_BYTES), b = a + A_TILE;
#pragma unroll
            for (int kk = 0; kk < BK / 32; kk++) {   // 32 int8 = 32 bytes of K per instruction
                const uint64_t db = tc::smem_desc(b + kk * 32, 16, 1024, tc::SWZ_128B);
#pragma unroll
                for (int half = 0; half < 2; half++)   // both row halves share the B tile
                    mma_i8(tmem + (uint32_t)half * BN, tc::smem_desc(a + half * (128 * BK) + kk * 32, 16, 1024, tc::SWZ_128B),
                           db, idesc, (kt | kk) ? 1u : 0u);
            }
            tc::mma_commit(&sm->empty[s]);
            sm->consumed = kt + 1;
        }
        if (ok) tc::mma_commit(&sm->accum);
    }
    __syncwarp();
    // epilogue: every warp reads its 32 TMEM lanes (= rows), stages each 32x32 int32 block
    // in the drained pipeline smem and stores it by rows (lane j: column j), coalesced
    if (tc::mbar_wait(&sm->accum, 0, abort, &g_i8_watchdog, 3)) {
        tc::tc_fence_after();
        const double scale = act_scale(amax, scale_w);
        int* sb = reinterpret_cast<int*>(tiles) + (size_t)warp * 32 * 33;
        for (int half = 0; half < 2; half++) {
            const int row0 = m0 + half * 128 + 32 * warp;
            if (m0 + half * 128 >= M) break;                   // warp-uniform
            for (int c = 0; c < BN; c += 32) {
                if (n0 + c >= N) break;                        // warp-uniform
                float v[32];
                tc::tmem_ld32(tmem + ((uint32_t)(32 * warp) << 16) + (uint32_t)(half * BN + c), v);
#pragma unroll
                for (int j = 0; j < 32; j++) sb[lane * 33 + j] = __float_as_int(v[j]);
                __syncwarp();
                const int col = n0 + c + lane;
                if (col < N) {
#pragma unroll 4
                    for (int r = 0; r < 32; r++) {
                        const int row = row0 + r;
                        if (row >= M) break;
                        float x = (float)((double)sb[r * 33 + lane] * scale);
                        if (relu && x < 0.f) x = 0.f;
                        if (conv_hw) out[(size_t)(col / conv_hw) * M * conv_hw + (size_t)row * conv_hw + col % conv_hw] = x;
                        else out[(size_t)row * N + col] = x;
                    }
                }
                __syncwarp();
            }
        }
    }

    tc::tc_fence_before();
    __syncthreads();
    if (sm->abort) {
        int never = 0;
        if (warp == 0 && lane == 0)
            for (int kt = sm->consumed; kt < issued; kt++)
                if (!tc::mbar_wait(&sm->full[kt % STAGES], (kt / STAGES) & 1, &never, nullptr, 0)) break;
        if (warp == 1 && lane == 0) {
            tc::mma_commit(&sm->drain);
            tc::mbar_wait(&sm->drain, 0, &never, nullptr, 0);
        }
        __syncthreads();
    }
    if (warp == 1) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem, TMEM_COLS);
    }
}

// max |a| as float bits (non-negative floats order like their bit patterns)
__global__ void k_absmax_bits(unsigned* out, const float* __restrict__ a, size_t n) {
    float m = 0.f;
    const size_t tid = blockIdx.x * (size_t)blockDim.x + threadIdx.x, nth = (size_t)gridDim.x * blockDim.x;
    if ((reinterpret_cast<uintptr_t>(a) & 15) == 0) {
        const float4* a4 = reinterpret_cast<const float4*>(a);
        for (size_t i = tid; i < n / 4; i += nth) {
            const float4 v = __ldg(a4 + i);
            m = fmaxf(m, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
        }
        for (size_t i = n / 4 * 4 + tid; i < n; i += nth) m = fmaxf(m, fabsf(a[i]));
    } else {
        for (size_t i = tid; i < n; i += nth) m = fmaxf(m, fabsf(a[i]));
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    if ((threadIdx.x & 31) == 0 && m > 0.f) atomicMax(out, __float_as_uint(m));
}

struct QScale { double sa, inv; };
__device__ __forceinline__ QScale qscale(const float* amax) {
    const double sa = amax[0] > 0.f ? (double)amax[0] / 127.0 : 1e-8;
    return {sa, 1.0 / sa};
}
// (int8)round(x / scale_a) exactly as the reference computes it (a double division,
// round half away from zero). x * (1 / scale_a) is within a few ulp of the quotient,
// which only matters next to a half-integer; there the division is redone.
__device__ __forceinline__ int8_t quant8(float x, QScale q) {
    double y = (double)x * q.inv;
    const double f = fabs(y - trunc(y));
    if (fabs(f - 0.5) < 1e-9) y = (double)x / q.sa;
    return (int8_t)(int)round(y);
}

// a [M][K] fp32 -> [M][Kp] int8, zero padded; four bytes per thread
__global__ void k_quant_rows(int8_t* __restrict__ dst, const float* __restrict__ a, const float* __restrict__ amax,
                             size_t M, size_t K, size_t Kp) {
    const QScale q = qscale(amax);
    const size_t words = M * Kp / 4;
    const bool vec = K % 4 == 0 && (reinterpret_cast<uintptr_t>(a) & 15) == 0;
    for (size_t w = blockIdx.x * (size_t)blockDim.x + threadIdx.x; w < words; w += (size_t)gridDim.x * blockDim.x) {
        const size_t m = (w * 4) / Kp, k0 = (w * 4) % Kp;
        char4 r;
        if (vec) {
            float4 v = k0 < K ? __ldg(reinterpret_cast<const float4*>(a + m * K + k0)) : make_float4(0.f, 0.f, 0.f, 0.f);
            r = make_char4(quant8(v.x, q), quant8(v.y, q), quant8(v.z, q), quant8(v.w, q));
        } else {
            int8_t* rb = reinterpret_cast<int8_t*>(&r);
#pragma unroll
            for (int t = 0; t < 4; t++) rb[t] = k0 + t < K ? quant8(a[m * K + k0 + t], q) : (int8_t)0;
        }
        reinterpret_cast<char4*>(dst)[w] = r;
    }
}

// im2col of the quantised NCHW input: [P = N*Ho*Wo][Kp] int8, k = (ci, kh, kw)
__global__ void k_im2col_q(int8_t* __restrict__ dst, const float* __restrict__ in, const float* __restrict__ amax,
                           LcuConvShape cs, size_t Kp) {
    const int K = cs.ci * cs.kh * cs.kw, hw = cs.ho * cs.wo;
    const QScale qs = qscale(amax);
    const size_t words = (size_t)cs.n * hw * Kp / 4;
    for (size_t w = blockIdx.x * (size_t)blockDim.x + threadIdx.x; w < words; w += (size_t)gridDim.x * blockDim.x) {
        const size_t p = (w * 4) / Kp;
        const int k0 = (int)((w * 4) % Kp);
        const int n = (int)(p / hw), r = (int)(p % hw), ho = r / cs.wo, wo = r % cs.wo;
        char4 q;
        int8_t* qb = reinterpret_cast<int8_t*>(&q);
#pragma unroll
        for (int t = 0; t < 4; t++) {
            const int k = k0 + t;
            int8_t v = 0;
            if (k < K) {
                const int kw = k % cs.kw, kh = (k / cs.kw) % cs.kh, ci = k / (cs.kw * cs.kh);
                const int ih = ho * cs.stride - cs.pad + kh, iw = wo * cs.stride - cs.pad + kw;
                // zero padding quantises to 0 (round(0 / scale) = 0)
                if (ih >= 0 && iw >= 0 && ih < cs.h && iw < cs.w)
                    v = quant8(in[(((size_t)n * cs.ci + ci) * cs.h + ih) * (size_t)cs.w + iw], qs);
            }
            qb[t] = v;
        }
        reinterpret_cast<char4*>(dst)[w] = q;
    }
}

// b [K][N] int8 -> [N][Kp] int8, zero padded: 64 x 64 byte tiles through shared
// memory, 4-byte words on both sides
__global__ void __launch_bounds__(256) k_transpose_i8(int8_t* __restrict__ dst, const int8_t* __restrict__ b, size_t K,
                                                      size_t N, size_t Kp) {
    __shared__ int8_t t[64][68];
    const size_t k0 = blockIdx.y * 64, n0 = blockIdx.x * 64;
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;     // 16 words x 16 rows per pass
    const bool vec_in = N % 4 == 0 && (reinterpret_cast<uintptr_t>(b) & 3) == 0;
    for (int i = ty; i < 64; i += 16) {
        const size_t k = k0 + i, n = n0 + 4 * tx;
        char4 v = make_char4(0, 0, 0, 0);
        if (k < K) {
            if (vec_in && n + 3 < N) v = *reinterpret_cast<const char4*>(b + k * N + n);
            else {
                int8_t* vb = reinterpret_cast<int8_t*>(&v);
                for (int u = 0; u < 4; u++) vb[u] = n + u < N ? b[k * N + n + u] : (int8_t)0;
            }
        }
        *reinterpret_cast<char4*>(&t[i][4 * tx]) = v;
    }
    __syncthreads();
    for (int i = ty; i < 64; i += 16) {
        const size_t n = n0 + i, k = k0 + 4 * tx;
        if (n >= N || k >= Kp) continue;
        const char4 v = make_char4(t[4 * tx][i], t[4 * tx + 1][i], t[4 * tx + 2][i], t[4 * tx + 3][i]);
        *reinterpret_cast<char4*>(dst + n * Kp + k) = v;   // Kp % 16 == 0: whole words stay in the row
    }
}

// [R][K] int8 -> [R][Kp] int8, zero padded
__global__ void k_repitch_i8(int8_t* __restrict__ dst, const int8_t* __restrict__ src, size_t R, size_t K, size_t Kp) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < R * Kp; i += (size_t)gridDim.x * blockDim.x) {
        const size_t r = i / Kp, k = i % Kp;
        dst[i] = k < K ? src[r * K + k] : (int8_t)0;
    }
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

// [rows][Kp] int8, box {BK, box_rows}, 128-byte swizzle (out-of-range reads are zero)
bool make_map_i8(CUtensorMap* m, const int8_t* base, size_t Kp, size_t rows, uint32_t box_rows) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[3] = {Kp, rows, 1};
    cuuint64_t strides[2] = {Kp, rows * Kp};
    cuuint32_t box[3] = {(cuuint32_t)BK, box_rows, 1};
    cuuint32_t es[3] = {1, 1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<int8_t*>(base), dims, strides, box, es,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

size_t pad16(size_t v) { return (v + 15) & ~size_t(15); }
size_t al256(size_t v) { return (v + 255) & ~size_t(255); }

bool configure() {
    static bool done[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && done[dev]) return true;
    if (cudaFuncSetAttribute(k_gemm_i8, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES) != cudaSuccess)
        return false;
    if (dev >= 0 && dev < 64) done[dev] = true;
    return true;
}

lancius_error absmax(float* amax, const float* a, size_t n, cudaStream_t st) {
    cudaError_t ce = cudaMemsetAsync(amax, 0, sizeof(float), st);
    if (ce != cudaSuccess) return lcu_check_cuda(ce);
    k_absmax_bits<<<lcu_blocks(n, 256, 148u * 8u), 256, 0, st>>>(reinterpret_cast<unsigned*>(amax), a, n);
    lcu_note_launch();
    return lcu_launch_status();
}

lancius_error run_gemm(const int8_t* a8, const int8_t* b8, float* out, const float* amax, double scale_w, size_t M,
                       size_t N, size_t Kp, int relu, int conv_hw, cudaStream_t st) {
    CUtensorMap ta, tb;
    if (!configure() || !make_map_i8(&ta, a8, Kp, M, BM) || !make_map_i8(&tb, b8, Kp, N, BN)) {
        lancius_set_error(LANCIUS_ERROR_INTERNAL);
        return LANCIUS_ERROR_INTERNAL;
    }
    dim3 grid((unsigned)((N + BN - 1) / BN), (unsigned)((M + BM - 1) / BM));
    k_gemm_i8<<<grid, THREADS, SMEM_BYTES, st>>>(ta, tb, out, amax, scale_w, (int)M, (int)N, (int)Kp, relu, conv_hw);
    lcu_note_launch();
    return lcu_launch_status();
}

std::mutex g_mu;
std::vector<std::pair<void*, size_t>> g_cache;   // per-device scratch for the per-op calls

void* per_op_scratch(size_t bytes) {
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lk(g_mu);
    if ((int)g_cache.size() <= dev) g_cache.resize(dev + 1, {nullptr, 0});
    auto& c = g_cache[dev];
    if (c.second < bytes) {
        if (c.first) { cudaDeviceSynchronize(); cudaFree(c.first); c = {nullptr, 0}; }
        if (cudaMalloc(&c.first, bytes) != cudaSuccess) { cudaGetLastError(); return nullptr; }
        c.second = bytes;
    }
    return c.first;
}

}  // namespace

extern "C" {

// Tensor-core INT8 path taken for products of at least 2^24 multiply-adds.
int lcu_int8_use_tc(size_t M, size_t N, size_t K) { return lcu_use_tensor_cores(M, N, K) && M >= 64 && N >= 64; }

size_t lcu_matmul_int8_scratch_bytes(size_t M, size_t K, size_t N) {
    if (!lcu_int8_use_tc(M, N, K)) return 0;
    return al256(M * pad16(K)) + al256(N * pad16(K));
}
size_t lcu_conv2d_int8_scratch_bytes(size_t N, size_t Ci, size_t H, size_t W, size_t Co, size_t Kh, size_t Kw,
                                     size_t stride, size_t pad) {
    if (!stride || H + 2 * pad < Kh || W + 2 * pad < Kw) return 0;
    const size_t Ho = (H + 2 * pad - Kh) / stride + 1, Wo = (W + 2 * pad - Kw) / stride + 1;
    const size_t K = Ci * Kh * Kw, P = N * Ho * Wo;
    if (!lcu_int8_use_tc(Co, P, K)) return 0;
    return al256(P * pad16(K)) + al256(Co * pad16(K));   // im2col + (if needed) re-pitched weights
}

// scratch: lcu_matmul_int8_scratch_bytes() bytes of device memory, or NULL for a
// library-owned per-device buffer (then the call synchronises the stream before it
// returns, so the buffer can be reused by the next call).
// B [K][N] int8 -> K-major [N][Kp] rows (Kp = K rounded up to 16), the tensor-core
// layout of the weights; the executor runs it when an INT8 weight is uploaded.
lancius_error lcu_int8_pack_kmajor(int8_t* dst, const int8_t* b, size_t K, size_t N, size_t Kp, void* s) {
    if (!K || !N) return LANCIUS_ERROR_OK;
    k_transpose_i8<<<dim3((unsigned)((N + 63) / 64), (unsigned)((Kp + 63) / 64)), 256, 0, lcu_as_stream(s)>>>(dst, b, K, N,
                                                                                                            Kp);
    lcu_note_launch();
    return lcu_launch_status();
}

lancius_error lcu_matmul_int8(float* out, const float* a, const int8_t* b, double scale_b, size_t M, size_t K, size_t N,
                              const int8_t* b_packed, float* amax_scratch, void* scratch, void* s) {
    if (!out || !a || !b || !amax_scratch) { lancius_set_error(LANCIUS_ERROR_NULL_PTR); return LANCIUS_ERROR_NULL_PTR; }
    const size_t need = lcu_matmul_int8_scratch_bytes(M, K, N);
    if (!need) return lcu_matmul_int8_simt(out, a, b, scale_b, M, K, N, amax_scratch, s);
    const bool own = scratch == nullptr;
    if (own && !(scratch = per_op_scratch(need))) { lancius_set_error(LANCIUS_ERROR_OOM); return LANCIUS_ERROR_OOM; }
    cudaStream_t st = lcu_as_stream(s);
    const size_t Kp = pad16(K);
    int8_t* a8 = static_cast<int8_t*>(scratch);
    int8_t* b8 = a8 + al256(M * Kp);
    lancius_error e = absmax(amax_scratch, a, M * K, st);
    if (e != LANCIUS_ERROR_OK) return e;
    k_quant_rows<<<lcu_blocks(M * Kp / 4, 256, 148u * 16u), 256, 0, st>>>(a8, a, amax_scratch, M, K, Kp);
    lcu_note_launch();
    if (b_packed) b8 = const_cast<int8_t*>(b_packed);
    else if ((e = lcu_int8_pack_kmajor(b8, b, K, N, Kp, s)) != LANCIUS_ERROR_OK) return e;
    if ((e = lcu_launch_status()) != LANCIUS_ERROR_OK) return e;
    e = run_gemm(a8, b8, out, amax_scratch, scale_b, M, N, Kp, 0, 0, st);
    if (e == LANCIUS_ERROR_OK && own) e = lcu_check_stream(st);
    return e;
}

lancius_error lcu_conv2d_int8(float* out, const float* in, const int8_t* w, double scale_w, size_t N, size_t Ci, size_t H,
                              size_t W, size_t Co, size_t Kh, size_t Kw, size_t stride, size_t pad, int relu,
                              float* amax_scratch, void* scratch, void* s) {
    if (!out || !in || !w || !amax_scratch) { lancius_set_error(LANCIUS_ERROR_NULL_PTR); return LANCIUS_ERROR_NULL_PTR; }
    const size_t need = lcu_conv2d_int8_scratch_bytes(N, Ci, H, W, Co, Kh, Kw, stride, pad);
    if (!need)
        return lcu_conv2d_int8_simt(out, in, w, scale_w, N, Ci, H, W, Co, Kh, Kw, stride, pad, relu, amax_scratch, s);
    const bool own = scratch == nullptr;
    if (own && !(scratch = per_op_scratch(need))) { lancius_set_error(LANCIUS_ERROR_OOM); return LANCIUS_ERROR_OOM; }
    cudaStream_t st = lcu_as_stream(s);
    const size_t Ho = (H + 2 * pad - Kh) / stride + 1, Wo = (W + 2 * pad - Kw) / stride + 1;
    const size_t K = Ci * Kh * Kw, Kp = pad16(K), P = N * Ho * Wo;
    LcuConvShape cs{(int)N, (int)Ci, (int)H, (int)W, (int)Co, (int)Kh, (int)Kw, (int)stride, (int)pad, (int)Ho, (int)Wo};
    int8_t* b8 = static_cast<int8_t*>(scratch);
    const int8_t* a8 = w;
    lancius_error e = absmax(amax_scratch, in, N * Ci * H * W, st);
    if (e != LANCIUS_ERROR_OK) return e;
    k_im2col_q<<<lcu_blocks(P * Kp / 4, 256, 148u * 16u), 256, 0, st>>>(b8, in, amax_scratch, cs, Kp);
    lcu_note_launch();
    if (K % 16 || reinterpret_cast<uintptr_t>(w) % 16) {   // TMA rows need a 16-byte pitch and base
        int8_t* wp = b8 + al256(P * Kp);
        k_repitch_i8<<<lcu_blocks(Co * Kp, 256), 256, 0, st>>>(wp, w, Co, K, Kp);
        lcu_note_launch();
        a8 = wp;
    }
    if ((e = lcu_launch_status()) != LANCIUS_ERROR_OK) return e;
    e = run_gemm(a8, b8, out, amax_scratch, scale_w, Co, P, Kp, relu, (int)(Ho * Wo), st);
    if (e == LANCIUS_ERROR_OK && own) e = lcu_check_stream(st);
    return e;
}

int lcu_int8_watchdog_read_and_clear(void) {
    int v = 0, z = 0;
    cudaMemcpyFromSymbol(&v, g_i8_watchdog, sizeof(int));
    if (v) cudaMemcpyToSymbol(g_i8_watchdog, &z, sizeof(int));
    return v;
}

}  // extern "C"

// Device address of this file's watchdog word on the current device (0 if unavailable).
extern "C" int* lcu_int8_watchdog_addr(void) {
    void* p = nullptr;
    return cudaGetSymbolAddress(&p, g_i8_watchdog) == cudaSuccess ? static_cast<int*>(p) : nullptr;
}
