// CUDA-core FP32 GEMM and implicit-GEMM conv launchers (see gemm_simt.cuh).
#include "gemm_simt.cuh"
#include "tc_common.cuh"

#include <algorithm>

using namespace lcu_simt;

__global__ void __launch_bounds__(THREADS) k_gemm_simt(const LcuGemmGroup* __restrict__ groups, size_t M, size_t N,
                                                       size_t K, int epi) {
    LcuGemmGroup gr = groups[blockIdx.z];
    DenseA A{gr.a, M, K, K};
    DenseB B{gr.b, K, N, N};
    DenseC C{gr.c, gr.bias, gr.resid, M, N, N, epi};
    gemm_tile(A, B, C, K, (size_t)blockIdx.y * BM, (size_t)blockIdx.x * BN);
}

// Small products (the MLP's 64 x 784 x 256): a 128 x 128 tile grid would leave almost
// every SM idle, so each CTA takes a 16 x 32 output tile. K is walked in chunks of 128
// whose A (16 x 128) and B (128 x 32) tiles are copied into shared memory several chunks
// ahead; warp w accumulates k = 16w .. 16w+15 of each chunk; the eight warps' partial
// tiles are summed in a fixed order (deterministic) and the epilogue is applied as in
// DenseC.
constexpr int SK_TM = 16, SK_TN = 32, SK_WARPS = 8, SK_KC = 128;
// K chunks in flight per CTA: each chunk (A 16 x 128, B 128 x 32) is copied global ->
// shared with cp.async (4-byte copies, zero-filled past the matrix edge) SK_STAGES - 1
// chunks ahead, so a small product pays about one memory latency instead of one per chunk.
constexpr int SK_STAGES = 6;
constexpr int SK_AP = SK_KC + 4;                 // A row pitch in floats (16-byte rows for cp.async)
constexpr int SK_A_FLOATS = SK_TM * SK_AP, SK_B_FLOATS = SK_KC * SK_TN;
constexpr int SK_SMEM_BYTES = SK_STAGES * (SK_A_FLOATS + SK_B_FLOATS) * 4 + SK_WARPS * SK_TM * (SK_TN + 1) * 4;

// `src` must be a valid address even when !valid (nothing is read then; the word is zeroed)
__device__ __forceinline__ void cp_async4(float* dst, const float* src, bool valid) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)),
                 "l"(src), "r"(valid ? 4 : 0) : "memory");
}
__device__ __forceinline__ void cp_async16(float* dst, const float* src, bool valid) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)),
                 "l"(src), "r"(valid ? 16 : 0) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// One 16 x 32 output tile (rows m0.., columns n0..) of C = A B with the epilogue `epi`,
// computed by the 256 threads of the calling CTA in the dynamic shared memory.
__device__ __forceinline__ void skinny_tile(const LcuGemmGroup& gr, size_t M, size_t N, size_t K, int epi, size_t m0,
                                            size_t n0) {
    extern __shared__ float sk_smem[];
    float* As0 = sk_smem;                                          // [stage][16][129]
    float* Bs0 = sk_smem + SK_STAGES * SK_A_FLOATS;                // [stage][128][32]
    float* part = Bs0 + SK_STAGES * SK_B_FLOATS;                   // [warp][16][33]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int chunks = (int)((K + SK_KC - 1) / SK_KC);
    // 16-byte copies when every row starts 16-byte aligned (a float4 is then wholly inside
    // or wholly outside the matrix), else 4-byte ones
    const bool vec = K % 4 == 0 && N % 4 == 0 && ((reinterpret_cast<uintptr_t>(gr.a) | reinterpret_cast<uintptr_t>(gr.b)) & 15) == 0;
    auto load = [&](int kc) {                                      // chunk kc -> stage kc % SK_STAGES
        const size_t k0 = (size_t)kc * SK_KC;
        float* As = As0 + (kc % SK_STAGES) * SK_A_FLOATS;
        float* Bs = Bs0 + (kc % SK_STAGES) * SK_B_FLOATS;
        if (vec) {
#pragma unroll
            for (int r = 0; r < SK_TM * SK_KC / 4 / 256; r++) {   // A: 16 rows x 32 float4
                const int idx = threadIdx.x + 256 * r, i = idx / (SK_KC / 4), kk = 4 * (idx % (SK_KC / 4));
                const bool v = m0 + i < M && k0 + kk < K;
                cp_async16(As + i * SK_AP + kk, v ? gr.a + (m0 + i) * K + k0 + kk : gr.a, v);
            }
#pragma unroll
            for (int r = 0; r < SK_KC * SK_TN / 4 / 256; r++) {   // B: 128 k x 8 float4
                const int idx = threadIdx.x + 256 * r, kk = idx / (SK_TN / 4), j = 4 * (idx % (SK_TN / 4));
                const bool v = k0 + kk < K && n0 + j < N;
                cp_async16(Bs + kk * SK_TN + j, v ? gr.b + (k0 + kk) * N + n0 + j : gr.b, v);
            }
            return;
        }
#pragma unroll
        for (int r = 0; r < SK_TM * SK_KC / 256; r++) {           // A: 16 rows x 128 k, coalesced along k
            const int idx = threadIdx.x + 256 * r, i = idx / SK_KC, kk = idx % SK_KC;
            const bool v = m0 + i < M && k0 + kk < K;
            cp_async4(As + i * SK_AP + kk, v ? gr.a + (m0 + i) * K + k0 + kk : gr.a, v);
        }
#pragma unroll
        for (int r = 0; r < SK_KC * SK_TN / 256; r++) {           // B: 128 k x 32 n, coalesced along n
            const int idx = threadIdx.x + 256 * r, kk = idx / SK_TN, j = idx % SK_TN;
            const bool v = k0 + kk < K && n0 + j < N;
            cp_async4(Bs + kk * SK_TN + j, v ? gr.b + (k0 + kk) * N + n0 + j : gr.b, v);
        }
    };
    float acc[SK_TM];
#pragma unroll
    for (int i = 0; i < SK_TM; i++) acc[i] = 0.f;
#pragma unroll
    for (int kc = 0; kc < SK_STAGES - 1; kc++) {                   // prologue: the first chunks in flight
        if (kc < chunks) load(kc);
        cp_async_commit();
    }
    for (int kc = 0; kc < chunks; kc++) {
        cp_async_wait<SK_STAGES - 2>();                            // this thread's copies of chunk kc landed
        __syncthreads();                                           // everyone's; chunk kc - 1 is consumed
        if (kc + SK_STAGES - 1 < chunks) load(kc + SK_STAGES - 1);
        cp_async_commit();
        const float* As = As0 + (kc % SK_STAGES) * SK_A_FLOATS;
        const float* Bs = Bs0 + (kc % SK_STAGES) * SK_B_FLOATS;
#pragma unroll
        for (int kk = warp * (SK_KC / SK_WARPS); kk < (warp + 1) * (SK_KC / SK_WARPS); kk++) {
            const float b = Bs[kk * SK_TN + lane];
#pragma unroll
            for (int i = 0; i < SK_TM; i++) acc[i] = fmaf(As[i * SK_AP + kk], b, acc[i]);
        }
    }
    cp_async_wait<0>();
#pragma unroll
    for (int i = 0; i < SK_TM; i++) part[(warp * SK_TM + i) * (SK_TN + 1) + lane] = acc[i];
    __syncthreads();
    if (epi == LCU_EPI_SOFTMAX_ROW) {
        // the whole row is in this tile (N <= 32, n0 == 0): + bias, then softmax as k_softmax
        // computes it for rows of at most 32 (max, exp-sum, scale; same shuffle order)
        for (int i = warp; i < SK_TM; i += SK_WARPS) {
            const size_t m = m0 + i;
            if (m >= M) break;                                  // warp-uniform
            float v = -INFINITY;
            if (lane < (int)N) {
                v = 0.f;
#pragma unroll
                for (int w = 0; w < SK_WARPS; w++) v += part[(w * SK_TM + i) * (SK_TN + 1) + lane];
                if (gr.bias) v += __ldg(gr.bias + lane);
            }
            float mx = v;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
            float e = lane < (int)N ? expf(v - mx) : 0.f, s = e;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
            if (lane < (int)N) gr.c[m * N + lane] = expf(v - mx) * (1.f / s);
        }
        return;
    }
    const DenseC C{gr.c, gr.bias, gr.resid, M, N, N, epi};
    for (int o = threadIdx.x; o < SK_TM * SK_TN; o += blockDim.x) {
        const int i = o / SK_TN, j = o % SK_TN;
        float sum = 0.f;
#pragma unroll
        for (int w = 0; w < SK_WARPS; w++) sum += part[(w * SK_TM + i) * (SK_TN + 1) + j];
        C(m0 + i, n0 + j, sum);
    }
}

__global__ void __launch_bounds__(256) k_gemm_skinny(const LcuGemmGroup* __restrict__ groups, LcuGemmGroup one,
                                                     size_t M, size_t N, size_t K, int epi) {
    const LcuGemmGroup gr = groups ? groups[blockIdx.z] : one;
    skinny_tile(gr, M, N, K, epi, (size_t)blockIdx.y * SK_TM, (size_t)blockIdx.x * SK_TN);
}

// Two chained small products in one launch: H = epi1(A1 B1 + bias1) [M, N1], then
// Y = epi2(H B2 + bias2) [M, N2 <= 32] -- the MLP's Linear -> ReLU -> Linear -> softmax.
// Each CTA computes one 16 x 32 tile of H as k_gemm_skinny does and stores it. The CTAs of
// a 16-row block then take a ticket after a device-scope fence; the last one of the block,
// which sees every tile of those H rows, computes the block's rows of Y (one tile: all N2
// columns) and resets the ticket for the next launch on the stream. One launch, and no
// CTA ever waits for another.
__global__ void __launch_bounds__(256) k_mlp2(const LcuGemmGroup* __restrict__ l1, const LcuGemmGroup* __restrict__ l2,
                                              size_t M, size_t N1, size_t K1, int epi1, size_t N2, int epi2,
                                              unsigned* __restrict__ tickets) {
    __shared__ unsigned last;
    const size_t m0 = (size_t)blockIdx.y * SK_TM;
    {   // the second product's weights and bias into L2 now, for whichever CTA finishes last
        const LcuGemmGroup g2 = *l2;
        const size_t lines = (N1 * N2 * 4 + 127) / 128, nb = (size_t)gridDim.x * gridDim.y;
        const size_t cta = blockIdx.x + (size_t)gridDim.x * blockIdx.y;
        for (size_t i = cta * blockDim.x + threadIdx.x; i < lines; i += nb * blockDim.x)
            asm volatile("prefetch.global.L2 [%0];" ::"l"(reinterpret_cast<const char*>(g2.b) + 128 * i));
        if (g2.bias && cta == 0 && threadIdx.x == 0) asm volatile("prefetch.global.L2 [%0];" ::"l"(g2.bias));
    }
    skinny_tile(*l1, M, N1, K1, epi1, m0, (size_t)blockIdx.x * SK_TN);
    __threadfence();                     // this CTA's H tile is visible device-wide before its ticket
    __syncthreads();
    if (threadIdx.x == 0) last = atomicAdd(&tickets[blockIdx.y], 1u) == gridDim.x - 1;
    __syncthreads();
    if (!last) return;
    __threadfence();                     // ... and every other tile of the block is visible here
    skinny_tile(*l2, M, N2, N1, epi2, m0, 0);
    if (threadIdx.x == 0) tickets[blockIdx.y] = 0u;
}

static bool skinny_configured() {
    static bool done[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return false;
    if (!done[dev] &&
        cudaFuncSetAttribute(k_gemm_skinny, cudaFuncAttributeMaxDynamicSharedMemorySize, SK_SMEM_BYTES) == cudaSuccess &&
        cudaFuncSetAttribute(k_mlp2, cudaFuncAttributeMaxDynamicSharedMemorySize, SK_SMEM_BYTES) == cudaSuccess)
        done[dev] = true;
    return done[dev];
}

static bool use_skinny(size_t M, size_t N, int count) {
    const size_t tiles = ((N + BN - 1) / BN) * ((M + BM - 1) / BM) * (size_t)count;
    return tiles < 64 && M * N <= (1u << 20);
}

int lcu_mlp2_ok(size_t M, size_t N1, size_t K1, size_t N2) {
    return M > 0 && M <= 4096 && N2 > 0 && N2 <= (size_t)SK_TN && use_skinny(M, N1, 1) && !lcu_use_tensor_cores(M, N1, K1) &&
           !lcu_use_tensor_cores(M, N2, N1);
}

lancius_error lcu_mlp2(const LcuGemmGroup* d_l1, const LcuGemmGroup* d_l2, size_t M, size_t N1, size_t K1, int epi1,
                       size_t N2, int epi2, unsigned* d_tickets, void* stream) {
    if (!lcu_mlp2_ok(M, N1, K1, N2)) { lancius_set_error(LANCIUS_ERROR_INTERNAL); return LANCIUS_ERROR_INTERNAL; }
    if (!skinny_configured()) return lcu_launch_status();
    dim3 g((unsigned)((N1 + SK_TN - 1) / SK_TN), (unsigned)((M + SK_TM - 1) / SK_TM), 1);
    k_mlp2<<<g, 256, SK_SMEM_BYTES, lcu_as_stream(stream)>>>(d_l1, d_l2, M, N1, K1, epi1, N2, epi2, d_tickets);
    lcu_note_launch();
    return lcu_launch_status();
}

int lcu_gemm_softmax_fold_ok(size_t M, size_t N, size_t K) {
    return N > 0 && N <= (size_t)SK_TN && M * N <= (1u << 20) && !lcu_use_tensor_cores(M, N, K);
}

__global__ void __launch_bounds__(THREADS) k_gemm_simt1(LcuGemmGroup gr, size_t M, size_t N, size_t K, int epi) {
    DenseA A{gr.a, M, K, K};
    DenseB B{gr.b, K, N, N};
    DenseC C{gr.c, gr.bias, gr.resid, M, N, N, epi};
    gemm_tile(A, B, C, K, (size_t)blockIdx.y * BM, (size_t)blockIdx.x * BN);
}

__global__ void __launch_bounds__(THREADS) k_conv_simt(float* out, const float* in, const float* w, int N, int Ci, int H,
                                                       int W, int Co, int Kh, int Kw, int stride, int pad, int Ho,
                                                       int Wo, int relu) {
    size_t Kdim = (size_t)Ci * Kh * Kw, P = (size_t)N * Ho * Wo;
    DenseA A{w, (size_t)Co, Kdim, Kdim};
    Im2colB B{in, Ci, H, W, Kh, Kw, stride, pad, Ho, Wo, P, Kdim};
    ConvC C{out, (size_t)Co, P, (size_t)Ho * Wo, relu};
    gemm_tile(A, B, C, Kdim, (size_t)blockIdx.y * BM, (size_t)blockIdx.x * BN);
}

// Direct conv for a short reduction (Ci*Kh*Kw <= 32, e.g. an RGB input layer): each
// thread takes two output pixels (one grid stride apart, so stores stay coalesced),
// gathers their K input values (zero padding) into registers through a per-k offset
// table, and accumulates every output channel in FP32 in k order against weights
// [Co][K4*4] read from shared memory as broadcast float4s (one read feeds both
// pixels). Restates kernel_conv2d_fwd (lancius_kernels.c:28-60).
template <int K4>
__global__ void __launch_bounds__(256) k_conv_smallk(float* __restrict__ out, const float* __restrict__ in,
                                                     const float* __restrict__ w, int N, int Ci, int H, int W, int Co,
                                                     int Kh, int Kw, int stride, int pad, int Ho, int Wo, int relu) {
    extern __shared__ float4 wsh[];                     // [Co][K4]
    __shared__ int koff[K4 * 4], kdy[K4 * 4], kdx[K4 * 4];
    const int K = Ci * Kh * Kw;
    for (int i = threadIdx.x; i < Co * K4 * 4; i += blockDim.x) {
        const int co = i / (K4 * 4), k = i % (K4 * 4);
        reinterpret_cast<float*>(wsh)[i] = k < K ? w[(size_t)co * K + k] : 0.f;
    }
    for (int k = threadIdx.x; k < K4 * 4; k += blockDim.x) {
        const int kw = k % Kw, kh = (k / Kw) % Kh, ci = k / (Kw * Kh);
        koff[k] = k < K ? (ci * H + kh) * W + kw : 0;
        kdy[k] = k < K ? kh : -(1 << 20);               // padded k: always out of range
        kdx[k] = kw;
    }
    __syncthreads();
    const int hw = Ho * Wo, P = N * hw, chw = Ci * H * W;
    const int S = gridDim.x * blockDim.x;
    for (int p0 = blockIdx.x * blockDim.x + threadIdx.x; p0 < P; p0 += 2 * S) {
        const int pp[2] = {p0, p0 + S};
        float x[2][K4 * 4];
        int obase[2];
#pragma unroll
        for (int j = 0; j < 2; j++) {
            const int p = pp[j] < P ? pp[j] : p0;
            const int n = p / hw, r = p - n * hw, ho = r / Wo, wo = r - ho * Wo;
            const int y0 = ho * stride - pad, x0 = wo * stride - pad;
            const float* base = in + (size_t)n * chw + y0 * W + x0;
            obase[j] = n * Co * hw + r;
#pragma unroll
            for (int k = 0; k < K4 * 4; k++) {
                const int iy = y0 + kdy[k], ix = x0 + kdx[k];
                x[j][k] = (iy >= 0 && ix >= 0 && iy < H && ix < W) ? __ldg(base + koff[k]) : 0.f;
            }
        }
        const bool second = pp[1] < P;
        for (int co = 0; co < Co; co++) {
            float a0 = 0.f, a1 = 0.f;
#pragma unroll
            for (int k4 = 0; k4 < K4; k4++) {
                const float4 wv = wsh[co * K4 + k4];
                a0 = fmaf(wv.x, x[0][4 * k4], a0); a1 = fmaf(wv.x, x[1][4 * k4], a1);
                a0 = fmaf(wv.y, x[0][4 * k4 + 1], a0); a1 = fmaf(wv.y, x[1][4 * k4 + 1], a1);
                a0 = fmaf(wv.z, x[0][4 * k4 + 2], a0); a1 = fmaf(wv.z, x[1][4 * k4 + 2], a1);
                a0 = fmaf(wv.w, x[0][4 * k4 + 3], a0); a1 = fmaf(wv.w, x[1][4 * k4 + 3], a1);
            }
            out[(size_t)obase[0] + (size_t)co * hw] = relu && a0 < 0.f ? 0.f : a0;
            if (second) out[(size_t)obase[1] + (size_t)co * hw] = relu && a1 < 0.f ? 0.f : a1;
        }
    }
}

// Short-reduction conv with compile-time geometry: a thread computes 4 consecutive
// output pixels of one row (Wo % 4 == 0) for 16 output channels. Its input patch
// (CI x KH x (3*S + KW) values) sits in registers and serves all 16 channels; weights
// are stored [K][Co] in shared memory, so one float4 broadcast load feeds 16 FMAs
// (4 channels x 4 pixels). The warps of a block cover the same 32 pixel quads for
// different 16-channel groups (the patch loads hit L1), and each channel row is stored
// as float4 (a warp writes 512 contiguous bytes). Per output the reduction runs in k
// order, as in k_conv_smallk: the same bits. NHWC = true stores the output NHWC (4
// channels of one pixel per float4) for a conv that reads it next.
template <int CI, int KH, int KW, int S, bool NHWC>
__global__ void __launch_bounds__(256) k_conv_smallk_q(float* __restrict__ out, const float* __restrict__ in,
                                                       const float* __restrict__ w, int N, int H, int W, int Co,
                                                       int pad, int Ho, int Wo, int relu, float* __restrict__ out_lo) {
    constexpr int K = CI * KH * KW, PW = 3 * S + KW;
    extern __shared__ float4 wt4[];                      // [K][Co / 4], then (NHWC) 8 x [128 px][16 ch]
    float* wt = reinterpret_cast<float*>(wt4);
    for (int i = threadIdx.x; i < K * Co; i += blockDim.x) {
        const int k = i / Co, co = i - k * Co;
        wt[i] = w[(size_t)co * K + k];
    }
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // NHWC: the warp's 128 pixels x 16 channels are staged, float4 slots XOR-swizzled by
    // pixel quad, and stored as 64-byte channel runs (whole sectors) instead of 16-byte pieces
    float4* stg = reinterpret_cast<float4*>(wt + K * Co) + warp * 128 * 4;
    const int groups = Co / 16, quads_per_img = Ho * Wo / 4;
    const long long Q = (long long)N * quads_per_img;
    // warp job: (32 quads, one 16-channel group); blocks stride over the jobs
    const long long jobs = ((Q + 31) / 32) * groups;
    for (long long job = (long long)blockIdx.x * 8 + warp; job < jobs; job += (long long)gridDim.x * 8) {
        const int g = (int)(job % groups);
        const long long q0 = (job / groups) * 32, qi = q0 + lane;
        const bool active = qi < Q;
        if (!NHWC && !active) continue;
        const long long qc = active ? qi : Q - 1;       // inactive lanes compute a valid quad, store nothing
        const int n = (int)(qc / quads_per_img);
        const int r = (int)(qc - (long long)n * quads_per_img) * 4;
        const int ho = r / Wo, wo0 = r - ho * Wo;
        const int y0 = ho * S - pad, x0 = wo0 * S - pad;
        float x[CI][KH][PW];
        const float* base = in + (size_t)n * CI * H * W;
#pragma unroll
        for (int ci = 0; ci < CI; ci++)
#pragma unroll
            for (int kh = 0; kh < KH; kh++)
#pragma unroll
                for (int c = 0; c < PW; c++) {
                    const int iy = y0 + kh, ix = x0 + c;
                    x[ci][kh][c] = (iy >= 0 && ix >= 0 && iy < H && ix < W) ? __ldg(base + ((size_t)ci * H + iy) * W + ix) : 0.f;
                }
        float* obase = out + ((size_t)n * Co + g * 16) * Ho * Wo + (size_t)ho * Wo + wo0;
#pragma unroll 1
        for (int cq = 0; cq < 4; cq++) {
            float acc[4][4] = {};
            const float4* wk = wt4 + (g * 16 + cq * 4) / 4;
#pragma unroll
            for (int ci = 0; ci < CI; ci++)
#pragma unroll
                for (int kh = 0; kh < KH; kh++)
#pragma unroll
                    for (int kw = 0; kw < KW; kw++) {
                        const int k = (ci * KH + kh) * KW + kw;
                        const float4 wv = wk[k * (Co / 4)];
                        const float wc[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
                        for (int c = 0; c < 4; c++)
#pragma unroll
                            for (int j = 0; j < 4; j++) acc[c][j] = fmaf(wc[c], x[ci][kh][j * S + kw], acc[c][j]);
                    }
            if (NHWC) {
#pragma unroll
                for (int j = 0; j < 4; j++) {        // pixel 4*lane + j, channel slot cq
                    float4 v = make_float4(acc[0][j], acc[1][j], acc[2][j], acc[3][j]);
                    if (relu) { v.x = fmaxf(v.x, 0.f); v.y = fmaxf(v.y, 0.f); v.z = fmaxf(v.z, 0.f); v.w = fmaxf(v.w, 0.f); }
                    stg[(4 * lane + j) * 4 + (cq ^ (lane & 3))] = v;
                }
            } else {
#pragma unroll
                for (int c = 0; c < 4; c++) {
                    float4 v = make_float4(acc[c][0], acc[c][1], acc[c][2], acc[c][3]);
                    if (relu) { v.x = fmaxf(v.x, 0.f); v.y = fmaxf(v.y, 0.f); v.z = fmaxf(v.z, 0.f); v.w = fmaxf(v.w, 0.f); }
                    *reinterpret_cast<float4*>(obase + (size_t)(cq * 4 + c) * Ho * Wo) = v;
                }
            }
        }
        if (NHWC) {
            __syncwarp();
            // 4 lanes per pixel write its 64-byte run of this group's 16 channels
#pragma unroll 4
            for (int it = 0; it < 16; it++) {
                const int idx = it * 32 + lane, px = idx >> 2, c4 = idx & 3;
                if (q0 + (px >> 2) < Q) {
                    const size_t o = ((size_t)q0 * 4 + px) * Co + g * 16 + c4 * 4;
                    const float4 v = stg[px * 4 + (c4 ^ ((px >> 2) & 3))];
                    *reinterpret_cast<float4*>(out + o) = v;
                    if (out_lo)      // tf32_lo for a tensor-core conv that loads hi and lo
                        *reinterpret_cast<float4*>(out_lo + o) =
                            tc::tf32_lo4(v);
                }
            }
            __syncwarp();
        }
    }
}


extern "C" {

int lcu_conv_smallk_supported(size_t Ci, size_t Kh, size_t Kw, size_t Co) {
    return Ci * Kh * Kw <= 32 && Co <= 512 && Ci * Kh * Kw > 0;
}
static bool smallk_fits_int(size_t N, size_t Ci, size_t H, size_t W, size_t Co, size_t Ho, size_t Wo) {
    return N * Co * Ho * Wo < (1u << 31) && Ci * H * W < (1u << 31);
}

// the register-blocked geometries (Ci, Kh, Kw, stride) instantiated below
static bool smallk_q_geometry(size_t Ci, size_t Kh, size_t Kw, size_t stride) {
    return (Ci == 3 && Kh == 3 && Kw == 3 && (stride == 1 || stride == 2)) || (Ci == 1 && Kh == 3 && Kw == 3 && stride == 1) ||
           (Ci == 3 && Kh == 1 && Kw == 1 && stride == 1);
}
static bool smallk_q_shape(size_t N, size_t Ci, size_t H, size_t W, size_t Co, size_t Kh, size_t Kw, size_t stride,
                           size_t pad) {
    const size_t Ho = (H + 2 * pad - Kh) / stride + 1, Wo = (W + 2 * pad - Kw) / stride + 1;
    return smallk_q_geometry(Ci, Kh, Kw, stride) && Wo % 4 == 0 && Co % 16 == 0 && Co * Ci * Kh * Kw * 4 <= 48 * 1024 &&
           smallk_fits_int(N, Ci, H, W, Co, Ho, Wo);
}

int lcu_conv_smallk_nhwc_ok(size_t N, size_t Ci, size_t H, size_t W, size_t Co, size_t Kh, size_t Kw, size_t stride,
                            size_t pad) {
    return smallk_q_shape(N, Ci, H, W, Co, Kh, Kw, stride, pad);
}

lancius_error lcu_conv2d_smallk(float* out, const float* in, const float* w, size_t N, size_t Ci, size_t H, size_t W,
                                size_t Co, size_t Kh, size_t Kw, size_t stride, size_t pad, int relu, void* stream) {
    return lcu_conv2d_smallk_ex(out, in, w, N, Ci, H, W, Co, Kh, Kw, stride, pad, relu, 0, stream, nullptr);
}

lancius_error lcu_conv2d_smallk_ex(float* out, const float* in, const float* w, size_t N, size_t Ci, size_t H, size_t W,
                                   size_t Co, size_t Kh, size_t Kw, size_t stride, size_t pad, int relu, int out_nhwc,
                                   void* stream, float* out_lo) {
    const size_t Ho = (H + 2 * pad - Kh) / stride + 1, Wo = (W + 2 * pad - Kw) / stride + 1;
    const size_t P = N * Ho * Wo, K = Ci * Kh * Kw;
    if (P == 0 || Co == 0) return LANCIUS_ERROR_OK;
    if (!smallk_fits_int(N, Ci, H, W, Co, Ho, Wo))
        return lcu_conv2d_simt(out, in, w, N, Ci, H, W, Co, Kh, Kw, stride, pad, relu, stream);
    cudaStream_t st = lcu_as_stream(stream);
    // NHWC output for a tensor-core conv that reads it next: the tensor-core stem kernel
    // (FP32-exact), whose TMA stores keep the output write at HBM speed
    if (out_nhwc && lcu_conv_small_tc_ok(N, Ci, H, W, Co, Kh, Kw, stride, pad) && (reinterpret_cast<uintptr_t>(out) & 15) == 0 &&
        (reinterpret_cast<uintptr_t>(out_lo) & 15) == 0)
        return lcu_conv2d_small_tc_nhwc(out, out_lo, in, w, N, Ci, H, W, Co, Kh, Kw, stride, pad, relu, LCU_MODE_FP32_EXACT,
                                        stream);
    // register-blocked variants for common stems (4 pixels x 16 channels per thread)
    const bool qshape = smallk_q_shape(N, Ci, H, W, Co, Kh, Kw, stride, pad) && (reinterpret_cast<uintptr_t>(out) & 15) == 0;
    if (out_nhwc && !qshape) { lancius_set_error(LANCIUS_ERROR_UNSUPPORTED_OP); return LANCIUS_ERROR_UNSUPPORTED_OP; }
    if (qshape) {
        const size_t jobs = ((N * Ho * Wo / 4 + 31) / 32) * (Co / 16);
        const unsigned qgrid = (unsigned)std::min<size_t>((jobs + 7) / 8, 148u * 16u);
        const size_t qsmem = Co * K * 4 + (out_nhwc ? 8 * 128 * 16 * 4 : 0);
#define LCU_SMALLKQ(ci, kh, kw, s)                                                                                    \
        if (Ci == ci && Kh == kh && Kw == kw && stride == s) {                                                        \
            if (out_nhwc && cudaFuncSetAttribute(k_conv_smallk_q<ci, kh, kw, s, true>,                              \
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize, (int)qsmem) != cudaSuccess)\
                return lcu_launch_status();                                                                           \
            if (out_nhwc)                                                                                             \
                k_conv_smallk_q<ci, kh, kw, s, true><<<qgrid, 256, qsmem, st>>>(out, in, w, (int)N, (int)H, (int)W,  \
                                                                               (int)Co, (int)pad, (int)Ho, (int)Wo,  \
                                                                               relu, out_lo);                        \
            else                                                                                                      \
                k_conv_smallk_q<ci, kh, kw, s, false><<<qgrid, 256, qsmem, st>>>(out, in, w, (int)N, (int)H, (int)W, \
                                                                                (int)Co, (int)pad, (int)Ho, (int)Wo, \
                                                                                relu, nullptr);                      \
            lcu_note_launch();                                                                                        \
            return lcu_launch_status();                                                                               \
        }
        LCU_SMALLKQ(3, 3, 3, 1) LCU_SMALLKQ(3, 3, 3, 2) LCU_SMALLKQ(1, 3, 3, 1) LCU_SMALLKQ(3, 1, 1, 1)
#undef LCU_SMALLKQ
    }
    const int K4 = (int)((K + 3) / 4);
    const size_t smem = Co * K4 * sizeof(float4);
    const unsigned grid = lcu_blocks(P, 256, 148u * 8u);
#define LCU_SMALLK(k4)                                                                                                \
    case k4:                                                                                                          \
        if (smem > 48 * 1024 && cudaFuncSetAttribute(k_conv_smallk<k4>, cudaFuncAttributeMaxDynamicSharedMemorySize,  \
                                                     (int)smem) != cudaSuccess)                                       \
            return lcu_launch_status();                                                                               \
        k_conv_smallk<k4><<<grid, 256, smem, st>>>(out, in, w, (int)N, (int)Ci, (int)H, (int)W, (int)Co, (int)Kh,    \
                                                  (int)Kw, (int)stride, (int)pad, (int)Ho, (int)Wo, relu);            \
        break;
    switch (K4) {
        LCU_SMALLK(1) LCU_SMALLK(2) LCU_SMALLK(3) LCU_SMALLK(4) LCU_SMALLK(5) LCU_SMALLK(6) LCU_SMALLK(7) LCU_SMALLK(8)
        default: lancius_set_error(LANCIUS_ERROR_UNSUPPORTED_OP); return LANCIUS_ERROR_UNSUPPORTED_OP;
    }
#undef LCU_SMALLK
    lcu_note_launch();
    return lcu_launch_status();
}

// Grouped launch over a device-resident table of `count` products of one shape.
lancius_error lcu_gemm_simt_grouped(const LcuGemmGroup* d_groups, int count, size_t M, size_t N, size_t K, int epi,
                                    void* stream) {
    if (count <= 0 || M == 0 || N == 0) return LANCIUS_ERROR_OK;
    if (epi == LCU_EPI_SOFTMAX_ROW && N > (size_t)SK_TN) { lancius_set_error(LANCIUS_ERROR_INTERNAL); return LANCIUS_ERROR_INTERNAL; }
    if (use_skinny(M, N, count) || epi == LCU_EPI_SOFTMAX_ROW) {
        dim3 g((unsigned)((N + SK_TN - 1) / SK_TN), (unsigned)((M + SK_TM - 1) / SK_TM), (unsigned)count);
        if (!skinny_configured()) return lcu_launch_status();
        k_gemm_skinny<<<g, 256, SK_SMEM_BYTES, lcu_as_stream(stream)>>>(d_groups, LcuGemmGroup{}, M, N, K, epi);
        lcu_note_launch();
        return lcu_launch_status();
    }
    dim3 grid((unsigned)((N + BN - 1) / BN), (unsigned)((M + BM - 1) / BM), (unsigned)count);
    k_gemm_simt<<<grid, THREADS, 0, lcu_as_stream(stream)>>>(d_groups, M, N, K, epi);
    lcu_note_launch();
    return lcu_launch_status();
}

lancius_error lcu_gemm_simt(float* c, const float* a, const float* b, size_t M, size_t K, size_t N, const float* bias,
                            int epi, void* stream) {
    if (M == 0 || N == 0) return LANCIUS_ERROR_OK;
    LcuGemmGroup g{a, b, c, bias, nullptr};
    if (use_skinny(M, N, 1)) {
        dim3 gs((unsigned)((N + SK_TN - 1) / SK_TN), (unsigned)((M + SK_TM - 1) / SK_TM), 1);
        if (!skinny_configured()) return lcu_launch_status();
        k_gemm_skinny<<<gs, 256, SK_SMEM_BYTES, lcu_as_stream(stream)>>>(nullptr, g, M, N, K, epi);
        lcu_note_launch();
        return lcu_launch_status();
    }
    dim3 grid((unsigned)((N + BN - 1) / BN), (unsigned)((M + BM - 1) / BM), 1);
    k_gemm_simt1<<<grid, THREADS, 0, lcu_as_stream(stream)>>>(g, M, N, K, epi);
    lcu_note_launch();
    return lcu_launch_status();
}

lancius_error lcu_conv2d_simt(float* out, const float* in, const float* w, size_t N, size_t Ci, size_t H, size_t W,
                              size_t Co, size_t Kh, size_t Kw, size_t stride, size_t pad, int relu, void* stream) {
    size_t Ho = (H + 2 * pad - Kh) / stride + 1, Wo = (W + 2 * pad - Kw) / stride + 1;
    size_t P = N * Ho * Wo;
    dim3 grid((unsigned)((P + BN - 1) / BN), (unsigned)((Co + BM - 1) / BM), 1);
    k_conv_simt<<<grid, THREADS, 0, lcu_as_stream(stream)>>>(out, in, w, (int)N, (int)Ci, (int)H, (int)W, (int)Co,
                                                             (int)Kh, (int)Kw, (int)stride, (int)pad, (int)Ho, (int)Wo, relu);
    lcu_note_launch();
    return lcu_launch_status();
}

}  // extern "C"
