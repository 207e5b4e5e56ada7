// FP32 CUDA-core GEMM core (FFMA, FP32 accumulate) for shapes the tensor-core
// path does not take: tiny problems (launch-bound MLP layers), row strides that
// break TMA's 16-byte rule (e.g. N = 10), and per-launch fallbacks.
// 128x128x8 tile, 256 threads, 8x8 outputs per thread, double-buffered smem.
#pragma once
#include "lcu_internal.h"


namespace lcu_simt {

constexpr int BM = 128, BN = 128, BK = 8, THREADS = 256;

// Loader / storer policies ---------------------------------------------------
struct DenseA {   // A[M,K] row-major
    const float* p; size_t M, K, lda;
    __device__ float operator()(size_t m, size_t k) const { return (m < M && k < K) ? __ldg(p + m * lda + k) : 0.f; }
};
struct DenseB {   // B[K,N] row-major
    const float* p; size_t K, N, ldb;
    __device__ float operator()(size_t k, size_t n) const { return (k < K && n < N) ? __ldg(p + k * ldb + n) : 0.f; }
};
struct DenseC {   // C[M,N] row-major: act(acc + bias[n]) + resid[m,n]
    float* p; const float* bias; const float* resid; size_t M, N, ldc; int epi;
    __device__ void operator()(size_t m, size_t n, float v) const {
        if (m < M && n < N) {
            if (bias) v += __ldg(bias + n);
            v = lcu_apply_epi(v, epi);
            if (resid) v += resid[m * ldc + n];
            p[m * ldc + n] = v;
        }
    }
};
// Implicit-GEMM conv: A = W[Co, Ci*Kh*Kw]; B[k, P] gathered from NCHW input on the fly.
struct Im2colB {
    const float* in; int Ci, H, W, Kh, Kw, stride, pad, Ho, Wo; size_t P, Kdim;
    __device__ float operator()(size_t k, size_t p) const {
        if (k >= Kdim || p >= P) return 0.f;
        int kw = (int)(k % Kw); size_t t = k / Kw; int kh = (int)(t % Kh); int ci = (int)(t / Kh);
        size_t hw = (size_t)Ho * Wo; size_t n = p / hw; size_t r = p % hw;
        int ho = (int)(r / Wo), wo = (int)(r % Wo);
        int ih = ho * stride - pad + kh, iw = wo * stride - pad + kw;
        if (ih < 0 || iw < 0 || ih >= H || iw >= W) return 0.f;
        return __ldg(in + (((n * Ci + ci) * H + ih) * (size_t)W + iw));
    }
};
struct ConvC {    // (co, P) -> out[n][co][pixel], NCHW
    float* out; size_t Co, P, HoWo; int relu;
    __device__ void operator()(size_t co, size_t p, float v) const {
        if (co < Co && p < P) {
            size_t n = p / HoWo, r = p % HoWo;
            out[(n * Co + co) * HoWo + r] = (relu && !(v > 0.f)) ? 0.f : v;
        }
    }
};

template <class AL, class BL, class ST>
__device__ __forceinline__ void gemm_tile(const AL& A, const BL& B, const ST& C, size_t K, size_t m0, size_t n0) {
    __shared__ float As[2][BK][BM];
    __shared__ float Bs[2][BK][BN];
    const int tid = threadIdx.x;
    const int tx = tid % 16, ty = tid / 16;
    float acc[8][8];
#pragma unroll
    for (int i = 0; i < 8; i++)
#pragma unroll
        for (int j = 0; j < 8; j++) acc[i][j] = 0.f;

    // each thread stages 4 A values (rows am, k-cols ak..ak+3) and 4 B values
    const int am = tid / 2, ak = (tid % 2) * 4;
    const int bk = tid / 32, bn = (tid % 32) * 4;
    float ra[4], rb[4];
    auto fetch = [&](size_t k0) {
#pragma unroll
        for (int i = 0; i < 4; i++) ra[i] = A(m0 + am, k0 + ak + i);
#pragma unroll
        for (int i = 0; i < 4; i++) rb[i] = B(k0 + bk, n0 + bn + i);
    };
    auto stash = [&](int buf) {
#pragma unroll
        for (int i = 0; i < 4; i++) As[buf][ak + i][am] = ra[i];
#pragma unroll
        for (int i = 0; i < 4; i++) Bs[buf][bk][bn + i] = rb[i];
    };
    size_t tiles = (K + BK - 1) / BK;
    fetch(0);
    stash(0);
    __syncthreads();
    for (size_t t = 0; t < tiles; t++) {
        int buf = (int)(t & 1);
        if (t + 1 < tiles) fetch((t + 1) * BK);
#pragma unroll
        for (int kk = 0; kk < BK; kk++) {
            float a[8], b[8];
            float4 a0 = *reinterpret_cast<const float4*>(&As[buf][kk][ty * 4]);
            float4 a1 = *reinterpret_cast<const float4*>(&As[buf][kk][ty * 4 + 64]);
            float4 b0 = *reinterpret_cast<const float4*>(&Bs[buf][kk][tx * 4]);
            float4 b1 = *reinterpret_cast<const float4*>(&Bs[buf][kk][tx * 4 + 64]);
            a[0] = a0.x; a[1] = a0.y; a[2] = a0.z; a[3] = a0.w; a[4] = a1.x; a[5] = a1.y; a[6] = a1.z; a[7] = a1.w;
            b[0] = b0.x; b[1] = b0.y; b[2] = b0.z; b[3] = b0.w; b[4] = b1.x; b[5] = b1.y; b[6] = b1.z; b[7] = b1.w;
#pragma unroll
            for (int i = 0; i < 8; i++)
#pragma unroll
                for (int j = 0; j < 8; j++) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
        }
        if (t + 1 < tiles) stash(buf ^ 1);
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 8; i++) {
        size_t m = m0 + ty * 4 + (i & 3) + (i >= 4 ? 64 : 0);
#pragma unroll
        for (int j = 0; j < 8; j++) {
            size_t n = n0 + tx * 4 + (j & 3) + (j >= 4 ? 64 : 0);
            C(m, n, acc[i][j]);
        }
    }
}

}  // namespace lcu_simt
