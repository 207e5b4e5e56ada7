// CUDA-core FP32 GEMM and implicit-GEMM conv launchers (see gemm_simt.cuh).
#include "gemm_simt.cuh"

using namespace lcu_simt;

__global__ void __launch_bounds__(THREADS) k_gemm_simt(const LcuGemmGroup* __restrict__ groups, size_t M, size_t N,
                                                       size_t K, int epi) {
    LcuGemmGroup gr = groups[blockIdx.z];
    DenseA A{gr.a, M, K, K};
    DenseB B{gr.b, K, N, N};
    DenseC C{gr.c, gr.bias, gr.resid, M, N, N, epi};
    gemm_tile(A, B, C, K, (size_t)blockIdx.y * BM, (size_t)blockIdx.x * BN);
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

extern "C" {

// Grouped launch over a device-resident table of `count` products of one shape.
lancius_error lcu_gemm_simt_grouped(const LcuGemmGroup* d_groups, int count, size_t M, size_t N, size_t K, int epi,
                                    void* stream) {
    if (count <= 0 || M == 0 || N == 0) return LANCIUS_ERROR_OK;
    dim3 grid((unsigned)((N + BN - 1) / BN), (unsigned)((M + BM - 1) / BM), (unsigned)count);
    k_gemm_simt<<<grid, THREADS, 0, lcu_as_stream(stream)>>>(d_groups, M, N, K, epi);
    lcu_note_launch();
    return lcu_launch_status();
}

lancius_error lcu_gemm_simt(float* c, const float* a, const float* b, size_t M, size_t K, size_t N, const float* bias,
                            int epi, void* stream) {
    if (M == 0 || N == 0) return LANCIUS_ERROR_OK;
    LcuGemmGroup g{a, b, c, bias, nullptr};
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
