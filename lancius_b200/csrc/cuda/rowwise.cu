// Row-wise HBM-bound kernels: one warp per row, shuffle reductions, 128-bit IO.
//   layernorm  -- kernel_layernorm  (lancius_kernels.c:217-236)
//   softmax    -- executor SOFTMAX  (lancius_scheduler.c:284-294)
//   sum_axis1  -- executor SUM_AXIS1 (lancius_scheduler.c:263-267), the GAP reduction
//   maxpool2d  -- vision op MAXPOOL2D (lancius_vision_ops.c:82-112)
#include "lcu_internal.h"

namespace {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Row held in registers: VPL float4 per lane, hidden == 128 * VPL at most.
template <int VPL>
__global__ void __launch_bounds__(256) k_layernorm_reg(const LcuRowGroup* __restrict__ table, LcuRowGroup g,
                                                       size_t rows, int hidden, float eps) {
    if (table) g = table[blockIdx.y];
    float* __restrict__ out = g.out;
    const float* __restrict__ in = g.in;
    const float* __restrict__ gamma = g.gamma;
    const float* __restrict__ beta = g.beta;
    int lane = threadIdx.x & 31;
    size_t row = (size_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (row >= rows) return;
    const float4* x = reinterpret_cast<const float4*>(in + row * hidden);
    int n4 = hidden >> 2;
    float4 v[VPL];
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < VPL; i++) {
        int c = lane + 32 * i;
        v[i] = c < n4 ? __ldcs(x + c) : make_float4(0.f, 0.f, 0.f, 0.f);
        s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
    }
    float mean = warp_sum(s) / (float)hidden;
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < VPL; i++) {
        int c = lane + 32 * i;
        if (c < n4) {
            float a = v[i].x - mean, b = v[i].y - mean, cc = v[i].z - mean, d = v[i].w - mean;
            q += (a * a + b * b) + (cc * cc + d * d);
        }
    }
    float var = warp_sum(q) / (float)hidden;
    float inv = rsqrtf(var + eps);
    float4* y = reinterpret_cast<float4*>(out + row * hidden);
    const float4* g4 = reinterpret_cast<const float4*>(gamma);
    const float4* b4 = reinterpret_cast<const float4*>(beta);
#pragma unroll
    for (int i = 0; i < VPL; i++) {
        int c = lane + 32 * i;
        if (c < n4) {
            float4 gg = __ldg(g4 + c), bb = __ldg(b4 + c), r;
            r.x = (v[i].x - mean) * inv * gg.x + bb.x;
            r.y = (v[i].y - mean) * inv * gg.y + bb.y;
            r.z = (v[i].z - mean) * inv * gg.z + bb.z;
            r.w = (v[i].w - mean) * inv * gg.w + bb.w;
            __stcs(y + c, r);
        }
    }
}

// Any width / alignment: three passes over the row (passes 2-3 hit L1).
__global__ void k_layernorm_any(const LcuRowGroup* __restrict__ table, LcuRowGroup g, size_t rows, size_t hidden,
                                float eps) {
    if (table) g = table[blockIdx.y];
    float* __restrict__ out = g.out;
    const float* __restrict__ in = g.in;
    const float* __restrict__ gamma = g.gamma;
    const float* __restrict__ beta = g.beta;
    int lane = threadIdx.x & 31;
    size_t row = (size_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (row >= rows) return;
    const float* x = in + row * hidden;
    float s = 0.f;
    for (size_t c = lane; c < hidden; c += 32) s += x[c];
    float mean = warp_sum(s) / (float)hidden;
    float q = 0.f;
    for (size_t c = lane; c < hidden; c += 32) { float d = x[c] - mean; q += d * d; }
    float inv = rsqrtf(warp_sum(q) / (float)hidden + eps);
    for (size_t c = lane; c < hidden; c += 32) out[row * hidden + c] = (x[c] - mean) * inv * gamma[c] + beta[c];
}

__global__ void k_softmax(float* __restrict__ out, const float* __restrict__ in, size_t rows, size_t cols) {
    int lane = threadIdx.x & 31;
    size_t row = (size_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (row >= rows) return;
    const float* x = in + row * cols;
    float m = -INFINITY;
    for (size_t c = lane; c < cols; c += 32) m = fmaxf(m, x[c]);
    m = warp_max(m);
    float s = 0.f;
    for (size_t c = lane; c < cols; c += 32) s += expf(x[c] - m);
    float inv = 1.f / warp_sum(s);
    for (size_t c = lane; c < cols; c += 32) out[row * cols + c] = expf(x[c] - m) * inv;
}

__global__ void k_sum_axis1(float* __restrict__ out, const float* __restrict__ in, size_t rows, size_t cols) {
    int lane = threadIdx.x & 31;
    size_t row = (size_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (row >= rows) return;
    const float* x = in + row * cols;
    float s = 0.f;
    if (((uintptr_t)x & 15u) == 0 && (cols & 3u) == 0) {
        const float4* x4 = reinterpret_cast<const float4*>(x);
        for (size_t c = lane; c < cols / 4; c += 32) { float4 v = __ldcs(x4 + c); s += (v.x + v.y) + (v.z + v.w); }
    } else {
        for (size_t c = lane; c < cols; c += 32) s += x[c];
    }
    s = warp_sum(s);
    if (lane == 0) out[row] = s;
}

__global__ void k_maxpool(float* __restrict__ out, const float* __restrict__ in, size_t planes, size_t H, size_t W,
                          size_t Ho, size_t Wo, int K, int stride) {
    size_t n = planes * Ho * Wo;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        size_t wo = i % Wo, t = i / Wo, ho = t % Ho, p = t / Ho;
        const float* src = in + (p * H + ho * stride) * W + wo * stride;
        float m = -1e9f;
        for (int kh = 0; kh < K; kh++)
            for (int kw = 0; kw < K; kw++) m = fmaxf(m, src[kh * W + kw]);
        out[i] = m;
    }
}

}  // namespace

extern "C" {

lancius_error lcu_layernorm_grouped(const LcuRowGroup* d_table, int count, LcuRowGroup one, size_t rows, size_t hidden,
                                    float eps, int vec, void* s) {
    if (rows == 0 || hidden == 0 || count <= 0) return LANCIUS_ERROR_OK;
    cudaStream_t st = lcu_as_stream(s);
    dim3 grid((unsigned)((rows + 7) / 8), (unsigned)count);
    int n4 = (int)(hidden / 4);
    vec = vec && hidden % 4 == 0;
    if (vec && n4 <= 32 * 2) k_layernorm_reg<2><<<grid, 256, 0, st>>>(d_table, one, rows, (int)hidden, eps);
    else if (vec && n4 <= 32 * 6) k_layernorm_reg<6><<<grid, 256, 0, st>>>(d_table, one, rows, (int)hidden, eps);
    else if (vec && n4 <= 32 * 16) k_layernorm_reg<16><<<grid, 256, 0, st>>>(d_table, one, rows, (int)hidden, eps);
    else k_layernorm_any<<<grid, 256, 0, st>>>(d_table, one, rows, hidden, eps);
    lcu_note_launch();
    return lcu_launch_status();
}

lancius_error lcu_layernorm(float* out, const float* in, const float* gamma, const float* beta, size_t rows,
                            size_t hidden, float eps, void* s) {
    if (!out || !in || !gamma || !beta) { lancius_set_error(LANCIUS_ERROR_NULL_PTR); return LANCIUS_ERROR_NULL_PTR; }
    bool vec = ((uintptr_t)out % 16 == 0) && ((uintptr_t)in % 16 == 0) && ((uintptr_t)gamma % 16 == 0) &&
               ((uintptr_t)beta % 16 == 0);
    return lcu_layernorm_grouped(nullptr, 1, LcuRowGroup{out, in, gamma, beta}, rows, hidden, eps, vec, s);
}

lancius_error lcu_softmax(float* out, const float* in, size_t rows, size_t cols, void* s) {
    if (!out || !in) { lancius_set_error(LANCIUS_ERROR_NULL_PTR); return LANCIUS_ERROR_NULL_PTR; }
    if (rows == 0 || cols == 0) return LANCIUS_ERROR_OK;
    k_softmax<<<(unsigned)((rows + 7) / 8), 256, 0, lcu_as_stream(s)>>>(out, in, rows, cols);
    lcu_note_launch();
    return lcu_launch_status();
}

lancius_error lcu_sum_axis1(float* out, const float* in, size_t rows, size_t cols, void* s) {
    if (!out || !in) { lancius_set_error(LANCIUS_ERROR_NULL_PTR); return LANCIUS_ERROR_NULL_PTR; }
    if (rows == 0) return LANCIUS_ERROR_OK;
    k_sum_axis1<<<(unsigned)((rows + 7) / 8), 256, 0, lcu_as_stream(s)>>>(out, in, rows, cols);
    lcu_note_launch();
    return lcu_launch_status();
}

lancius_error lcu_maxpool2d(float* out, const float* in, size_t N, size_t C, size_t H, size_t W, size_t K,
                            size_t stride, void* s) {
    if (!out || !in) { lancius_set_error(LANCIUS_ERROR_NULL_PTR); return LANCIUS_ERROR_NULL_PTR; }
    if (K == 0 || stride == 0 || H < K || W < K) { lancius_set_error(LANCIUS_ERROR_SHAPE_MISMATCH); return LANCIUS_ERROR_SHAPE_MISMATCH; }
    size_t Ho = (H - K) / stride + 1, Wo = (W - K) / stride + 1;
    k_maxpool<<<lcu_blocks(N * C * Ho * Wo, 256), 256, 0, lcu_as_stream(s)>>>(out, in, N * C, H, W, Ho, Wo, (int)K, (int)stride);
    lcu_note_launch();
    return lcu_launch_status();
}

}  // extern "C"
