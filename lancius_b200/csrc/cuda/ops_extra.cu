// Executor opcodes beyond the benchmark configurations: training operators (the
// reference autodiff's backward nodes), LLM operators and the INT8 weight path.
// Each kernel restates the reference line range named beside it, in FP32.
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
// block-wide sum of a 1024-thread block (result valid in every thread)
__device__ float block_sum(float v) {
    __shared__ float part[32];
    v = warp_sum(v);
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = v;
    __syncthreads();
    float r = threadIdx.x < (blockDim.x >> 5) ? part[threadIdx.x] : 0.f;
    r = warp_sum(r);
    __syncthreads();
    return r;
}

// SUM (scheduler.c:251-256): one 1024-thread block, fixed order -> deterministic
__global__ void k_sum_all(float* out, const float* a, size_t n) {
    float s = 0.f;
    for (size_t i = threadIdx.x; i < n; i += blockDim.x) s += a[i];
    s = block_sum(s);
    if (threadIdx.x == 0) out[0] = s;
}
// SUM_AXIS0 (scheduler.c:257-262): thread per column
__global__ void k_sum_axis0(float* out, const float* a, size_t R, size_t C) {
    for (size_t c = blockIdx.x * (size_t)blockDim.x + threadIdx.x; c < C; c += (size_t)gridDim.x * blockDim.x) {
        float s = 0.f;
        for (size_t r = 0; r < R; r++) s += a[r * C + c];
        out[c] = s;
    }
}
// TRANSPOSE (scheduler.c:246-250): 32x32 tiles through shared memory
__global__ void k_transpose(float* out, const float* a, size_t R, size_t C) {
    __shared__ float t[32][33];
    size_t r0 = (size_t)blockIdx.y * 32, c0 = (size_t)blockIdx.x * 32;
    for (int i = threadIdx.y; i < 32; i += 8) {
        size_t r = r0 + i, c = c0 + threadIdx.x;
        if (r < R && c < C) t[i][threadIdx.x] = a[r * C + c];
    }
    __syncthreads();
    for (int i = threadIdx.y; i < 32; i += 8) {
        size_t c = c0 + i, r = r0 + threadIdx.x;
        if (r < R && c < C) out[c * R + r] = t[threadIdx.x][i];
    }
}
// RELU_BWD (scheduler.c:279-283)
__global__ void k_relu_bwd(float* out, const float* grad, const float* fwd, size_t n) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        out[i] = fwd[i] > 0.f ? grad[i] : 0.f;
}
// SOFTMAX_BWD (scheduler.c:295-304): warp per row
__global__ void k_softmax_bwd(float* out, const float* dy, const float* y, size_t R, size_t C) {
    size_t row = (size_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    int lane = threadIdx.x & 31;
    if (row >= R) return;
    float d = 0.f;
    for (size_t c = lane; c < C; c += 32) d += dy[row * C + c] * y[row * C + c];
    d = warp_sum(d);
    for (size_t c = lane; c < C; c += 32) out[row * C + c] = y[row * C + c] * (dy[row * C + c] - d);
}
// CROSS_ENTROPY (scheduler.c:68-86): |mean over rows of -(x_t - logsumexp(x))|, one block
__global__ void k_cross_entropy(float* out, const float* x, const float* y, size_t R, size_t C) {
    float tot = 0.f;
    for (size_t r = threadIdx.x >> 5; r < R; r += blockDim.x >> 5) {
        int lane = threadIdx.x & 31;
        float m = -INFINITY;
        for (size_t c = lane; c < C; c += 32) m = fmaxf(m, x[r * C + c]);
        m = warp_max(m);
        float se = 0.f;
        for (size_t c = lane; c < C; c += 32) se += expf(x[r * C + c] - m);
        float lse = logf(warp_sum(se)) + m;
        float part = 0.f;
        for (size_t c = lane; c < C; c += 32) if (y[r * C + c] == 1.f) part -= x[r * C + c] - lse;
        part = warp_sum(part);
        if (lane == 0) tot += part;
    }
    tot = block_sum((threadIdx.x & 31) == 0 ? tot : 0.f);
    if (threadIdx.x == 0) out[0] = fabsf(tot / (float)R);
}
// CROSS_ENTROPY_BWD (scheduler.c:90-106): (softmax(x) - y) * g[0] / R, warp per row
__global__ void k_cross_entropy_bwd(float* out, const float* x, const float* y, const float* g, size_t R, size_t C) {
    size_t row = (size_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    int lane = threadIdx.x & 31;
    if (row >= R) return;
    float m = -INFINITY;
    for (size_t c = lane; c < C; c += 32) m = fmaxf(m, x[row * C + c]);
    m = warp_max(m);
    float se = 0.f;
    for (size_t c = lane; c < C; c += 32) se += expf(x[row * C + c] - m);
    se = warp_sum(se);
    const float sc = g[0] / (float)R;
    for (size_t c = lane; c < C; c += 32) out[row * C + c] = (expf(x[row * C + c] - m) / se - y[row * C + c]) * sc;
}
// RMSNORM (lancius_kernels.c:381-396): warp per row
__global__ void k_rmsnorm(float* out, const float* in, const float* gamma, size_t R, size_t Hd, float eps) {
    size_t row = (size_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    int lane = threadIdx.x & 31;
    if (row >= R) return;
    const float* x = in + row * Hd;
    float q = 0.f;
    for (size_t c = lane; c < Hd; c += 32) q += x[c] * x[c];
    float inv = rsqrtf(warp_sum(q) / (float)Hd + eps);
    for (size_t c = lane; c < Hd; c += 32) out[row * Hd + c] = x[c] * inv * gamma[c];
}
// SWIGLU (lancius_kernels.c:398-405)
__global__ void k_swiglu(float* out, const float* gate, const float* up, size_t n) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        float g = gate[i];
        out[i] = g / (1.f + expf(-g)) * up[i];
    }
}
// ROPE (lancius_kernels.c:248-272), in place on interleaved pairs
__global__ void k_rope(float* q, float* k, size_t B, size_t S, size_t H, size_t D, int pos_offset) {
    size_t pairs = B * S * H * (D / 2);
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < pairs; i += (size_t)gridDim.x * blockDim.x) {
        size_t d = (i % (D / 2)) * 2, t = i / (D / 2), s = (t / H) % S;
        float freq = (float)(1.0 / pow(10000.0, (double)d / (double)D));
        float ang = (float)((long)s + pos_offset) * freq;
        float c, sn;
        sincosf(ang, &sn, &c);
        size_t o = t * D + d;
        float q0 = q[o], q1 = q[o + 1], k0 = k[o], k1 = k[o + 1];
        q[o] = q0 * c - q1 * sn; q[o + 1] = q0 * sn + q1 * c;
        k[o] = k0 * c - k1 * sn; k[o + 1] = k0 * sn + k1 * c;
    }
}
// MAXPOOL2D_BWD (vision_ops.c:149-190): gradient to the first maximum of each window.
// Thread per input element gathers the windows that route to it (deterministic).
__global__ void k_maxpool_bwd(float* out, const float* grad, const float* in, size_t planes, int H, int W, int Ho, int Wo,
                              int K, int stride) {
    size_t n = planes * H * W;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        int iw = (int)(i % W), ih = (int)((i / W) % H);
        size_t p = i / ((size_t)H * W);
        const float* src = in + p * H * W;
        float acc = 0.f;
        int ho_lo = ih >= K ? (ih - K) / stride + 1 : 0, wo_lo = iw >= K ? (iw - K) / stride + 1 : 0;
        for (int ho = ho_lo; ho <= ih / stride && ho < Ho; ho++)
            for (int wo = wo_lo; wo <= iw / stride && wo < Wo; wo++) {
                if (ih < ho * stride || iw < wo * stride || ih >= ho * stride + K || iw >= wo * stride + K) continue;
                float m = -1e9f;
                int bi = 0, bj = 0;
                for (int kh = 0; kh < K; kh++)
                    for (int kw = 0; kw < K; kw++) {
                        float v = src[(ho * stride + kh) * W + wo * stride + kw];
                        if (v > m) { m = v; bi = ho * stride + kh; bj = wo * stride + kw; }
                    }
                if (bi == ih && bj == iw) acc += grad[(p * Ho + ho) * Wo + wo];
            }
        out[i] = acc;
    }
}
// CONV2D_BWD (kernel_conv2d_bwd_in, lancius_kernels.c:62-91) as a gather per input element
__global__ void k_conv_bwd_in(float* out, const float* grad, const float* w, int N, int Ci, int H, int W, int Co, int Ho,
                              int Wo, int Kh, int Kw, int stride, int pad) {
    size_t n_el = (size_t)N * Ci * H * W;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n_el; i += (size_t)gridDim.x * blockDim.x) {
        int iw = (int)(i % W), ih = (int)((i / W) % H), ci = (int)((i / ((size_t)W * H)) % Ci);
        size_t n = i / ((size_t)W * H * Ci);
        float acc = 0.f;
        for (int co = 0; co < Co; co++)
            for (int kh = 0; kh < Kh; kh++) {
                int t = ih + pad - kh;
                if (t < 0 || t % stride) continue;
                int ho = t / stride;
                if (ho >= Ho) continue;
                for (int kw = 0; kw < Kw; kw++) {
                    int u = iw + pad - kw;
                    if (u < 0 || u % stride) continue;
                    int wo = u / stride;
                    if (wo >= Wo) continue;
                    acc += grad[((n * Co + co) * Ho + ho) * (size_t)Wo + wo] * w[((size_t)(co * Ci + ci) * Kh + kh) * Kw + kw];
                }
            }
        out[i] = acc;
    }
}
// CONV2D_BWD_W (kernel_conv2d_bwd_w, lancius_kernels.c:93-136): one block per weight
// element reduces over (n, ho, wo) in a fixed order
__global__ void k_conv_bwd_w(float* out, const float* grad, const float* in, int N, int Ci, int H, int W, int Co, int Ho,
                             int Wo, int Kh, int Kw, int stride, int pad) {
    const int e = blockIdx.x;
    const int kw = e % Kw, kh = (e / Kw) % Kh, ci = (e / (Kw * Kh)) % Ci, co = e / (Kw * Kh * Ci);
    const size_t cnt = (size_t)N * Ho * Wo;
    float acc = 0.f;
    for (size_t i = threadIdx.x; i < cnt; i += blockDim.x) {
        int wo = (int)(i % Wo), ho = (int)((i / Wo) % Ho);
        size_t n = i / ((size_t)Wo * Ho);
        int ih = ho * stride - pad + kh, iw = wo * stride - pad + kw;
        if (ih < 0 || iw < 0 || ih >= H || iw >= W) continue;
        acc += grad[((n * Co + co) * Ho + ho) * (size_t)Wo + wo] * in[((n * Ci + ci) * H + ih) * (size_t)W + iw];
    }
    acc = block_sum(acc);
    if (threadIdx.x == 0) out[e] = acc;
}
// INT8 path (scheduler.c:195-220, vision_ops.c:16-57): max |a| of the activation ...
__global__ void k_absmax(float* out, const float* a, size_t n) {
    __shared__ float part[32];
    float m = 0.f;
    for (size_t i = threadIdx.x; i < n; i += blockDim.x) m = fmaxf(m, fabsf(a[i]));
    m = warp_max(m);
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x < 32) {
        float r = threadIdx.x < (blockDim.x >> 5) ? part[threadIdx.x] : 0.f;
        r = warp_max(r);
        if (threadIdx.x == 0) out[0] = r;
    }
}
__device__ __forceinline__ int quant(float x, double scale) {
    return (int)(signed char)(int)round((double)x / scale);         // round half away from zero, wraps like the C cast
}
// ... then int8 x int8 products summed in int32, times scale_a * scale_b
__global__ void k_matmul_int8(float* out, const float* a, const int8_t* b, const float* amax, double scale_b, size_t M,
                              size_t K, size_t N) {
    const double sa = amax[0] > 0.f ? (double)amax[0] / 127.0 : 1e-8;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < M * N; i += (size_t)gridDim.x * blockDim.x) {
        size_t r = i / N, c = i % N;
        int acc = 0;
        for (size_t k = 0; k < K; k++) acc += quant(a[r * K + k], sa) * (int)b[k * N + c];
        out[i] = (float)((double)acc * (sa * scale_b));
    }
}
__global__ void k_conv_int8(float* out, const float* in, const int8_t* w, const float* amax, double scale_w, int N, int Ci,
                            int H, int W, int Co, int Kh, int Kw, int stride, int pad, int Ho, int Wo, int relu) {
    const double sa = amax[0] > 0.f ? (double)amax[0] / 127.0 : 1e-8;
    size_t n_el = (size_t)N * Co * Ho * Wo;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n_el; i += (size_t)gridDim.x * blockDim.x) {
        int wo = (int)(i % Wo), ho = (int)((i / Wo) % Ho), co = (int)((i / ((size_t)Wo * Ho)) % Co);
        size_t n = i / ((size_t)Wo * Ho * Co);
        int acc = 0;
        for (int ci = 0; ci < Ci; ci++)
            for (int kh = 0; kh < Kh; kh++)
                for (int kw = 0; kw < Kw; kw++) {
                    int ih = ho * stride - pad + kh, iw = wo * stride - pad + kw;
                    if (ih < 0 || iw < 0 || ih >= H || iw >= W) continue;
                    acc += quant(in[((n * Ci + ci) * H + ih) * (size_t)W + iw], sa) * (int)w[((co * Ci + ci) * Kh + kh) * Kw + kw];
                }
        float v = (float)((double)acc * (sa * scale_w));
        out[i] = (relu && v < 0.f) ? 0.f : v;
    }
}

lancius_error done() { lcu_note_launch(); return lcu_launch_status(); }
lancius_error nul() { lancius_set_error(LANCIUS_ERROR_NULL_PTR); return LANCIUS_ERROR_NULL_PTR; }

}  // namespace

extern "C" {

lancius_error lcu_sum(float* out, const float* a, size_t n, void* s) {
    if (!out || !a) return nul();
    k_sum_all<<<1, 1024, 0, lcu_as_stream(s)>>>(out, a, n);
    return done();
}
lancius_error lcu_sum_axis0(float* out, const float* a, size_t R, size_t C, void* s) {
    if (!out || !a) return nul();
    if (!C) return LANCIUS_ERROR_OK;
    k_sum_axis0<<<lcu_blocks(C, 256), 256, 0, lcu_as_stream(s)>>>(out, a, R, C);
    return done();
}
lancius_error lcu_transpose(float* out, const float* a, size_t R, size_t C, void* s) {
    if (!out || !a) return nul();
    if (!R || !C) return LANCIUS_ERROR_OK;
    k_transpose<<<dim3((unsigned)((C + 31) / 32), (unsigned)((R + 31) / 32)), dim3(32, 8), 0, lcu_as_stream(s)>>>(out, a, R, C);
    return done();
}
lancius_error lcu_relu_bwd(float* out, const float* grad, const float* fwd, size_t n, void* s) {
    if (!out || !grad || !fwd) return nul();
    if (!n) return LANCIUS_ERROR_OK;
    k_relu_bwd<<<lcu_blocks(n, 1024), 256, 0, lcu_as_stream(s)>>>(out, grad, fwd, n);
    return done();
}
lancius_error lcu_softmax_bwd(float* out, const float* dy, const float* y, size_t R, size_t C, void* s) {
    if (!out || !dy || !y) return nul();
    if (!R) return LANCIUS_ERROR_OK;
    k_softmax_bwd<<<(unsigned)((R + 7) / 8), 256, 0, lcu_as_stream(s)>>>(out, dy, y, R, C);
    return done();
}
lancius_error lcu_cross_entropy(float* out, const float* x, const float* y, size_t R, size_t C, void* s) {
    if (!out || !x || !y) return nul();
    k_cross_entropy<<<1, 1024, 0, lcu_as_stream(s)>>>(out, x, y, R, C);
    return done();
}
lancius_error lcu_cross_entropy_bwd(float* out, const float* x, const float* y, const float* g, size_t R, size_t C, void* s) {
    if (!out || !x || !y || !g) return nul();
    if (!R) return LANCIUS_ERROR_OK;
    k_cross_entropy_bwd<<<(unsigned)((R + 7) / 8), 256, 0, lcu_as_stream(s)>>>(out, x, y, g, R, C);
    return done();
}
lancius_error lcu_rmsnorm(float* out, const float* in, const float* gamma, size_t R, size_t Hd, float eps, void* s) {
    if (!out || !in || !gamma) return nul();
    if (!R) return LANCIUS_ERROR_OK;
    k_rmsnorm<<<(unsigned)((R + 7) / 8), 256, 0, lcu_as_stream(s)>>>(out, in, gamma, R, Hd, eps);
    return done();
}
lancius_error lcu_swiglu(float* out, const float* gate, const float* up, size_t n, void* s) {
    if (!out || !gate || !up) return nul();
    if (!n) return LANCIUS_ERROR_OK;
    k_swiglu<<<lcu_blocks(n, 1024), 256, 0, lcu_as_stream(s)>>>(out, gate, up, n);
    return done();
}
lancius_error lcu_rope(float* q, float* k, size_t B, size_t S, size_t H, size_t D, int pos_offset, void* s) {
    if (!q || !k) return nul();
    if (D % 2) { lancius_set_error(LANCIUS_ERROR_SHAPE_MISMATCH); return LANCIUS_ERROR_SHAPE_MISMATCH; }
    if (!(B * S * H * D)) return LANCIUS_ERROR_OK;
    k_rope<<<lcu_blocks(B * S * H * D / 2, 256), 256, 0, lcu_as_stream(s)>>>(q, k, B, S, H, D, pos_offset);
    return done();
}
lancius_error lcu_maxpool2d_bwd(float* out, const float* grad, const float* in, size_t N, size_t C, size_t H, size_t W,
                                size_t K, size_t stride, void* s) {
    if (!out || !grad || !in) return nul();
    if (!K || !stride || H < K || W < K) { lancius_set_error(LANCIUS_ERROR_SHAPE_MISMATCH); return LANCIUS_ERROR_SHAPE_MISMATCH; }
    size_t Ho = (H - K) / stride + 1, Wo = (W - K) / stride + 1;
    k_maxpool_bwd<<<lcu_blocks(N * C * H * W, 256), 256, 0, lcu_as_stream(s)>>>(out, grad, in, N * C, (int)H, (int)W, (int)Ho,
                                                                              (int)Wo, (int)K, (int)stride);
    return done();
}
lancius_error lcu_conv2d_bwd(float* out, const float* grad, const float* w, size_t N, size_t Ci, size_t H, size_t W,
                             size_t Co, size_t Ho, size_t Wo, size_t Kh, size_t Kw, size_t stride, size_t pad, void* s) {
    if (!out || !grad || !w) return nul();
    if (!stride) { lancius_set_error(LANCIUS_ERROR_SHAPE_MISMATCH); return LANCIUS_ERROR_SHAPE_MISMATCH; }
    k_conv_bwd_in<<<lcu_blocks(N * Ci * H * W, 256), 256, 0, lcu_as_stream(s)>>>(out, grad, w, (int)N, (int)Ci, (int)H, (int)W,
                                                                               (int)Co, (int)Ho, (int)Wo, (int)Kh, (int)Kw,
                                                                               (int)stride, (int)pad);
    return done();
}
lancius_error lcu_conv2d_bwd_w(float* out, const float* grad, const float* in, size_t N, size_t Ci, size_t H, size_t W,
                               size_t Co, size_t Ho, size_t Wo, size_t Kh, size_t Kw, size_t stride, size_t pad, void* s) {
    if (!out || !grad || !in) return nul();
    size_t e = Co * Ci * Kh * Kw;
    if (!e) return LANCIUS_ERROR_OK;
    k_conv_bwd_w<<<(unsigned)e, 256, 0, lcu_as_stream(s)>>>(out, grad, in, (int)N, (int)Ci, (int)H, (int)W, (int)Co, (int)Ho,
                                                           (int)Wo, (int)Kh, (int)Kw, (int)stride, (int)pad);
    return done();
}
// INT8 weights (dtype INT8 + per-tensor scale). amax_scratch: one float of device memory.
lancius_error lcu_matmul_int8_simt(float* out, const float* a, const int8_t* b, double scale_b, size_t M, size_t K, size_t N,
                              float* amax_scratch, void* s) {
    if (!out || !a || !b || !amax_scratch) return nul();
    cudaStream_t st = lcu_as_stream(s);
    k_absmax<<<1, 1024, 0, st>>>(amax_scratch, a, M * K);
    lcu_note_launch();
    k_matmul_int8<<<lcu_blocks(M * N, 256), 256, 0, st>>>(out, a, b, amax_scratch, scale_b, M, K, N);
    return done();
}
lancius_error lcu_conv2d_int8_simt(float* out, const float* in, const int8_t* w, double scale_w, size_t N, size_t Ci, size_t H,
                              size_t W, size_t Co, size_t Kh, size_t Kw, size_t stride, size_t pad, int relu,
                              float* amax_scratch, void* s) {
    if (!out || !in || !w || !amax_scratch) return nul();
    if (!stride || H + 2 * pad < Kh || W + 2 * pad < Kw) { lancius_set_error(LANCIUS_ERROR_SHAPE_MISMATCH); return LANCIUS_ERROR_SHAPE_MISMATCH; }
    size_t Ho = (H + 2 * pad - Kh) / stride + 1, Wo = (W + 2 * pad - Kw) / stride + 1;
    cudaStream_t st = lcu_as_stream(s);
    k_absmax<<<1, 1024, 0, st>>>(amax_scratch, in, N * Ci * H * W);
    lcu_note_launch();
    k_conv_int8<<<lcu_blocks(N * Co * Ho * Wo, 256), 256, 0, st>>>(out, in, w, amax_scratch, scale_w, (int)N, (int)Ci, (int)H,
                                                                  (int)W, (int)Co, (int)Kh, (int)Kw, (int)stride, (int)pad,
                                                                  (int)Ho, (int)Wo, relu);
    return done();
}

}  // extern "C"
