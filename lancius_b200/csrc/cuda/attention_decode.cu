// KV-cache (decode) attention: one new query token per sequence against its cached
// keys and values. Restates kernel_attention_kv_cache (lancius_kernels.c:338-379):
// per head, scores q . k_j / sqrt(D) over all seq_len cached keys (no mask), softmax,
// then the probability-weighted sum of the cached values.
//
// The work is a stream over the caches (2 * seq_len * H * D floats per sequence,
// about one FLOP per byte), so the kernel is HBM-bound. Split-KV: the keys of each
// (sequence, head) are cut into `splits` chunks so that B * H * splits CTAs fill all
// SMs several times over; each CTA keeps an online softmax (m, l, o) per warp, merges
// its four warps in shared memory and writes a partial, and a second kernel merges
// the partials of a (sequence, head). With one split the first kernel writes the
// output directly. Layouts: q, out [B][H*D]; caches [B][seq_len][H][D].
#include "lcu_internal.h"

namespace {

constexpr int WARPS = 4, THREADS = 32 * WARPS;
constexpr int KEYS = 4;   // keys per warp iteration (their loads are in flight together)

__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// R = ceil(D / 32) values of a D-vector per lane (d = lane + 32 r)
template <int R>
__global__ void __launch_bounds__(THREADS) k_decode(const float* __restrict__ q, const float* __restrict__ k,
                                                    const float* __restrict__ v, float* __restrict__ out,
                                                    float* __restrict__ part, int S, int H, int D, int chunk,
                                                    float scale_log2) {
    __shared__ float sm_m[WARPS], sm_l[WARPS];
    __shared__ float sm_o[WARPS][32 * R];
    const int split = blockIdx.x, h = blockIdx.y, b = blockIdx.z, splits = gridDim.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const size_t hd = (size_t)H * D;
    const float* qp = q + (size_t)b * hd + (size_t)h * D;
    const float* kp = k + (size_t)b * S * hd + (size_t)h * D;
    const float* vp = v + (size_t)b * S * hd + (size_t)h * D;

    float qr[R], o[R];
#pragma unroll
    for (int r = 0; r < R; r++) {
        const int d = lane + 32 * r;
        qr[r] = d < D ? __ldg(qp + d) * scale_log2 : 0.f;   // scores come out in log2 units
        o[r] = 0.f;
    }
    float m = -INFINITY, l = 0.f;
    const int k_begin = split * chunk, k_end = min(S, k_begin + chunk);
    for (int j0 = k_begin + KEYS * warp; j0 < k_end; j0 += KEYS * WARPS) {
        float kv[KEYS][R], vv[KEYS][R], s[KEYS];
#pragma unroll
        for (int u = 0; u < KEYS; u++) {
            const bool in = j0 + u < k_end;
            const size_t row = (size_t)(j0 + u) * hd;
#pragma unroll
            for (int r = 0; r < R; r++) {
                const int d = lane + 32 * r;
                kv[u][r] = in && d < D ? __ldg(kp + row + d) : 0.f;
                vv[u][r] = in && d < D ? __ldg(vp + row + d) : 0.f;
            }
        }
#pragma unroll
        for (int u = 0; u < KEYS; u++) {
            float acc = 0.f;
#pragma unroll
            for (int r = 0; r < R; r++) acc = fmaf(qr[r], kv[u][r], acc);
            s[u] = acc;
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1)
#pragma unroll
            for (int u = 0; u < KEYS; u++) s[u] += __shfl_xor_sync(0xffffffffu, s[u], off);
        float mx = m;
#pragma unroll
        for (int u = 0; u < KEYS; u++) {
            if (j0 + u >= k_end) s[u] = -INFINITY;
            mx = fmaxf(mx, s[u]);
        }
        const float corr = ex2(m - mx);   // 0 while m is -inf
        l *= corr;
#pragma unroll
        for (int r = 0; r < R; r++) o[r] *= corr;
#pragma unroll
        for (int u = 0; u < KEYS; u++) {
            const float p = ex2(s[u] - mx);
            l += p;
#pragma unroll
            for (int r = 0; r < R; r++) o[r] = fmaf(p, vv[u][r], o[r]);
        }
        m = mx;
    }
    // merge the warps of this CTA
    if (lane == 0) { sm_m[warp] = m; sm_l[warp] = l; }
#pragma unroll
    for (int r = 0; r < R; r++) sm_o[warp][lane + 32 * r] = o[r];
    __syncthreads();
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < WARPS; w++) M = fmaxf(M, sm_m[w]);
    float wgt[WARPS], L = 0.f;
#pragma unroll
    for (int w = 0; w < WARPS; w++) {
        wgt[w] = sm_m[w] == -INFINITY ? 0.f : ex2(sm_m[w] - M);
        L += wgt[w] * sm_l[w];
    }
    for (int d = threadIdx.x; d < D; d += THREADS) {
        float acc = 0.f;
#pragma unroll
        for (int w = 0; w < WARPS; w++) acc += wgt[w] * sm_o[w][d];
        if (splits == 1) out[(size_t)b * hd + (size_t)h * D + d] = acc / L;
        else part[(((size_t)b * H + h) * splits + split) * (D + 2) + 2 + d] = acc;
    }
    if (splits > 1 && threadIdx.x == 0) {
        float* pp = part + (((size_t)b * H + h) * splits + split) * (D + 2);
        pp[0] = M;
        pp[1] = L;
    }
}

// out[b, h, :] = sum_s 2^(m_s - M) o_s / sum_s 2^(m_s - M) l_s
__global__ void __launch_bounds__(THREADS) k_decode_merge(const float* __restrict__ part, float* __restrict__ out,
                                                          int H, int D, int splits) {
    const int h = blockIdx.x, b = blockIdx.y;
    const float* pp = part + ((size_t)b * H + h) * splits * (D + 2);
    float M = -INFINITY;
    for (int s = 0; s < splits; s++) M = fmaxf(M, pp[(size_t)s * (D + 2)]);
    float L = 0.f;
    for (int s = 0; s < splits; s++) {
        const float ms = pp[(size_t)s * (D + 2)];
        if (ms != -INFINITY) L += ex2(ms - M) * pp[(size_t)s * (D + 2) + 1];
    }
    const float inv = 1.f / L;
    for (int d = threadIdx.x; d < D; d += THREADS) {
        float acc = 0.f;
        for (int s = 0; s < splits; s++) {
            const float ms = pp[(size_t)s * (D + 2)];
            if (ms != -INFINITY) acc += ex2(ms - M) * pp[(size_t)s * (D + 2) + 2 + d];
        }
        out[(size_t)b * H * D + (size_t)h * D + d] = acc * inv;
    }
}

}  // namespace

extern "C" lancius_error lcu_attention_kv_cache_batched(float* out, const float* q, const float* k_cache,
                                                        const float* v_cache, size_t batch, size_t seq_len,
                                                        size_t n_heads, size_t head_dim, void* stream) {
    if (batch == 0 || n_heads == 0 || head_dim == 0) return LANCIUS_ERROR_OK;
    if (seq_len == 0 || head_dim > 256 || seq_len > (size_t)INT32_MAX || batch > 65535 || n_heads > 65535) {
        lancius_set_error(LANCIUS_ERROR_SHAPE_MISMATCH);
        return LANCIUS_ERROR_SHAPE_MISMATCH;
    }
    const int S = (int)seq_len, H = (int)n_heads, D = (int)head_dim;
    // enough CTAs for ~8 per SM, each split at least 64 keys
    const size_t heads = batch * n_heads;
    size_t splits = (8 * (size_t)LCU_SMS + heads - 1) / heads;
    const size_t max_splits = (seq_len + 63) / 64;
    if (splits > max_splits) splits = max_splits;
    if (splits > 1024) splits = 1024;
    if (splits < 1) splits = 1;
    const int chunk = (int)((seq_len + splits - 1) / splits);
    splits = (seq_len + chunk - 1) / chunk;
    float* part = nullptr;
    if (splits > 1) {
        part = static_cast<float*>(lcu_scratch_acquire_decode(heads * splits * (head_dim + 2) * sizeof(float)));
        if (!part) { lancius_set_error(LANCIUS_ERROR_OOM); return LANCIUS_ERROR_OOM; }
    }
    const float scale_log2 = (float)(1.4426950408889634 / sqrt((double)head_dim));
    cudaStream_t st = lcu_as_stream(stream);
    const dim3 grid((unsigned)splits, (unsigned)H, (unsigned)batch);
    if (D <= 32) k_decode<1><<<grid, THREADS, 0, st>>>(q, k_cache, v_cache, out, part, S, H, D, chunk, scale_log2);
    else if (D <= 64) k_decode<2><<<grid, THREADS, 0, st>>>(q, k_cache, v_cache, out, part, S, H, D, chunk, scale_log2);
    else if (D <= 128) k_decode<4><<<grid, THREADS, 0, st>>>(q, k_cache, v_cache, out, part, S, H, D, chunk, scale_log2);
    else k_decode<8><<<grid, THREADS, 0, st>>>(q, k_cache, v_cache, out, part, S, H, D, chunk, scale_log2);
    lcu_note_launch();
    lancius_error e = lcu_launch_status();
    if (e != LANCIUS_ERROR_OK || splits == 1) return e;
    k_decode_merge<<<dim3((unsigned)H, (unsigned)batch), THREADS, 0, st>>>(part, out, H, D, (int)splits);
    lcu_note_launch();
    return lcu_launch_status();
}

extern "C" lancius_error lcu_attention_kv_cache(float* out, const float* q, const float* k_cache, const float* v_cache,
                                                size_t seq_len, size_t n_heads, size_t head_dim, void* stream) {
    return lcu_attention_kv_cache_batched(out, q, k_cache, v_cache, 1, seq_len, n_heads, head_dim, stream);
}
