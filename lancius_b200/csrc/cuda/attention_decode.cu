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


// D = 4 * G with G in {8, 16, 32}: a key row is read by G lanes as float4s, so one
// warp instruction covers 32 / G keys; U such instructions are in flight per
// iteration. Lanes of a key group share (m, l) and own 4 columns of o; the groups
// are merged with shuffles, then the warps through shared memory.
template <int G, int U>
__global__ void __launch_bounds__(THREADS) k_decode_vec(const float* __restrict__ q, const float* __restrict__ k,
                                                        const float* __restrict__ v, float* __restrict__ out,
                                                        float* __restrict__ part, int S, int H, int chunk,
                                                        float scale_log2) {
    constexpr int D = 4 * G, KPW = 32 / G, STEP = KPW * U;
    __shared__ float sm_m[WARPS], sm_l[WARPS];
    __shared__ float4 sm_o[WARPS][G];
    const int split = blockIdx.x, h = blockIdx.y, b = blockIdx.z, splits = gridDim.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int c4 = lane % G, kg = lane / G;            // float4 column, key slot in the warp
    const size_t hd = (size_t)H * D;
    const float4 qv = __ldg(reinterpret_cast<const float4*>(q + (size_t)b * hd + (size_t)h * D) + c4);
    const float qx = qv.x * scale_log2, qy = qv.y * scale_log2, qz = qv.z * scale_log2, qw = qv.w * scale_log2;
    const float* kp = k + (size_t)b * S * hd + (size_t)h * D + 4 * c4;
    const float* vp = v + (size_t)b * S * hd + (size_t)h * D + 4 * c4;
    float m = -INFINITY, l = 0.f;
    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
    const int k_begin = split * chunk, k_end = min(S, k_begin + chunk);
    for (int j0 = k_begin + STEP * warp; j0 < k_end; j0 += STEP * WARPS) {
        float4 kv[U], vv[U];
        float s[U];
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int j = j0 + u * KPW + kg;
            const bool in = j < k_end;
            kv[u] = in ? __ldg(reinterpret_cast<const float4*>(kp + (size_t)j * hd)) : make_float4(0.f, 0.f, 0.f, 0.f);
            vv[u] = in ? __ldg(reinterpret_cast<const float4*>(vp + (size_t)j * hd)) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int u = 0; u < U; u++) s[u] = fmaf(qx, kv[u].x, fmaf(qy, kv[u].y, fmaf(qz, kv[u].z, qw * kv[u].w)));
#pragma unroll
        for (int off = G / 2; off > 0; off >>= 1)
#pragma unroll
            for (int u = 0; u < U; u++) s[u] += __shfl_xor_sync(0xffffffffu, s[u], off);
        float mx = m;
#pragma unroll
        for (int u = 0; u < U; u++) {
            if (j0 + u * KPW + kg >= k_end) s[u] = -INFINITY;
            mx = fmaxf(mx, s[u]);
        }
        if (mx == -INFINITY) continue;                 // no key of this group in range
        const float corr = ex2(m - mx);
        l *= corr;
        o.x *= corr; o.y *= corr; o.z *= corr; o.w *= corr;
#pragma unroll
        for (int u = 0; u < U; u++) {
            const float p = ex2(s[u] - mx);
            l += p;
            o.x = fmaf(p, vv[u].x, o.x); o.y = fmaf(p, vv[u].y, o.y);
            o.z = fmaf(p, vv[u].z, o.z); o.w = fmaf(p, vv[u].w, o.w);
        }
        m = mx;
    }
    // merge the key groups of the warp (lanes c4, c4 + G, ...)
#pragma unroll
    for (int off = G; off < 32; off <<= 1) {
        const float m2 = __shfl_xor_sync(0xffffffffu, m, off), l2 = __shfl_xor_sync(0xffffffffu, l, off);
        float4 o2;
        o2.x = __shfl_xor_sync(0xffffffffu, o.x, off); o2.y = __shfl_xor_sync(0xffffffffu, o.y, off);
        o2.z = __shfl_xor_sync(0xffffffffu, o.z, off); o2.w = __shfl_xor_sync(0xffffffffu, o.w, off);
        const float M = fmaxf(m, m2);
        const float a = m == -INFINITY ? 0.f : ex2(m - M), c = m2 == -INFINITY ? 0.f : ex2(m2 - M);
        l = a * l + c * l2;
        o.x = a * o.x + c * o2.x; o.y = a * o.y + c * o2.y; o.z = a * o.z + c * o2.z; o.w = a * o.w + c * o2.w;
        m = M;
    }
    if (lane == 0) { sm_m[warp] = m; sm_l[warp] = l; }
    if (kg == 0) sm_o[warp][c4] = o;
    __syncthreads();
    if (threadIdx.x >= G) return;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < WARPS; w++) M = fmaxf(M, sm_m[w]);
    float L = 0.f;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int w = 0; w < WARPS; w++) {
        const float wgt = sm_m[w] == -INFINITY ? 0.f : ex2(sm_m[w] - M);
        L += wgt * sm_l[w];
        const float4 ow = sm_o[w][threadIdx.x];
        acc.x += wgt * ow.x; acc.y += wgt * ow.y; acc.z += wgt * ow.z; acc.w += wgt * ow.w;
    }
    const int d = 4 * threadIdx.x;
    if (splits == 1) {
        const float inv = 1.f / L;
        *reinterpret_cast<float4*>(out + (size_t)b * hd + (size_t)h * D + d) =
            make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
    } else {
        float* pp = part + (((size_t)b * H + h) * splits + split) * (D + 2);
        pp[2 + d] = acc.x; pp[3 + d] = acc.y; pp[4 + d] = acc.z; pp[5 + d] = acc.w;
        if (threadIdx.x == 0) { pp[0] = M; pp[1] = L; }
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
    // about eight waves of CTAs (tail under ~1/8 of a wave), each split at least 64 keys
    const bool vec = (D == 32 || D == 64 || D == 128) && ((uintptr_t)q % 16 == 0) && ((uintptr_t)k_cache % 16 == 0) &&
                     ((uintptr_t)v_cache % 16 == 0) && ((uintptr_t)out % 16 == 0);
    static int resident[64] = {};   // CTAs per SM, per device
    int dev = 0;
    cudaGetDevice(&dev);
    int per_sm = dev >= 0 && dev < 64 ? resident[dev] : 0;
    if (!per_sm) {
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_decode_vec<32, 4>, THREADS, 0) != cudaSuccess ||
            per_sm <= 0)
            per_sm = 4;
        if (dev >= 0 && dev < 64) resident[dev] = per_sm;
    }
    const size_t heads = batch * n_heads;
    size_t splits = (8 * (size_t)LCU_SMS * per_sm + heads - 1) / heads;
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
    if (vec && D == 32) k_decode_vec<8, 2><<<grid, THREADS, 0, st>>>(q, k_cache, v_cache, out, part, S, H, chunk, scale_log2);
    else if (vec && D == 64) k_decode_vec<16, 4><<<grid, THREADS, 0, st>>>(q, k_cache, v_cache, out, part, S, H, chunk, scale_log2);
    else if (vec && D == 128) k_decode_vec<32, 4><<<grid, THREADS, 0, st>>>(q, k_cache, v_cache, out, part, S, H, chunk, scale_log2);
    else if (D <= 32) k_decode<1><<<grid, THREADS, 0, st>>>(q, k_cache, v_cache, out, part, S, H, D, chunk, scale_log2);
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
