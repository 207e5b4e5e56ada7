// Flash-style attention on CUDA cores (FP32 FFMA), the portable path:
// one CTA per (64-query tile, head, batch element), K/V streamed through shared
// memory in 64-key tiles, online softmax with 16-lane shuffle reductions, and the
// score matrix never written to HBM. Restates kernel_attention
// (lancius_kernels.c:278-332): scale 1/sqrt(D), causal mask j > i.
#include "lcu_internal.h"


namespace {

constexpr int BQ = 64, BKV = 64, THREADS = 256;

template <int D>
__global__ void __launch_bounds__(THREADS) k_attn_simt(const LcuAttnGroup* __restrict__ table, LcuAttnGroup base,
                                                       size_t batch_stride, int S, int H, int causal, float scale_log2,
                                                       int Hkv) {
    extern __shared__ float4 smem4[];
    float* smem = reinterpret_cast<float*>(smem4);
    float* Qs = smem;                 // [D][BQ]
    float* Ks = Qs + D * BQ;          // [D][BKV]
    float* Vs = Ks + D * BKV;         // [BKV][D]
    float* Ps = Vs + BKV * D;         // [BKV][BQ]

    LcuAttnGroup p;
    if (table) p = table[blockIdx.z];
    else {
        size_t off = (size_t)blockIdx.z * batch_stride;
        p.q = base.q + off; p.k = base.k + off; p.v = base.v + off; p.o = base.o + off;
    }
    const int h = blockIdx.y, q0 = blockIdx.x * BQ;
    const int hk = h / (H / Hkv);                      // grouped-query: kv head of this query head
    const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
    const size_t row_stride = (size_t)H * D, kv_stride = (size_t)Hkv * D;
    constexpr int DC = D / 16;        // output columns per thread

    // stage Q (transposed into [d][r])
    for (int idx = tid; idx < BQ * D / 4; idx += THREADS) {
        int r = idx / (D / 4), d4 = (idx % (D / 4)) * 4;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (q0 + r < S) v = __ldg(reinterpret_cast<const float4*>(p.q + (size_t)(q0 + r) * row_stride + (size_t)h * D + d4));
        Qs[(d4 + 0) * BQ + r] = v.x; Qs[(d4 + 1) * BQ + r] = v.y; Qs[(d4 + 2) * BQ + r] = v.z; Qs[(d4 + 3) * BQ + r] = v.w;
    }

    float m[4], l[4], o[4][DC];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        m[i] = -INFINITY; l[i] = 0.f;
#pragma unroll
        for (int c = 0; c < DC; c++) o[i][c] = 0.f;
    }

    int kv_end = causal ? min(S, q0 + BQ) : S;
    for (int k0 = 0; k0 < kv_end; k0 += BKV) {
        __syncthreads();
        for (int idx = tid; idx < BKV * D / 4; idx += THREADS) {
            int j = idx / (D / 4), d4 = (idx % (D / 4)) * 4;
            float4 kv = make_float4(0.f, 0.f, 0.f, 0.f), vv = kv;
            if (k0 + j < S) {
                size_t g = (size_t)(k0 + j) * kv_stride + (size_t)hk * D + d4;
                kv = __ldg(reinterpret_cast<const float4*>(p.k + g));
                vv = __ldg(reinterpret_cast<const float4*>(p.v + g));
            }
            Ks[(d4 + 0) * BKV + j] = kv.x; Ks[(d4 + 1) * BKV + j] = kv.y; Ks[(d4 + 2) * BKV + j] = kv.z; Ks[(d4 + 3) * BKV + j] = kv.w;
            *reinterpret_cast<float4*>(Vs + j * D + d4) = vv;
        }
        __syncthreads();

        float s[4][4];
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int j = 0; j < 4; j++) s[i][j] = 0.f;
#pragma unroll 8
        for (int d = 0; d < D; d++) {
            float4 a = *reinterpret_cast<const float4*>(Qs + d * BQ + ty * 4);
            float4 b = *reinterpret_cast<const float4*>(Ks + d * BKV + tx * 4);
            float av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int j = 0; j < 4; j++) s[i][j] = fmaf(av[i], bv[j], s[i][j]);
        }
        // mask + online softmax (log2 domain)
#pragma unroll
        for (int i = 0; i < 4; i++) {
            int qi = q0 + ty * 4 + i;
            float mx = -INFINITY;
#pragma unroll
            for (int j = 0; j < 4; j++) {
                int kj = k0 + tx * 4 + j;
                float v = s[i][j] * scale_log2;
                if (kj >= S || (causal && kj > qi)) v = -INFINITY;
                s[i][j] = v;
                mx = fmaxf(mx, v);
            }
#pragma unroll
            for (int off = 8; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
            float mn = fmaxf(m[i], mx);
            float alpha = exp2f(m[i] - mn);
            float rs = 0.f;
#pragma unroll
            for (int j = 0; j < 4; j++) { float e = exp2f(s[i][j] - mn); s[i][j] = e; rs += e; }
#pragma unroll
            for (int off = 8; off > 0; off >>= 1) rs += __shfl_xor_sync(0xffffffffu, rs, off);
            l[i] = l[i] * alpha + rs;
            m[i] = mn;
#pragma unroll
            for (int c = 0; c < DC; c++) o[i][c] *= alpha;
        }
#pragma unroll
        for (int j = 0; j < 4; j++)
            *reinterpret_cast<float4*>(Ps + (tx * 4 + j) * BQ + ty * 4) = make_float4(s[0][j], s[1][j], s[2][j], s[3][j]);
        __syncthreads();
#pragma unroll 4
        for (int j = 0; j < BKV; j++) {
            float4 a = *reinterpret_cast<const float4*>(Ps + j * BQ + ty * 4);
            float av[4] = {a.x, a.y, a.z, a.w};
            float bv[DC];
#pragma unroll
            for (int c = 0; c < DC; c += 4) {
                float4 b = *reinterpret_cast<const float4*>(Vs + j * D + tx * DC + c);
                bv[c] = b.x; bv[c + 1] = b.y; bv[c + 2] = b.z; bv[c + 3] = b.w;
            }
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int c = 0; c < DC; c++) o[i][c] = fmaf(av[i], bv[c], o[i][c]);
        }
    }
#pragma unroll
    for (int i = 0; i < 4; i++) {
        int qi = q0 + ty * 4 + i;
        if (qi >= S) continue;
        float inv = 1.f / l[i];
        float* dst = p.o + (size_t)qi * row_stride + (size_t)h * D + tx * DC;
#pragma unroll
        for (int c = 0; c < DC; c += 4)
            *reinterpret_cast<float4*>(dst + c) = make_float4(o[i][c] * inv, o[i][c + 1] * inv, o[i][c + 2] * inv, o[i][c + 3] * inv);
    }
}

template <int D>
lancius_error launch(const LcuAttnGroup* table, LcuAttnGroup base, size_t bstride, int B, int S, int H, int causal,
                     cudaStream_t st, int Hkv) {
    size_t smem = sizeof(float) * (size_t)(2 * D * BQ + BKV * D + BKV * BQ);
    static bool configured[64] = {};   // the attribute is per device
    int dev_ = 0;
    cudaGetDevice(&dev_);
    if (dev_ >= 0 && dev_ < 64 && !configured[dev_]) {
        cudaFuncSetAttribute(k_attn_simt<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        configured[dev_] = true;
    }
    float scale_log2 = (float)(1.4426950408889634 / sqrt((double)D));
    dim3 grid((unsigned)((S + BQ - 1) / BQ), (unsigned)H, (unsigned)B);
    k_attn_simt<D><<<grid, THREADS, smem, st>>>(table, base, bstride, S, H, causal, scale_log2, Hkv);
    lcu_note_launch();
    return lcu_launch_status();
}

}  // namespace

extern "C" lancius_error lcu_attention_simt(const LcuAttnGroup* d_table, const float* q, const float* k, const float* v,
                                            float* o, size_t B, size_t S, size_t H, size_t D, int causal, void* stream) {
    if (B == 0 || S == 0 || H == 0) return LANCIUS_ERROR_OK;
    if (!d_table && (((uintptr_t)q | (uintptr_t)k | (uintptr_t)v | (uintptr_t)o) & 15u)) {
        lancius_set_error(LANCIUS_ERROR_UNSUPPORTED_DTYPE);   // float4 IO needs 16-byte aligned rows
        return LANCIUS_ERROR_UNSUPPORTED_DTYPE;
    }
    LcuAttnGroup base{q, k, v, o};
    size_t bstride = S * H * D;
    cudaStream_t st = lcu_as_stream(stream);
    switch (D) {
        case 64: return launch<64>(d_table, base, bstride, (int)B, (int)S, (int)H, causal, st, (int)H);
        case 128: return launch<128>(d_table, base, bstride, (int)B, (int)S, (int)H, causal, st, (int)H);
        default: lancius_set_error(LANCIUS_ERROR_UNSUPPORTED_OP); return LANCIUS_ERROR_UNSUPPORTED_OP;
    }
}

// Grouped-query attention (kernel_gqa, lancius_kernels.c:407-448): causal, query head h
// reads kv head h / (Hq / Hkv); q/out [S, Hq, D], k/v [S, Hkv, D].
extern "C" lancius_error lcu_gqa(float* o, const float* q, const float* k, const float* v, size_t S, size_t Hq,
                                 size_t Hkv, size_t D, void* stream) {
    if (!o || !q || !k || !v) { lancius_set_error(LANCIUS_ERROR_NULL_PTR); return LANCIUS_ERROR_NULL_PTR; }
    if (Hkv == 0 || Hq % Hkv) { lancius_set_error(LANCIUS_ERROR_SHAPE_MISMATCH); return LANCIUS_ERROR_SHAPE_MISMATCH; }
    if ((((uintptr_t)q | (uintptr_t)k | (uintptr_t)v | (uintptr_t)o) & 15u)) {
        lancius_set_error(LANCIUS_ERROR_UNSUPPORTED_DTYPE);
        return LANCIUS_ERROR_UNSUPPORTED_DTYPE;
    }
    if (S == 0) return LANCIUS_ERROR_OK;
    LcuAttnGroup base{q, k, v, o};
    cudaStream_t st = lcu_as_stream(stream);
    switch (D) {
        case 64: return launch<64>(nullptr, base, 0, 1, (int)S, (int)Hq, 1, st, (int)Hkv);
        case 128: return launch<128>(nullptr, base, 0, 1, (int)S, (int)Hq, 1, st, (int)Hkv);
        default: lancius_set_error(LANCIUS_ERROR_UNSUPPORTED_OP); return LANCIUS_ERROR_UNSUPPORTED_OP;
    }
}
