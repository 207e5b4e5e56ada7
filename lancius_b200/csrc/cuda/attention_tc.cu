// Flash attention on the tcgen05 tensor cores, FP32-exact (3xTF32), head_dim 64.
// Restates kernel_attention (lancius_kernels.c:278-332): per query row an online
// softmax over all keys (causal: keys j > i masked), scale 1/sqrt(D); the score
// matrix never leaves the SM.
//
// One CTA = (128-query tile, head, batch element). Roles:
//   warps 0-3  softmax: one query row per thread (= its TMEM lane). Loads the Q row
//              and splits it into TF32 hi/lo TMEM columns; per key tile reads S,
//              writes P = exp2(S - m) as hi/lo TMEM columns and keeps the row sum.
//              The running max m is only raised when a tile's max exceeds it by more
//              than 2^8 (then the O accumulator in TMEM is rescaled); any fixed offset
//              gives the same softmax, so this is exact, and P stays <= 256.
//   warp 4     TMEM allocation + MMA issue (one lane), in the order
//                S_0, S_1, PV_0, S_2, PV_1, ...
//              S_j = Q K_j^T (A = Q from TMEM), O += P_j V_j (A = P_j from TMEM).
//              tcgen05 costs about the same per instruction whatever its N, so the
//              hi/lo halves of B are concatenated along N: Q_hi*[K_hi|K_lo] (N = 128)
//              and Q_lo*K_hi (N = 64) accumulate Q_hi K_hi + Q_lo K_hi in the left and
//              Q_hi K_lo in the right half of S, and S = left + right; same for
//              P_hi*[V_hi|V_lo] and P_lo*V_hi into O
//   warps 5-8  loaders: K_j, V_j from global (coalesced float4, next tile prefetched
//              into registers), split hi/lo, stored in the swizzled layouts tcgen05
//              reads (K: K-major 128B swizzle; V: N-major 128B swizzle, 32B atoms)
// TMEM columns: Q hi [0,64) lo [64,128); S halves [128,256); O halves [256,384);
// P hi [384,448) lo [448,512). Every mbarrier wait is bounded.
#include "tc_common.cuh"

namespace {

constexpr int D = 64, BQ = 128, BKV = 64, NS = 2;
constexpr int THREADS = 288;
constexpr int KV_HALF = BKV * D * 4;            // 16 KB: one hi or lo tile
constexpr int STAGE = 2 * KV_HALF;              // hi + lo
constexpr int SMEM_BYTES = 2 * NS * STAGE + 1024 + 512;
constexpr uint32_t TM_QHI = 0, TM_QLO = 64, TM_S = 128, TM_O = 256, TM_P = 384, TM_COLS = 512;
constexpr float RESCALE_THRESHOLD = 8.0f;       // log2 units

__device__ int g_attn_watchdog = 0;

// Optional per-CTA phase timestamps (%globaltimer) for tuning; compiled out unless
// built with -DLCU_ATTN_TRACE=1.
#ifndef LCU_ATTN_TRACE
#define LCU_ATTN_TRACE 0
#endif
#if LCU_ATTN_TRACE
__device__ unsigned long long g_trace[512][64];
__device__ __forceinline__ unsigned long long gtime() { unsigned long long t; asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t)); return t; }
#define TRACE(slot) do { unsigned cta = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z); if (cta < 512 && (slot) < 64) g_trace[cta][slot] = gtime(); } while (0)
#else
#define TRACE(slot) do {} while (0)
#endif

struct Bars {
    uint64_t k_full[NS], k_empty[NS], v_full[NS], v_empty[NS];
    uint64_t s_full, s_free, q_ready, o_free, drain;
    uint64_t p_ready, pv_done;
    uint32_t tmem;
    int abort;
};

// K stage: per 32-d atom, 128 rows of 128 B: rows 0-63 = K_hi keys, rows 64-127 = K_lo keys
// (K-major, 128B swizzle), so one descriptor spans [K_hi | K_lo] as N = 128.
__device__ __forceinline__ uint32_t k_off(int row, int d) {
    return (uint32_t)((d >> 5) * (2 * BKV * 128) + row * 128 + ((((d & 31) >> 2) ^ (row & 7)) << 4));
}
// V stage: 32-d chunks of 64 key rows (N-major, 128B swizzle of 32B atoms); V_hi fills
// chunks 0-1 and V_lo chunks 2-3, so one descriptor spans [V_hi | V_lo] as N = 128.
__device__ __forceinline__ uint32_t v_off(int j, int d) {
    return (uint32_t)((d >> 5) * (BKV * 128) + j * 128 + ((((d & 31) >> 3) ^ (j & 3)) << 5) + ((d & 7) << 2));
}
// TF32 split: hi keeps the top 10 mantissa bits (exactly what the tensor core reads),
// lo = x - hi is exact in FP32 and carries the next bits.
__device__ __forceinline__ float hi_part(float x) { return __uint_as_float(__float_as_uint(x) & 0xFFFFE000u); }
__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

struct Item { LcuAttnGroup p; int h, q0, T; bool valid; };

// Work slots of the persistent grid. Causal cost grows with the query tile index, so
// tile qt is paired with tile nqt-1-qt: slot 2p is the heavy member of pair p, slot
// 2p+1 the light one (empty for the middle tile of an odd nqt), and every pair costs
// the same number of key tiles. A CTA takes both slots of a pair, then strides by the
// grid over pairs; pairs are ordered so the light (unpaired) ones come last.
__device__ __forceinline__ int next_slot(int x) { return (x & 1) ? x - 1 + 2 * (int)gridDim.x : x + 1; }

__device__ __forceinline__ Item get_item(int x, const LcuAttnGroup* table, const LcuAttnGroup& base, size_t bstride,
                                         int B, int H, int nqt, int S, int causal) {
    Item it;
    const int per = B * H;
    const int pair = x >> 1, qp = pair / per, r = pair % per, b = r / H;
    const int qt = (x & 1) ? qp : nqt - 1 - qp;
    it.valid = !((x & 1) && qt == nqt - 1 - qp);
    it.h = r % H;
    if (table) it.p = table[b];
    else {
        size_t off = (size_t)b * bstride;
        it.p.q = base.q + off; it.p.k = base.k + off; it.p.v = base.v + off; it.p.o = base.o + off;
    }
    it.q0 = qt * BQ;
    const int kv_end = causal ? min(S, it.q0 + BQ) : S;
    it.T = (kv_end + BKV - 1) / BKV;
    return it;
}

__global__ void __launch_bounds__(THREADS, 1)
k_attn_tc(const LcuAttnGroup* __restrict__ table, LcuAttnGroup base, size_t bstride, int B, int S, int H, int causal,
          float scale_log2) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* tiles = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* kst = tiles;                          // NS stages of K hi|lo
    uint8_t* vst = tiles + NS * STAGE;             // NS stages of V hi|lo
    Bars* bar = reinterpret_cast<Bars*>(tiles + 2 * NS * STAGE);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nqt = (S + BQ - 1) / BQ;
    const int n_slots = 2 * ((nqt + 1) / 2) * B * H;
    const size_t rs = (size_t)H * D;                // row stride of [S, H, D]
    volatile int* abort = &bar->abort;

    if (threadIdx.x == 0) {
        for (int s = 0; s < NS; s++) {
            tc::mbar_init(&bar->k_full[s], 128); tc::mbar_init(&bar->k_empty[s], 1);
            tc::mbar_init(&bar->v_full[s], 128); tc::mbar_init(&bar->v_empty[s], 1);
        }
        tc::mbar_init(&bar->s_full, 1);
        tc::mbar_init(&bar->s_free, 128);
        tc::mbar_init(&bar->q_ready, 128);
        tc::mbar_init(&bar->o_free, 128);
        tc::mbar_init(&bar->p_ready, 128);
        tc::mbar_init(&bar->pv_done, 1);
        tc::mbar_init(&bar->drain, 1);
        bar->abort = 0;
        tc::fence_barrier_init();
    }
    if (warp == 4) tc::tmem_alloc(&bar->tmem, TM_COLS);
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tm = bar->tmem;
    if (threadIdx.x == 0) TRACE(0);

    // Every role walks the same item sequence; `gt` numbers this CTA's key tiles across
    // items and drives all ring stages and barrier phases.
    if (warp < 4) {
        // ======================= softmax warps =======================
        const int row = 32 * warp + lane;              // TMEM lane == query row in tile
        const uint32_t lb = tm + ((uint32_t)(32 * warp) << 16);
        int gt = 0;
        bool ok = true;
        for (int x = 2 * (int)blockIdx.x; x < n_slots && ok; x = next_slot(x)) {
            const Item it = get_item(x, table, base, bstride, B, H, nqt, S, causal);
            if (!it.valid) continue;
            const int qi = it.q0 + row;
            {   // Q row -> TMEM hi/lo (the previous item is fully read out at this point)
                float hi[32], lo[32];
#pragma unroll 1
                for (int half = 0; half < 2; half++) {
                    const float4* src = reinterpret_cast<const float4*>(it.p.q + (size_t)qi * rs + (size_t)it.h * D + half * 32);
#pragma unroll
                    for (int c = 0; c < 8; c++) {
                        float4 v = qi < S ? __ldg(src + c) : make_float4(0.f, 0.f, 0.f, 0.f);
                        float x[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                        for (int t = 0; t < 4; t++) { hi[4 * c + t] = hi_part(x[t]); lo[4 * c + t] = x[t] - hi[4 * c + t]; }
                    }
                    tc::tmem_st32(lb + TM_QHI + half * 32, hi);
                    tc::tmem_st32(lb + TM_QLO + half * 32, lo);
                }
                tc::tmem_st_wait();
                tc::tc_fence_before();
                tc::mbar_arrive(&bar->q_ready);
                if (threadIdx.x == 0) TRACE(1);
            }
            float m = -INFINITY, l = 0.f;
            for (int j = 0; j < it.T; j++, gt++) {
                if (!tc::mbar_wait(&bar->s_full, gt & 1, abort, &g_attn_watchdog, 11)) { ok = false; break; }
                if (threadIdx.x == 0 && gt < 8) TRACE(2 + 4 * gt);
                tc::tc_fence_after();
                float s[64];
#pragma unroll
                for (int half = 0; half < 2; half++) {
                    float a[32], b[32];
                    tc::tmem_ld32(lb + TM_S + half * 32, a);         // Q_hi K_hi + Q_lo K_hi
                    tc::tmem_ld32(lb + TM_S + 64 + half * 32, b);    // Q_hi K_lo
#pragma unroll
                    for (int c = 0; c < 32; c++) s[half * 32 + c] = (a[c] + b[c]) * scale_log2;
                }
                tc::tc_fence_before();
                tc::mbar_arrive(&bar->s_free);               // the MMA warp may overwrite S now
                const int k0 = j * BKV;
                if (k0 + BKV > S || (causal && k0 + BKV - 1 > it.q0)) {   // tile touches the diagonal or the end
#pragma unroll
                    for (int c = 0; c < 64; c++)
                        if (k0 + c >= S || (causal && k0 + c > qi)) s[c] = -INFINITY;
                }
                float mx4[4] = {s[0], s[1], s[2], s[3]};      // 4 independent chains
#pragma unroll
                for (int c = 4; c < 64; c++) mx4[c & 3] = fmaxf(mx4[c & 3], s[c]);
                const float mx = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3]));
                const bool raise = mx > m + RESCALE_THRESHOLD;
                if (__any_sync(0xffffffffu, raise)) {
                    const float mn = raise ? mx : m;
                    const float f = ex2(m - mn);             // 0 on the first tile, 1 for rows that keep m
                    if (j > 0) {   // O holds this item's P_0..P_{j-1} V: wait for it, rescale moved rows
                        if (!tc::mbar_wait(&bar->pv_done, (gt - 1) & 1, abort, &g_attn_watchdog, 12)) { ok = false; break; }
                        tc::tc_fence_after();
#pragma unroll 1
                        for (int q4 = 0; q4 < 4; q4++) {
                            float o[32];
                            tc::tmem_ld32(lb + TM_O + q4 * 32, o);
#pragma unroll
                            for (int c = 0; c < 32; c++) o[c] *= f;
                            tc::tmem_st32(lb + TM_O + q4 * 32, o);
                        }
                        tc::tmem_st_wait();
                    }
                    l *= f;
                    m = mn;
                }
                if (threadIdx.x == 0 && gt < 8) TRACE(3 + 4 * gt);
                float rs4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                for (int c = 0; c < 64; c++) { s[c] = ex2(s[c] - m); rs4[c & 3] += s[c]; }
                l += (rs4[0] + rs4[1]) + (rs4[2] + rs4[3]);
                // the P columns were last read by PV of tile gt-1 (exponentials above overlap it)
                if (j >= 1 && !tc::mbar_wait(&bar->pv_done, (gt - 1) & 1, abort, &g_attn_watchdog, 14)) { ok = false; break; }
#pragma unroll
                for (int half = 0; half < 2; half++) {
                    float hi[32], lo[32];
#pragma unroll
                    for (int c = 0; c < 32; c++) { hi[c] = hi_part(s[half * 32 + c]); lo[c] = s[half * 32 + c] - hi[c]; }
                    tc::tmem_st32(lb + TM_P + half * 32, hi);
                    tc::tmem_st32(lb + TM_P + 64 + half * 32, lo);
                }
                if (threadIdx.x == 0 && gt < 8) TRACE(4 + 4 * gt);
                tc::tmem_st_wait();
                tc::tc_fence_before();
                tc::mbar_arrive(&bar->p_ready);
                if (threadIdx.x == 0 && gt < 8) TRACE(5 + 4 * gt);
            }
            if (!ok) break;
            if (it.T > 0) {
                if (!tc::mbar_wait(&bar->pv_done, (gt - 1) & 1, abort, &g_attn_watchdog, 13)) { ok = false; break; }
                tc::tc_fence_after();
                const float inv = 1.f / l;
#pragma unroll 1
                for (int half = 0; half < 2; half++) {
                    float o[32], o2[32];
                    tc::tmem_ld32(lb + TM_O + half * 32, o);         // P_hi V_hi + P_lo V_hi
                    tc::tmem_ld32(lb + TM_O + 64 + half * 32, o2);   // P_hi V_lo
                    if (qi < S) {
                        float4* dst = reinterpret_cast<float4*>(it.p.o + (size_t)qi * rs + (size_t)it.h * D + half * 32);
#pragma unroll
                        for (int c = 0; c < 8; c++)
                            dst[c] = make_float4((o[4 * c] + o2[4 * c]) * inv, (o[4 * c + 1] + o2[4 * c + 1]) * inv,
                                                 (o[4 * c + 2] + o2[4 * c + 2]) * inv, (o[4 * c + 3] + o2[4 * c + 3]) * inv);
                    }
                }
            }
            tc::tc_fence_before();
            tc::mbar_arrive(&bar->o_free);                   // O (and Q) columns reusable
        }
    } else if (warp == 4) {
        // ======================= MMA issuer =======================
        if (lane == 0) {
            constexpr uint32_t id_s = tc::idesc_tf32(BQ, 2 * BKV, false, false);
            constexpr uint32_t id_o = tc::idesc_tf32(BQ, 2 * D, false, true);
            // the lo x lo product is below FP32 resolution: the lo operand multiplies only
            // the hi half of B (N = 64)
            constexpr uint32_t id_s_lo = tc::idesc_tf32(BQ, BKV, false, false);
            constexpr uint32_t id_o_lo = tc::idesc_tf32(BQ, D, false, true);
            bool ok = true;
            int gt = 0, ii = 0;
            auto issue_s = [&](int g) -> bool {
                const int st = g % NS;
                if (!tc::mbar_wait(&bar->k_full[st], (g / NS) & 1, abort, &g_attn_watchdog, 22)) return false;
                if (g >= 1 && !tc::mbar_wait(&bar->s_free, (g - 1) & 1, abort, &g_attn_watchdog, 23)) return false;
                tc::tc_fence_after();
                const uint32_t kb0 = tc::smem_u32(kst + st * STAGE);
#pragma unroll
                for (int kb = 0; kb < D / 8; kb++) {
                    const uint32_t off = (uint32_t)((kb >> 2) * (2 * BKV * 128) + (kb & 3) * 32);
                    const uint64_t bk = tc::smem_desc(kb0 + off, 16, 1024, tc::SWZ_128B);   // [K_hi | K_lo]
                    tc::mma_tf32_ts(tm + TM_S, tm + TM_QHI + kb * 8, bk, id_s, kb ? 1u : 0u);
                    tc::mma_tf32_ts(tm + TM_S, tm + TM_QLO + kb * 8, bk, id_s_lo, 1u);
                }
                tc::mma_commit(&bar->s_full);
                tc::mma_commit(&bar->k_empty[st]);
                if (g < 8) TRACE(34 + g);
                return true;
            };
            for (int x = 2 * (int)blockIdx.x; x < n_slots && ok; x = next_slot(x)) {
                const Item it = get_item(x, table, base, bstride, B, H, nqt, S, causal);
                if (!it.valid) continue;
                if (!tc::mbar_wait(&bar->q_ready, ii & 1, abort, &g_attn_watchdog, 21)) { ok = false; break; }
                if (it.T > 0 && !(ok = issue_s(gt))) break;
                for (int j = 0; j < it.T; j++, gt++) {
                    if (j + 1 < it.T && !(ok = issue_s(gt + 1))) break;
                    const int st = gt % NS;
                    if (!tc::mbar_wait(&bar->p_ready, gt & 1, abort, &g_attn_watchdog, 24) ||
                        !tc::mbar_wait(&bar->v_full[st], (gt / NS) & 1, abort, &g_attn_watchdog, 25)) { ok = false; break; }
                    // the first PV of an item overwrites O: the previous item's O must have been read
                    if (j == 0 && ii >= 1 && !tc::mbar_wait(&bar->o_free, (ii - 1) & 1, abort, &g_attn_watchdog, 26)) { ok = false; break; }
                    tc::tc_fence_after();
                    const uint32_t vb0 = tc::smem_u32(vst + st * STAGE);
#pragma unroll
                    for (int kb = 0; kb < BKV / 8; kb++) {
                        const uint64_t bv = tc::smem_desc(vb0 + kb * 1024, BKV * 128, 512, tc::SWZ_128B_BASE32B);   // [V_hi | V_lo]
                        const uint32_t acc0 = (j | kb) ? 1u : 0u;
                        tc::mma_tf32_ts(tm + TM_O, tm + TM_P + kb * 8, bv, id_o, acc0);
                        tc::mma_tf32_ts(tm + TM_O, tm + TM_P + 64 + kb * 8, bv, id_o_lo, 1u);
                    }
                    tc::mma_commit(&bar->pv_done);
                    tc::mma_commit(&bar->v_empty[st]);
                    if (gt < 8) TRACE(42 + gt);
                }
                ii++;
            }
        }
    } else {
        // ======================= loaders (warps 5-8) =======================
        const int t = threadIdx.x - 160;                 // 0..127
        const int jr = t >> 1, d0 = (t & 1) * 32;        // key row within tile, d half
        int gt = 0;
        bool ok = true;
        for (int x = 2 * (int)blockIdx.x; x < n_slots && ok; x = next_slot(x)) {
            const Item it = get_item(x, table, base, bstride, B, H, nqt, S, causal);
            if (!it.valid) continue;
            float4 kv[8], vv[8];
            auto fetch = [&](int j) {
                const int key = j * BKV + jr;
                const float4* ks = reinterpret_cast<const float4*>(it.p.k + (size_t)key * rs + (size_t)it.h * D + d0);
                const float4* vs = reinterpret_cast<const float4*>(it.p.v + (size_t)key * rs + (size_t)it.h * D + d0);
#pragma unroll
                for (int c = 0; c < 8; c++) {
                    kv[c] = key < S ? __ldg(ks + c) : make_float4(0.f, 0.f, 0.f, 0.f);
                    vv[c] = key < S ? __ldg(vs + c) : make_float4(0.f, 0.f, 0.f, 0.f);
                }
            };
            if (it.T > 0) fetch(0);
            for (int j = 0; j < it.T; j++, gt++) {
                const int st = gt % NS;
                float4 kn[8], vn[8];
#pragma unroll
                for (int c = 0; c < 8; c++) { kn[c] = kv[c]; vn[c] = vv[c]; }
                if (j + 1 < it.T) fetch(j + 1);              // next tile in flight while this one is stored
                if (gt >= NS && !tc::mbar_wait(&bar->k_empty[st], ((gt / NS) - 1) & 1, abort, &g_attn_watchdog, 31)) { ok = false; break; }
                uint8_t* kh = kst + st * STAGE;
#pragma unroll
                for (int c = 0; c < 8; c++) {
                    float x[4] = {kn[c].x, kn[c].y, kn[c].z, kn[c].w}, hi[4], lo[4];
#pragma unroll
                    for (int u = 0; u < 4; u++) { hi[u] = hi_part(x[u]); lo[u] = x[u] - hi[u]; }
                    *reinterpret_cast<float4*>(kh + k_off(jr, d0 + 4 * c)) = make_float4(hi[0], hi[1], hi[2], hi[3]);
                    *reinterpret_cast<float4*>(kh + k_off(jr + BKV, d0 + 4 * c)) = make_float4(lo[0], lo[1], lo[2], lo[3]);
                }
                tc::fence_proxy_async();
                tc::mbar_arrive(&bar->k_full[st]);
                if (t == 0 && gt < 7) TRACE(50 + gt);
                if (gt >= NS && !tc::mbar_wait(&bar->v_empty[st], ((gt / NS) - 1) & 1, abort, &g_attn_watchdog, 32)) { ok = false; break; }
                uint8_t* vh = vst + st * STAGE;
#pragma unroll
                for (int c = 0; c < 8; c++) {
                    float x[4] = {vn[c].x, vn[c].y, vn[c].z, vn[c].w}, hi[4], lo[4];
#pragma unroll
                    for (int u = 0; u < 4; u++) { hi[u] = hi_part(x[u]); lo[u] = x[u] - hi[u]; }
                    const uint32_t o = v_off(jr, d0 + 4 * c);
                    *reinterpret_cast<float4*>(vh + o) = make_float4(hi[0], hi[1], hi[2], hi[3]);
                    *reinterpret_cast<float4*>(vh + KV_HALF + o) = make_float4(lo[0], lo[1], lo[2], lo[3]);
                }
                tc::fence_proxy_async();
                tc::mbar_arrive(&bar->v_full[st]);
                if (t == 0 && gt < 6) TRACE(57 + gt);
            }
        }
    }

    tc::tc_fence_before();
    __syncthreads();
    if (threadIdx.x == 0) TRACE(63);
    if (bar->abort && warp == 4 && lane == 0) {    // let issued MMAs retire before TMEM is released
        int never = 0;
        tc::mma_commit(&bar->drain);
        tc::mbar_wait(&bar->drain, 0, &never, nullptr, 0);
    }
    __syncthreads();
    if (warp == 4) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tm, TM_COLS);
    }
}

}  // namespace

extern "C" int lcu_attention_tc_supported(size_t D_) { return D_ == (size_t)D; }

extern "C" lancius_error lcu_attention_tc(const LcuAttnGroup* d_table, const float* q, const float* k, const float* v,
                                          float* o, size_t B, size_t S, size_t H, int causal, void* stream) {
    if (B == 0 || S == 0 || H == 0) return LANCIUS_ERROR_OK;
    static bool configured[64] = {};   // the attribute is per device
    int dev_ = 0;
    cudaGetDevice(&dev_);
    if (dev_ >= 0 && dev_ < 64 && !configured[dev_]) {
        if (cudaFuncSetAttribute(k_attn_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES) != cudaSuccess)
            return lcu_launch_status();
        configured[dev_] = true;
    }
    LcuAttnGroup base{q, k, v, o};
    float scale_log2 = (float)(1.4426950408889634 / 8.0);   // log2(e) / sqrt(64)
    // persistent grid: one CTA per SM (TMEM and shared memory allow no more), each walks
    // pairs of query tiles of equal total cost with stride gridDim.x
    static int sms = 0;
    if (!sms) {
        int dev = 0;
        cudaGetDevice(&dev);
        if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0) sms = LCU_SMS;
    }
    const size_t pairs = ((S + BQ - 1) / BQ + 1) / 2 * H * B;
    const unsigned grid = (unsigned)(pairs < (size_t)sms ? pairs : (size_t)sms);
    k_attn_tc<<<grid, THREADS, SMEM_BYTES, lcu_as_stream(stream)>>>(d_table, base, S * H * D, (int)B, (int)S, (int)H,
                                                                     causal, scale_log2);
    lcu_note_launch();
    return lcu_launch_status();
}

extern "C" int lcu_attention_trace(unsigned long long* host, int n) {
#if LCU_ATTN_TRACE
    return cudaMemcpyFromSymbol(host, g_trace, sizeof(unsigned long long) * 64 * (n < 512 ? n : 512)) == cudaSuccess;
#else
    (void)host; (void)n;
    return 0;
#endif
}

extern "C" int lcu_attention_watchdog_read_and_clear(void) {
    int v = 0, z = 0;
    cudaMemcpyFromSymbol(&v, g_attn_watchdog, sizeof(int));
    if (v) cudaMemcpyToSymbol(g_attn_watchdog, &z, sizeof(int));
    return v;
}

// Device address of this file's watchdog word on the current device (0 if unavailable).
extern "C" int* lcu_attention_watchdog_addr(void) {
    void* p = nullptr;
    return cudaGetSymbolAddress(&p, g_attn_watchdog) == cudaSuccess ? static_cast<int*>(p) : nullptr;
}
