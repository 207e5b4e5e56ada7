// Flash attention on the tcgen05 tensor cores, FP32-exact (3xTF32), head_dim 64.
// Restates kernel_attention (lancius_kernels.c:278-332): per query row an online
// softmax over all keys (causal: keys j > i masked), scale 1/sqrt(D); the score
// matrix never leaves the SM.
//
// One CTA (persistent, one per SM) walks pairs of (128-query tile, head, batch element)
// items. Roles:
//   warps 0-3  softmax: one query row per thread (= its TMEM lane). Copies the Q row from
//              the shared-memory stage into TMEM as TF32 hi/lo columns; per key tile reads S,
//              writes P = exp2(S - m) as hi/lo columns IN PLACE of S and keeps the row sum.
//              The running max m is only raised when a tile's max exceeds it by more
//              than 2^8 (then the O accumulator in TMEM is rescaled); any fixed offset
//              gives the same softmax, so this is exact, and P stays <= 256.
//   warp 4     TMEM allocation + S issue (one lane): S_j = Q K_j^T (A = Q from TMEM).
//   warp 9     PV issue (one lane): O += P_j V_j (A = P_j from TMEM). One thread's
//              tcgen05.mma instructions complete one after another (~120 clk each for
//              N <= 128, measured); two issuing threads overlap on the tensor pipe, so the
//              S stream of tile j+1 runs beside the PV stream of tile j.
//              tcgen05 costs about the same per instruction whatever its N, so the
//              hi/lo halves of B are concatenated along N: Q_hi*[K_hi|K_lo] (N = 128)
//              and Q_lo*K_hi (N = 64) accumulate Q_hi K_hi + Q_lo K_hi in the left and
//              Q_hi K_lo in the right half of S, and S = left + right; same for
//              P_hi*[V_hi|V_lo] and P_lo*V_hi into O.
//   warps 5-6  K loaders: cp.async of the raw FP32 K tile (= the hi operand: the MMA reads
//              only the TF32 bits) into its swizzled place, then K_lo = x - hi(x) beside it;
//              they also stage the next item's Q rows (cp.async) while the current item runs,
//              and ask L2 for the key rows a few tiles ahead.
//   warps 7-8  V loaders: the same for V.
// S/P live in two TMEM buffers used by alternate key tiles, so the softmax of tile j never
// waits for PV of tile j-1. TMEM columns: Q hi [0,64) lo [64,128); S/P buffers [128,256)
// and [256,384); O halves [384,512). Every mbarrier wait is bounded.
// The TF32 fast mode (EXACT = false) runs one pass: Q K^T and P V on the raw operands.
#include "tc_common.cuh"

namespace {

constexpr int D = 64, BQ = 128, BKV = 64, NSK = 3, NSV = 3;
constexpr int THREADS = 320;
constexpr int KV_HALF = BKV * D * 4;            // 16 KB: one hi or lo tile
constexpr int STAGE = 2 * KV_HALF;              // hi + lo
constexpr int Q_STAGE = BQ * D * 4;             // Q rows of the next item: two 32-d halves, 128-byte swizzled rows
constexpr int SMEM_BYTES = (NSK + NSV) * STAGE + Q_STAGE + 1024 + 1024;
constexpr uint32_t TM_QHI = 0, TM_QLO = 64, TM_SP = 128, TM_O = 384, TM_COLS = 512;
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
    uint64_t k_full[NSK], k_empty[NSK], v_full[NSV], v_empty[NSV];
    uint64_t s_full[2], p_ready[2], pv_done[2];   // per S/P buffer (tile parity)
    uint64_t q_full, q_empty, q_ready, o_free, drain, drain_pv;
    uint32_t tmem;
    int abort;
};
static_assert(sizeof(Bars) <= 1024, "barrier block");

// Bounded mbarrier wait that polls (test_wait, no suspend): a suspending try_wait was
// measured to wake up to ~1 us after the phase completed, which serialised the roles.
__device__ __forceinline__ bool bwait(uint64_t* bar, uint32_t parity, volatile int* abort, int* watchdog, int where) {
    for (uint32_t i = 0; i < 64u * tc::kSpinLimit; i++) {
        uint32_t done;
        asm volatile("{\n\t.reg .pred p;\n\tmbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
                     "selp.b32 %0, 1, 0, p;\n\t}" : "=r"(done) : "r"(tc::smem_u32(bar)), "r"(parity) : "memory");
        if (done) return true;
        if ((i & 63) == 63 && *abort) return false;
    }
    *abort = 1;
    if (watchdog) atomicCAS(watchdog, 0, where);
    return false;
}
__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1, int c2,
                                            int c3) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6}], [%2];"
        ::"r"(tc::smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(tc::smem_u32(bar)), "r"(c0), "r"(c1),
          "r"(c2), "r"(c3)
        : "memory");
}

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

struct Item { LcuAttnGroup p; int b, h, q0, T; };
constexpr int NMAPS = 5;                // Q, K, V, K_lo, V_lo
struct AttnMaps { CUtensorMap m[NMAPS]; };   // over [B][S][H][D] (per-op launches)

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
    it.h = r % H;
    it.b = b;
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

__device__ __forceinline__ bool slot_valid(int x, int per, int nqt) {
    return !((x & 1) && 2 * ((x >> 1) / per) == nqt - 1);
}
// next valid slot after x in this CTA's walk (n_slots if none)
__device__ __forceinline__ int next_valid(int x, int n_slots, int per, int nqt) {
    for (x = next_slot(x); x < n_slots && !slot_valid(x, per, nqt); x = next_slot(x)) {}
    return x;
}

// EXACT: 3xTF32 (FP32-exact). Otherwise the TF32 fast mode: one pass, Q K^T and P V on the
// raw FP32 operands (the MMA reads their TF32 bits), no lo copies anywhere.
template <bool EXACT>
__global__ void __launch_bounds__(THREADS, 1)
k_attn_tc(const LcuAttnGroup* __restrict__ table, LcuAttnGroup base, size_t bstride, int B, int S, int H, int causal,
          float scale_log2, const CUtensorMap* __restrict__ gmaps, const __grid_constant__ AttnMaps pm) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* tiles = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* kst = tiles;                          // NSK stages of K hi|lo
    uint8_t* vst = tiles + NSK * STAGE;            // NSV stages of V hi|lo
    uint8_t* qst = vst + NSV * STAGE;              // raw Q rows of the next item, pitch Q_PITCH
    Bars* bar = reinterpret_cast<Bars*>(qst + Q_STAGE);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nqt = (S + BQ - 1) / BQ;
    const int per = B * H;
    const int n_slots = 2 * ((nqt + 1) / 2) * per;
    const size_t rs = (size_t)H * D;                // row stride of [S, H, D]
    volatile int* abort = &bar->abort;

    if (threadIdx.x == 0) {
        for (int s = 0; s < NSK; s++) {
            tc::mbar_init(&bar->k_full[s], 1); tc::mbar_init(&bar->k_empty[s], 1);
        }
        for (int s = 0; s < NSV; s++) {
            tc::mbar_init(&bar->v_full[s], 1); tc::mbar_init(&bar->v_empty[s], 1);
        }
        for (int b = 0; b < 2; b++) {
            tc::mbar_init(&bar->s_full[b], 1); tc::mbar_init(&bar->p_ready[b], 128); tc::mbar_init(&bar->pv_done[b], 1);
        }
        tc::mbar_init(&bar->q_full, 1);
        tc::mbar_init(&bar->q_empty, 128);
        tc::mbar_init(&bar->q_ready, 128);
        tc::mbar_init(&bar->o_free, 128);
        tc::mbar_init(&bar->drain, 1);
        tc::mbar_init(&bar->drain_pv, 1);
        bar->abort = 0;
        tc::fence_barrier_init();
    }
    if (warp == 4) tc::tmem_alloc(&bar->tmem, TM_COLS);
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tm = bar->tmem;
    if (threadIdx.x == 0) TRACE(0);
    const int x0 = slot_valid(2 * (int)blockIdx.x, per, nqt) ? 2 * (int)blockIdx.x
                                                              : next_valid(2 * (int)blockIdx.x, n_slots, per, nqt);

    // Every role walks the same item sequence; `gt` numbers this CTA's key tiles across
    // items and drives all ring stages and barrier phases (S/P buffer b = gt & 1, used for
    // the (gt >> 1)-th time).
    if (warp < 4) {
        // ======================= softmax warps =======================
        const int row = 32 * warp + lane;              // TMEM lane == query row in tile
        const uint32_t lb = tm + ((uint32_t)(32 * warp) << 16);
        int gt = 0, ii = 0;
        bool ok = true;
        // staged raw Q row -> TMEM hi/lo columns (the Q columns are free: every S of the
        // previous item has completed)
        auto take_q = [&](int phase) -> bool {
            if (!bwait(&bar->q_full, phase & 1, abort, &g_attn_watchdog, 10)) return false;
            const uint8_t* src = qst + row * 128;   // TMA 128-byte swizzle: chunk c of a row at c ^ (row & 7)
#pragma unroll 1
            for (int half = 0; half < 2; half++) {
                float hi[32], lo[32];
#pragma unroll
                for (int c = 0; c < 8; c++) {
                    const float4 v = *reinterpret_cast<const float4*>(src + half * (BQ * 128) + ((c ^ (row & 7)) << 4));
                    const float x[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                    for (int t = 0; t < 4; t++) { hi[4 * c + t] = hi_part(x[t]); lo[4 * c + t] = x[t] - hi[4 * c + t]; }
                }
                tc::tmem_st32(lb + TM_QHI + half * 32, hi);
                if (EXACT) tc::tmem_st32(lb + TM_QLO + half * 32, lo);
            }
            tc::mbar_arrive(&bar->q_empty);             // the stage may take the next item's rows
            tc::tmem_st_wait();
            tc::tc_fence_before();
            tc::mbar_arrive(&bar->q_ready);
            return true;
        };
        for (int x = x0; x < n_slots && ok; ii++) {
            const Item it = get_item(x, table, base, bstride, B, H, nqt, S, causal);
            const int xn = next_valid(x, n_slots, per, nqt);
            const int qi = it.q0 + row;
            if (ii == 0 && !(ok = take_q(0))) break;
            if (threadIdx.x == 0) TRACE(1);
            float m = -INFINITY, l = 0.f;
            for (int j = 0; j < it.T; j++, gt++) {
                const int b = gt & 1, use = gt >> 1;
                const uint32_t sp = lb + TM_SP + 128 * b;
                if (!bwait(&bar->s_full[b], use & 1, abort, &g_attn_watchdog, 11)) { ok = false; break; }
                if (threadIdx.x == 0 && gt < 8) TRACE(2 + 4 * gt);
                tc::tc_fence_after();
                float s[64];
#pragma unroll
                for (int half = 0; half < 2; half++) {
                    float a[32], c2[32];
                    tc::tmem_ld32(sp + half * 32, a);                      // Q_hi K_hi + Q_lo K_hi
                    if (EXACT) tc::tmem_ld32(sp + 64 + half * 32, c2);     // Q_hi K_lo
#pragma unroll
                    for (int c = 0; c < 32; c++) s[half * 32 + c] = (EXACT ? a[c] + c2[c] : a[c]) * scale_log2;
                }
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
                        const int pg = gt - 1;
                        if (!bwait(&bar->pv_done[pg & 1], (pg >> 1) & 1, abort, &g_attn_watchdog, 12)) { ok = false; break; }
                        tc::tc_fence_after();
#pragma unroll 1
                        for (int q4 = 0; q4 < (EXACT ? 4 : 2); q4++) {
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
                // P replaces S in the same buffer: hi in the left, lo in the right half
#pragma unroll
                for (int half = 0; half < 2; half++) {
                    float hi[32], lo[32];
#pragma unroll
                    for (int c = 0; c < 32; c++) { hi[c] = hi_part(s[half * 32 + c]); lo[c] = s[half * 32 + c] - hi[c]; }
                    tc::tmem_st32(sp + half * 32, hi);
                    if (EXACT) tc::tmem_st32(sp + 64 + half * 32, lo);
                }
                if (threadIdx.x == 0 && gt < 8) TRACE(4 + 4 * gt);
                tc::tmem_st_wait();
                tc::tc_fence_before();
                tc::mbar_arrive(&bar->p_ready[b]);
                if (threadIdx.x == 0 && gt < 8) TRACE(5 + 4 * gt);
            }
            if (!ok) break;
            // the next item's Q goes in now, so its first S overlaps this item's last PV and
            // the O epilogue below
            if (xn < n_slots && !(ok = take_q(ii + 1))) break;
            if (it.T > 0) {
                const int pg = gt - 1;
                if (!bwait(&bar->pv_done[pg & 1], (pg >> 1) & 1, abort, &g_attn_watchdog, 13)) { ok = false; break; }
                tc::tc_fence_after();
                const float inv = 1.f / l;
#pragma unroll 1
                for (int half = 0; half < 2; half++) {
                    float o[32], o2[32];
                    tc::tmem_ld32(lb + TM_O + half * 32, o);                      // P_hi V_hi + P_lo V_hi
                    if (EXACT) tc::tmem_ld32(lb + TM_O + 64 + half * 32, o2);     // P_hi V_lo
                    else {
#pragma unroll
                        for (int c = 0; c < 32; c++) o2[c] = 0.f;
                    }
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
            tc::mbar_arrive(&bar->o_free);                   // O columns reusable
            x = xn;
        }
    } else if (warp == 4) {
        // ======================= S issuer =======================
        if (lane == 0) {
            constexpr uint32_t id_s = tc::idesc_tf32(BQ, 2 * BKV, false, false);
            // the lo x lo product is below FP32 resolution: the lo operand multiplies only
            // the hi half of B (N = 64)
            constexpr uint32_t id_s_lo = tc::idesc_tf32(BQ, BKV, false, false);
            bool ok = true;
            int gt = 0, ii = 0;
            for (int x = x0; x < n_slots && ok; x = next_valid(x, n_slots, per, nqt), ii++) {
                const Item it = get_item(x, table, base, bstride, B, H, nqt, S, causal);
                if (!bwait(&bar->q_ready, ii & 1, abort, &g_attn_watchdog, 21)) { ok = false; break; }
                for (int j = 0; j < it.T; j++, gt++) {
                    const int st = gt % NSK, b = gt & 1, use = gt >> 1;
                    // buffer b is free once the PV of its previous tile (gt - 2) has read P
                    if (!bwait(&bar->k_full[st], (gt / NSK) & 1, abort, &g_attn_watchdog, 22) ||
                        (use >= 1 && !bwait(&bar->pv_done[b], (use - 1) & 1, abort, &g_attn_watchdog, 23))) { ok = false; break; }
                    tc::tc_fence_after();
                    if (gt < 4) TRACE(34 + 2 * gt);
                    const uint32_t kb0 = tc::smem_u32(kst + st * STAGE);
                    const uint32_t sd = tm + TM_SP + 128 * b;
#pragma unroll
                    for (int kb = 0; kb < D / 8; kb++) {
                        const uint32_t off = (uint32_t)((kb >> 2) * (2 * BKV * 128) + (kb & 3) * 32);
                        const uint64_t bk = tc::smem_desc(kb0 + off, 16, 1024, tc::SWZ_128B);   // [K_hi | K_lo]
                        if (EXACT) {
                            tc::mma_tf32_ts(sd, tm + TM_QHI + kb * 8, bk, id_s, kb ? 1u : 0u);
                            tc::mma_tf32_ts(sd, tm + TM_QLO + kb * 8, bk, id_s_lo, 1u);
                        } else {
                            tc::mma_tf32_ts(sd, tm + TM_QHI + kb * 8, bk, id_s_lo, kb ? 1u : 0u);   // Q K_hi
                        }
                    }
                    tc::mma_commit(&bar->s_full[b]);
                    tc::mma_commit(&bar->k_empty[st]);
                    if (gt < 4) TRACE(35 + 2 * gt);
                }
            }
        }
    } else if (warp == 9) {
        // ======================= PV issuer =======================
        if (lane == 0) {
            constexpr uint32_t id_o = tc::idesc_tf32(BQ, 2 * D, false, true);
            constexpr uint32_t id_o_lo = tc::idesc_tf32(BQ, D, false, true);
            bool ok = true;
            int gt = 0, ii = 0;
            for (int x = x0; x < n_slots && ok; x = next_valid(x, n_slots, per, nqt), ii++) {
                const Item it = get_item(x, table, base, bstride, B, H, nqt, S, causal);
                for (int j = 0; j < it.T; j++, gt++) {
                    const int st = gt % NSV, b = gt & 1, use = gt >> 1;
                    if (!bwait(&bar->p_ready[b], use & 1, abort, &g_attn_watchdog, 24) ||
                        !bwait(&bar->v_full[st], (gt / NSV) & 1, abort, &g_attn_watchdog, 25)) { ok = false; break; }
                    // the first PV of an item overwrites O: the previous item's O must have been read
                    if (j == 0 && ii >= 1 && !bwait(&bar->o_free, (ii - 1) & 1, abort, &g_attn_watchdog, 26)) { ok = false; break; }
                    tc::tc_fence_after();
                    if (gt < 4) TRACE(42 + 2 * gt);
                    const uint32_t vb0 = tc::smem_u32(vst + st * STAGE);
                    const uint32_t pa = tm + TM_SP + 128 * b;
#pragma unroll
                    for (int kb = 0; kb < BKV / 8; kb++) {
                        const uint64_t bv = tc::smem_desc(vb0 + kb * 1024, BKV * 128, 512, tc::SWZ_128B_BASE32B);   // [V_hi | V_lo]
                        const uint32_t acc0 = (j | kb) ? 1u : 0u;
                        if (EXACT) {
                            tc::mma_tf32_ts(tm + TM_O, pa + kb * 8, bv, id_o, acc0);
                            tc::mma_tf32_ts(tm + TM_O, pa + 64 + kb * 8, bv, id_o_lo, 1u);
                        } else {
                            tc::mma_tf32_ts(tm + TM_O, pa + kb * 8, bv, id_o_lo, acc0);     // P V_hi
                        }
                    }
                    tc::mma_commit(&bar->pv_done[b]);
                    tc::mma_commit(&bar->v_empty[st]);
                    if (gt < 4) TRACE(43 + 2 * gt);
                }
            }
        }
    } else {
        // ======================= producers: warp 5 K (+ Q stage), warp 7 V =======================
        // One thread per operand puts each key tile in place with TMA: the raw FP32 values
        // (= the hi operand: the MMA reads only their TF32 bits) and, FP32-exact, their lo
        // parts from the copies the split pass made (lcu_attention_tc runs it first), each as
        // two boxes of 32 d x 64 keys, swizzled as the MMA reads them. Nothing is computed
        // here: splitting in shared memory next to the MMAs' operand reads was measured to
        // cost more than the split pass's extra HBM traffic.
        const bool is_k = warp == 5;
        if ((warp == 5 || warp == 7) && lane == 0) {
            const int NSt = is_k ? NSK : NSV;
            uint8_t* base_st = is_k ? kst : vst;
            uint64_t* full = is_k ? bar->k_full : bar->v_full;
            uint64_t* empty = is_k ? bar->k_empty : bar->v_empty;
            int gt = 0, ii = 0;
            bool ok = true;
            for (int x = x0; x < n_slots && ok; x = next_valid(x, n_slots, per, nqt), ii++) {
                const Item it = get_item(x, table, base, bstride, B, H, nqt, S, causal);
                const CUtensorMap* maps = gmaps ? gmaps + NMAPS * it.b : pm.m;
                const int cb = gmaps ? 0 : it.b;         // the batch coordinate of the map
                const CUtensorMap* mhi = maps + (is_k ? 1 : 2);
                const CUtensorMap* mlo = maps + (is_k ? 3 : 4);
                if (gmaps) {
                    tc::tmap_acquire(mhi);
                    if (EXACT) tc::tmap_acquire(mlo);
                    if (is_k) tc::tmap_acquire(maps);
                }
                if (is_k) {   // this item's Q rows, once the previous ones were taken
                    if (ii >= 1 && !bwait(&bar->q_empty, (ii - 1) & 1, abort, &g_attn_watchdog, 30)) { ok = false; break; }
                    tc::mbar_expect_tx(&bar->q_full, Q_STAGE);
                    tma_load_4d(qst, maps + 0, &bar->q_full, 0, it.h, it.q0, cb);
                    tma_load_4d(qst + BQ * 128, maps + 0, &bar->q_full, 32, it.h, it.q0, cb);
                }
                for (int j = 0; j < it.T; j++, gt++) {
                    const int st = gt % NSt;
                    if (gt >= NSt && !bwait(&empty[st], ((gt / NSt) - 1) & 1, abort, &g_attn_watchdog, 31)) { ok = false; break; }
                    uint8_t* dst = base_st + st * STAGE;
                    tc::mbar_expect_tx(&full[st], EXACT ? 2 * KV_HALF : KV_HALF);
                    for (int a = 0; a < 2; a++) {   // d 0-31 and 32-63
                        // K: per 32-d atom 64 hi rows then 64 lo rows; V: hi chunks, then lo chunks
                        uint8_t* h = dst + a * (is_k ? 2 * BKV * 128 : BKV * 128);
                        tma_load_4d(h, mhi, &full[st], 32 * a, it.h, j * BKV, cb);
                        if (EXACT) tma_load_4d(h + (is_k ? BKV * 128 : KV_HALF), mlo, &full[st], 32 * a, it.h, j * BKV, cb);
                    }
                    if (gt < 7) TRACE(is_k ? 50 + gt : 57 + (gt < 6 ? gt : 5));
                }
            }
        }
    }

    tc::tc_fence_before();
    __syncthreads();
    if (threadIdx.x == 0) TRACE(63);
    if (bar->abort && (warp == 4 || warp == 9) && lane == 0) {   // let issued MMAs retire before TMEM is released
        int never = 0;
        uint64_t* d = warp == 4 ? &bar->drain : &bar->drain_pv;
        tc::mma_commit(d);
        tc::mbar_wait(d, 0, &never, nullptr, 0);
    }
    __syncthreads();
    if (warp == 4) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tm, TM_COLS);
    }
}

}  // namespace

namespace {
// lo = x - hi(x) (exact in FP32) of every K and V element, into lo[B][2][S][H][D]: the
// split pass of the FP32-exact attention (one read and one write of K and V in HBM).
__global__ void k_attn_split_lo(const LcuAttnGroup* __restrict__ table, LcuAttnGroup base, size_t bstride, int B,
                                size_t n, float* __restrict__ lo) {
    const size_t n4 = n / 4, total = (size_t)B * 2 * n4;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const size_t b = i / (2 * n4), r = i - b * 2 * n4, which = r / n4, e = r - which * n4;
        const float* src = table ? (which ? table[b].v : table[b].k) : (which ? base.v : base.k) + b * bstride;
        const float4 x = __ldg(reinterpret_cast<const float4*>(src) + e);
        reinterpret_cast<float4*>(lo + (b * 2 + which) * n)[e] =
            make_float4(x.x - hi_part(x.x), x.y - hi_part(x.y), x.z - hi_part(x.z), x.w - hi_part(x.w));
    }
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        return (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
                q == cudaDriverEntryPointSuccess) ? reinterpret_cast<EncodeTiledFn>(p) : nullptr;
    }();
    return fn;
}
// map over [B][S][H][D] FP32 (dims innermost first: d, h, s, b), box 32 d x rows keys/queries
bool make_qkv_map(CUtensorMap* m, const float* base, size_t B, size_t S, size_t H, size_t bstride, uint32_t rows,
                  CUtensorMapSwizzle swz) {
    EncodeTiledFn fn = encode_fn();
    if (!fn || (reinterpret_cast<uintptr_t>(base) & 15)) return false;
    cuuint64_t dims[4] = {(cuuint64_t)D, H, S, B};
    cuuint64_t strides[3] = {(cuuint64_t)D * 4, (cuuint64_t)H * D * 4, (cuuint64_t)(bstride ? bstride : S * H * D) * 4};
    cuuint32_t box[4] = {32, 1, rows, 1};
    cuuint32_t es[4] = {1, 1, 1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, const_cast<float*>(base), dims, strides, box, es,
              CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

// Q, K, V tensor maps of one attention operand set over [B][S][H][D] (B = 1 for one node of
// a grouped launch): Q in 128-row boxes, K in 64-row boxes (128-byte swizzle, K-major), V in
// 64-row boxes (128-byte swizzle of 32-byte atoms, N-major for the PV product).
// lo: the [B][2][S][H][D] lo copies (K then V per operand set) the split pass writes.
extern "C" bool lcu_attention_tc_make_maps(CUtensorMap* maps, const float* q, const float* k, const float* v,
                                           const float* lo, size_t B, size_t S, size_t H) {
    const size_t n = S * H * D;
    return make_qkv_map(maps + 0, q, B, S, H, 0, BQ, CU_TENSOR_MAP_SWIZZLE_128B) &&
           make_qkv_map(maps + 1, k, B, S, H, 0, BKV, CU_TENSOR_MAP_SWIZZLE_128B) &&
           make_qkv_map(maps + 2, v, B, S, H, 0, BKV, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B) &&
           make_qkv_map(maps + 3, lo, B, S, H, 2 * n, BKV, CU_TENSOR_MAP_SWIZZLE_128B) &&
           make_qkv_map(maps + 4, lo + n, B, S, H, 2 * n, BKV, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B);
}

extern "C" size_t lcu_attention_tc_lo_floats(size_t B, size_t S, size_t H) { return 2 * B * S * H * D; }

extern "C" int lcu_attention_tc_supported(size_t D_) { return D_ == (size_t)D; }

extern "C" lancius_error lcu_attention_tc(const LcuAttnGroup* d_table, const float* q, const float* k, const float* v,
                                          float* o, size_t B, size_t S, size_t H, int causal, int mode,
                                          const CUtensorMap* d_maps, float* lo, void* stream) {
    if (B == 0 || S == 0 || H == 0) return LANCIUS_ERROR_OK;
    AttnMaps pm{};
    if (!d_table) {
        if (!lo && !(lo = static_cast<float*>(lcu_scratch_acquire(lcu_attention_tc_lo_floats(B, S, H) * 4)))) {
            lancius_set_error(LANCIUS_ERROR_OOM);
            return LANCIUS_ERROR_OOM;
        }
        if (!lcu_attention_tc_make_maps(pm.m, q, k, v, lo, B, S, H)) {
            lancius_set_error(LANCIUS_ERROR_INTERNAL);
            return LANCIUS_ERROR_INTERNAL;
        }
    }
    if (d_table && (!d_maps || !lo)) { lancius_set_error(LANCIUS_ERROR_INTERNAL); return LANCIUS_ERROR_INTERNAL; }
    if (mode != LCU_MODE_TF32) {
        const size_t total4 = 2 * B * S * H * D / 4;
        k_attn_split_lo<<<lcu_blocks(total4, 256), 256, 0, lcu_as_stream(stream)>>>(d_table, LcuAttnGroup{q, k, v, o},
                                                                                  S * H * D, (int)B, S * H * D, lo);
        lcu_note_launch();
    }
    static bool configured[64] = {};   // the attribute is per device
    int dev_ = 0;
    cudaGetDevice(&dev_);
    if (dev_ >= 0 && dev_ < 64 && !configured[dev_]) {
        if (cudaFuncSetAttribute(k_attn_tc<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES) != cudaSuccess ||
            cudaFuncSetAttribute(k_attn_tc<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES) != cudaSuccess)
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
    if (mode == LCU_MODE_TF32)
        k_attn_tc<false><<<grid, THREADS, SMEM_BYTES, lcu_as_stream(stream)>>>(d_table, base, S * H * D, (int)B, (int)S,
                                                                              (int)H, causal, scale_log2, d_table ? d_maps : nullptr, pm);
    else
        k_attn_tc<true><<<grid, THREADS, SMEM_BYTES, lcu_as_stream(stream)>>>(d_table, base, S * H * D, (int)B, (int)S,
                                                                             (int)H, causal, scale_log2, d_table ? d_maps : nullptr, pm);
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
