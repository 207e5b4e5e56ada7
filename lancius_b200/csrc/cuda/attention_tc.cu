// Flash attention on the tcgen05 tensor cores, FP32-exact (3xTF32), head_dim 64.
// Restates kernel_attention (lancius_kernels.c:278-332): per query row an online
// softmax over all keys (causal: keys j > i masked), scale 1/sqrt(D); the score
// matrix never leaves the SM.
//
// One CTA (persistent, one per SM) walks pairs of (128-query tile, head, batch element)
// items. Roles:
//   warps 0-7  softmax: a query row per pair of threads (warps w and w + 4 share the TMEM
//              lanes of row quadrant w % 4; warp w < 4 takes keys 0-31 of each 64-key
//              tile, warp w + 4 keys 32-63). At an item's start they copy its Q rows from
//              the shared-memory stage into TMEM as TF32 hi/lo columns. Per key tile they
//              read S, agree on the row max through shared memory, and write
//              P = exp2(S - m) as hi/lo columns IN PLACE of S; each keeps the row sum of its
//              half. The running max m is only raised when a tile's max exceeds it by more
//              than 2^8 (then the O accumulator in TMEM is rescaled); any fixed offset gives
//              the same softmax, so this is exact, and P stays <= 256. At an item's end
//              they write the normalised O rows into the Q stage for a TMA store.
//   warp 8     TMEM allocation + S issue (one lane): S_j = Q K_j^T (A = Q from TMEM); it
//              also loads each item's Q rows into the stage (TMA).
//   warp 9     PV issue (one lane): O += P_j V_j (A = P_j from TMEM), then the item's O
//              store (TMA, from the stage). One thread's tcgen05.mma instructions complete
//              one after another (~120 clk each for N <= 128, measured); two issuing
//              threads overlap on the tensor pipe, so the S stream of tile j+1 runs beside
//              the PV stream of tile j.
//              tcgen05 costs about the same per instruction whatever its N, so the
//              hi/lo halves of B are concatenated along N: Q_hi*[K_hi|K_lo] (N = 128)
//              and Q_lo*K_hi (N = 64) accumulate Q_hi K_hi + Q_lo K_hi in the left and
//              Q_hi K_lo in the right half of S, and S = left + right; same for
//              P_hi*[V_hi|V_lo] and P_lo*V_hi into O.
//   warp 10    K producer, warp 11 V producer (one lane each): TMA of the raw key tile
//              (= the hi operand: the MMA reads only the TF32 bits).
//   warps 12-15 splitters (12-13 K, 14-15 V): lo = x - hi(x) of each landed tile into the
//              stage's lo half, then the stage is released to the issuers. (LCU_ATTN_SPLIT_PASS=1
//              instead runs a split pass over all of K and V first, whose lo copies the
//              producers load by TMA; the kernel is then that pass's programmatic
//              dependent. Measured 36.9 against 34.4 us per graph for the in-CTA split.)
// S/P live in two TMEM buffers used by alternate key tiles, so the softmax of tile j never
// waits for PV of tile j-1. TMEM columns: Q hi [0,64) lo [64,128); S/P buffers [128,256)
// and [256,384); O halves [384,512). Every mbarrier wait is bounded.
// The TF32 fast mode (EXACT = false) runs one pass: Q K^T and P V on the raw operands.
#include "tc_common.cuh"

namespace {

constexpr int D = 64, BQ = 128, BKV = 64, NSK = 3, NSV = 3, NBUF = 2;
constexpr int W_S = 8, W_PV = 9, W_K = 10, W_V = 11, W_KS = 12, W_VS = 14;   // splitters: 2 warps each
constexpr int NSPLIT = 2;                       // splitter warps per operand
constexpr int THREADS = 512;
constexpr int NSOFT = 256;                      // softmax threads (warps 0-7)
constexpr int KV_HALF = BKV * D * 4;            // 16 KB: one hi or lo tile
constexpr int STAGE = 2 * KV_HALF;              // hi + lo
constexpr int Q_STAGE = BQ * D * 4;             // Q rows of the next item: two 32-d halves, 128-byte swizzled rows
constexpr int TILE_BYTES = (NSK + NSV) * STAGE + Q_STAGE;
constexpr int RED_BYTES = 2 * 2 * BQ * 4;       // row-max / row-sum exchange: [parity][half][row]
constexpr int SMEM_BYTES = TILE_BYTES + RED_BYTES + 512;
static_assert(SMEM_BYTES <= 227 * 1024, "shared memory");
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
    uint64_t k_split[NSK], v_split[NSV];   // in-kernel split: the stage's lo half is written
    uint64_t s_full[NBUF], p_ready[NBUF], pv_done[NBUF];   // per S/P buffer
    uint64_t xch[4][2];      // per row quadrant and exchange parity: both halves posted
    uint64_t q_full, q_ready, o_free, drain, drain_pv;
    uint64_t o_staged;       // the softmax threads wrote the item's O rows into the Q stage
    uint64_t stage_free;     // the O store has read the stage
    uint32_t tmem;
    int abort;
};
static_assert(sizeof(Bars) <= 512, "barrier block");

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

// Shared-memory tiles, all 128-byte swizzled as the TMA writes them:
//   K stage: per 32-d atom 128 rows of 128 B: rows 0-63 = K_hi keys, rows 64-127 = K_lo
//            keys (K-major), so one descriptor spans [K_hi | K_lo] as N = 128.
//   V stage: 32-d chunks of 64 key rows (N-major, 32-byte atoms); V_hi fills chunks 0-1
//            and V_lo chunks 2-3, so one descriptor spans [V_hi | V_lo] as N = 128.
//   Q, Q_lo: per 32-d atom 128 query rows of 128 B (K-major A operand).
// TF32 split: hi keeps the top 10 mantissa bits (exactly what the tensor core reads),
// lo = x - hi is exact in FP32 and carries the next bits.
__device__ __forceinline__ float hi_part(float x) { return __uint_as_float(__float_as_uint(x) & 0xFFFFE000u); }
__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

struct Item { int b, h, q0, T; };   // operand set (batch element), head, first query row, key tiles
constexpr int NMAPS = LCU_ATTN_TC_MAPS;  // Q, K, V, K_lo, V_lo, O
struct AttnMaps { CUtensorMap m[NMAPS]; };   // over [B][S][H][D] (per-op launches)

// Work slots of the persistent grid. Causal cost grows with the query tile index, so
// tile qt is paired with tile nqt-1-qt: slot 2p is the light member of pair p (empty for
// the middle tile of an odd nqt), slot 2p+1 the heavy one, and every pair costs the same
// number of key tiles. A CTA takes both slots of a pair, then strides by the grid over
// pairs; pairs are ordered so the light (unpaired) ones come last. The light item runs
// first: its short chain of key tiles (and its O epilogue) overlaps the start of the
// heavy one, whose long run of tiles then keeps the tensor pipe busy to the end.
__device__ __forceinline__ int next_slot(int x) { return (x & 1) ? x - 1 + 2 * (int)gridDim.x : x + 1; }

// Everything an item needs comes from the slot index and the tensor maps: no global load
// (the operand table, cold after an L2 flush, cost ~0.7 us at each role's start).
__device__ __forceinline__ Item get_item(int x, const LcuAttnGroup* table, const LcuAttnGroup& base, size_t bstride,
                                         int B, int H, int nqt, int S, int causal) {
    (void)table; (void)base; (void)bstride;
    Item it;
    const int per = B * H;
    const int pair = x >> 1, qp = pair / per, r = pair % per, b = r / H;
    const int qt = (x & 1) ? nqt - 1 - qp : qp;
    it.h = r % H;
    it.b = b;
    it.q0 = qt * BQ;
    const int kv_end = causal ? min(S, it.q0 + BQ) : S;
    it.T = (kv_end + BKV - 1) / BKV;
    return it;
}

__device__ __forceinline__ bool slot_valid(int x, int per, int nqt) {
    return !(!(x & 1) && 2 * ((x >> 1) / per) == nqt - 1);
}
// next valid slot after x in this CTA's walk (n_slots if none)
__device__ __forceinline__ int next_valid(int x, int n_slots, int per, int nqt) {
    for (x = next_slot(x); x < n_slots && !slot_valid(x, per, nqt); x = next_slot(x)) {}
    return x;
}

// EXACT: 3xTF32 (FP32-exact). Otherwise the TF32 fast mode: one pass, Q K^T and P V on the
// raw FP32 operands (the MMA reads their TF32 bits), no lo copies anywhere.
// INSPLIT (FP32-exact only): the lo halves of the K and V stages are computed in the CTA
// (warps 12 and 13) from the raw tile the TMA brought, instead of loaded from the split
// pass's copies.
template <bool EXACT, bool INSPLIT>
__global__ void __launch_bounds__(THREADS, 1)
k_attn_tc(const LcuAttnGroup* __restrict__ table, LcuAttnGroup base, size_t bstride, int B, int S, int H, int causal,
          float scale_log2, const CUtensorMap* __restrict__ gmaps, const __grid_constant__ AttnMaps pm) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // the swizzled tiles need a 1024-byte aligned base; refuse (with a watchdog code) rather
    // than mis-address if the launch ever provides less
    if (tc::smem_u32(smem_raw) & 1023) {
        if (threadIdx.x == 0) atomicCAS(&g_attn_watchdog, 0, 99);
        return;
    }
    uint8_t* kst = smem_raw;                       // NSK stages of K hi|lo
    uint8_t* vst = kst + NSK * STAGE;              // NSV stages of V hi|lo
    uint8_t* qst = vst + NSV * STAGE;              // raw Q rows of the next item
    float* red = reinterpret_cast<float*>(qst + Q_STAGE);
    Bars* bar = reinterpret_cast<Bars*>(qst + Q_STAGE + RED_BYTES);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nqt = (S + BQ - 1) / BQ;
    const int per = B * H;
    const int n_slots = 2 * ((nqt + 1) / 2) * per;
    volatile int* abort = &bar->abort;

    if (threadIdx.x == 0) {
        TRACE(62);
        {   // the descriptors of this CTA's first pair of items, fetched while the CTA sets up
            const int xs[2] = {2 * (int)blockIdx.x, 2 * (int)blockIdx.x + 1};
            for (int i = 0; i < 2; i++) {
                const int bb = ((xs[i] >> 1) % per) / H;
                const CUtensorMap* mp = gmaps ? gmaps + NMAPS * bb : pm.m;
                if (xs[i] < n_slots) {
                    tc::prefetch_tmap(mp + 0); tc::prefetch_tmap(mp + 1); tc::prefetch_tmap(mp + 2); tc::prefetch_tmap(mp + 5);
                }
            }
        }
        for (int s = 0; s < NSK; s++) {
            tc::mbar_init(&bar->k_full[s], 1); tc::mbar_init(&bar->k_empty[s], 1); tc::mbar_init(&bar->k_split[s], NSPLIT);
        }
        for (int s = 0; s < NSV; s++) {
            tc::mbar_init(&bar->v_full[s], 1); tc::mbar_init(&bar->v_empty[s], 1); tc::mbar_init(&bar->v_split[s], NSPLIT);
        }
        for (int b = 0; b < NBUF; b++) {
            tc::mbar_init(&bar->s_full[b], 1); tc::mbar_init(&bar->p_ready[b], NSOFT); tc::mbar_init(&bar->pv_done[b], 1);
        }
        for (int q = 0; q < 4; q++) { tc::mbar_init(&bar->xch[q][0], 64); tc::mbar_init(&bar->xch[q][1], 64); }
        tc::mbar_init(&bar->q_full, 1);
        tc::mbar_init(&bar->q_ready, NSOFT);
        tc::mbar_init(&bar->o_free, NSOFT);
        tc::mbar_init(&bar->o_staged, NSOFT);
        tc::mbar_init(&bar->stage_free, 1);
        tc::mbar_init(&bar->drain, 1);
        tc::mbar_init(&bar->drain_pv, 1);
        bar->abort = 0;
        tc::fence_barrier_init();
    }
    if (warp == W_S) tc::tmem_alloc(&bar->tmem, TM_COLS);
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tm = bar->tmem;
    if (threadIdx.x == 0) TRACE(0);
    const int x0 = slot_valid(2 * (int)blockIdx.x, per, nqt) ? 2 * (int)blockIdx.x
                                                              : next_valid(2 * (int)blockIdx.x, n_slots, per, nqt);

    // Every role walks the same item sequence; `gt` numbers this CTA's key tiles across
    // items and drives all ring stages and barrier phases (S/P buffer b = gt % NBUF, used
    // for the (gt / NBUF)-th time).
    if (warp < 8) {
        // ======================= softmax warps =======================
        const int quad = warp & 3, hf = warp >> 2;
        const int row = 32 * quad + lane;              // TMEM lane == query row in tile
        const uint32_t lb = tm + ((uint32_t)(32 * quad) << 16);
        int gt = 0, ii = 0, xc = 0;
        bool ok = true;
        // The two threads of a row post a value each and read the other's. Exchange n uses
        // slot n & 1: a thread can only rewrite that slot at exchange n + 2, after the
        // partner arrived at n + 1, i.e. after it read exchange n.
        auto exchange = [&](float v, float& other) -> bool {
            const int p = xc & 1;
            red[(p * 2 + hf) * BQ + row] = v;
            tc::mbar_arrive(&bar->xch[quad][p]);
            if (!bwait(&bar->xch[quad][p], (xc >> 1) & 1, abort, &g_attn_watchdog, 14)) return false;
            other = red[(p * 2 + (hf ^ 1)) * BQ + row];
            xc++;
            return true;
        };
        // The staged raw Q rows of an item -> TMEM hi/lo columns, 32 d of its row per thread
        // (the Q columns are free: every S of the previous item has completed). Reading the
        // stage lets the S issuer load the next item's rows into it.
        auto take_q = [&](int phase) -> bool {
            if (!bwait(&bar->q_full, phase & 1, abort, &g_attn_watchdog, 10)) return false;
            const uint8_t* src = qst + hf * (BQ * 128) + row * 128;   // 128-byte swizzle: chunk c of a row at c ^ (row & 7)
            float hi[32], lo[32];
#pragma unroll
            for (int c = 0; c < 8; c++) {
                const float4 v = *reinterpret_cast<const float4*>(src + ((c ^ (row & 7)) << 4));
                const float x[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int t = 0; t < 4; t++) { hi[4 * c + t] = hi_part(x[t]); lo[4 * c + t] = x[t] - hi[4 * c + t]; }
            }
            tc::tmem_st32(lb + TM_QHI + hf * 32, hi);
            if (EXACT) tc::tmem_st32(lb + TM_QLO + hf * 32, lo);
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
                const int b = gt % NBUF, use = gt / NBUF;
                const uint32_t sp = lb + TM_SP + 128 * b;
                if (!bwait(&bar->s_full[b], use & 1, abort, &g_attn_watchdog, 11)) { ok = false; break; }
                if (threadIdx.x == 0 && gt < 7) TRACE(2 + 4 * gt);
                tc::tc_fence_after();
                float s[32];
                {
                    float a[32], c2[32];
                    tc::tmem_ld32(sp + hf * 32, a);                      // Q_hi K_hi + Q_lo K_hi
                    if (EXACT) tc::tmem_ld32(sp + 64 + hf * 32, c2);     // Q_hi K_lo
#pragma unroll
                    for (int c = 0; c < 32; c++) s[c] = (EXACT ? a[c] + c2[c] : a[c]) * scale_log2;
                }
                const int k0 = j * BKV + hf * 32;
                if (k0 + 32 > S || (causal && k0 + 31 > it.q0)) {   // half-tile touches the diagonal or the end
#pragma unroll
                    for (int c = 0; c < 32; c++)
                        if (k0 + c >= S || (causal && k0 + c > qi)) s[c] = -INFINITY;
                }
                float mx4[4] = {s[0], s[1], s[2], s[3]};      // 4 independent chains
#pragma unroll
                for (int c = 4; c < 32; c++) mx4[c & 3] = fmaxf(mx4[c & 3], s[c]);
                float mx = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3])), mo;
                if (!exchange(mx, mo)) { ok = false; break; }
                mx = fmaxf(mx, mo);                            // the same value in both threads of the row
                const bool raise = mx > m + RESCALE_THRESHOLD;
                if (__any_sync(0xffffffffu, raise)) {
                    const float mn = raise ? mx : m;
                    const float f = ex2(m - mn);             // 0 on the first tile, 1 for rows that keep m
                    if (j > 0) {   // O holds this item's P_0..P_{j-1} V: wait for it, rescale moved rows
                        const int pg = gt - 1;
                        if (!bwait(&bar->pv_done[pg % NBUF], (pg / NBUF) & 1, abort, &g_attn_watchdog, 12)) { ok = false; break; }
                        tc::tc_fence_after();
#pragma unroll 1
                        for (int q2 = 0; q2 < (EXACT ? 2 : 1); q2++) {
                            float o[32];
                            const uint32_t oc = lb + TM_O + q2 * 64 + hf * 32;
                            tc::tmem_ld32(oc, o);
#pragma unroll
                            for (int c = 0; c < 32; c++) o[c] *= f;
                            tc::tmem_st32(oc, o);
                        }
                        tc::tmem_st_wait();
                    }
                    l *= f;
                    m = mn;
                }
                                float rs4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                for (int c = 0; c < 32; c++) { s[c] = ex2(s[c] - m); rs4[c & 3] += s[c]; }
                l += (rs4[0] + rs4[1]) + (rs4[2] + rs4[3]);
                // P replaces this thread's half of S: hi in the left, lo in the right half
                {
                    float hi[32], lo[32];
#pragma unroll
                    for (int c = 0; c < 32; c++) { hi[c] = hi_part(s[c]); lo[c] = s[c] - hi[c]; }
                    tc::tmem_st32(sp + hf * 32, hi);
                    if (EXACT) tc::tmem_st32(sp + 64 + hf * 32, lo);
                }
                if (threadIdx.x == 0 && gt < 7) TRACE(4 + 4 * gt);
                tc::tmem_st_wait();
                tc::tc_fence_before();
                tc::mbar_arrive(&bar->p_ready[b]);
                if (threadIdx.x == 0 && gt < 7) TRACE(5 + 4 * gt);
            }
            if (!ok) break;
            // the next item's lo parts go in before the O epilogue, so its first S overlaps
            // this item's last PV and the epilogue's stores
            if (threadIdx.x == 0 && ii == 0) TRACE(30);
            if (xn < n_slots && !(ok = take_q(ii + 1))) break;
            if (it.T > 0) {
                float lo_other;
                if (!exchange(l, lo_other)) { ok = false; break; }
                const int pg = gt - 1;
                if (!bwait(&bar->pv_done[pg % NBUF], (pg / NBUF) & 1, abort, &g_attn_watchdog, 13)) { ok = false; break; }
                tc::tc_fence_after();
                if (threadIdx.x == 0 && ii == 0) TRACE(31);
                const float inv = 1.f / (l + lo_other);
                float o[32], o2[32];
                tc::tmem_ld32(lb + TM_O + hf * 32, o);                        // P_hi V_hi + P_lo V_hi
                if (EXACT) tc::tmem_ld32(lb + TM_O + 64 + hf * 32, o2);       // P_hi V_lo
                else {
#pragma unroll
                    for (int c = 0; c < 32; c++) o2[c] = 0.f;
                }
                // O is in registers: free its columns, then stage the rows in the Q stage
                // (this thread's part of it was read by take_q; the previous item's store must
                // have read it) for the PV issuer's TMA store. Stores from these threads were
                // measured to stall them ~1.4 us per item; the copy engine writes the tile
                // off their path.
                tc::tc_fence_before();
                tc::mbar_arrive(&bar->o_free);
                if (threadIdx.x == 0 && ii == 0) TRACE(15);
                if (ii >= 1 && !bwait(&bar->stage_free, (ii - 1) & 1, abort, &g_attn_watchdog, 15)) { ok = false; break; }
                uint8_t* dst = qst + hf * (BQ * 128) + row * 128;
#pragma unroll
                for (int c = 0; c < 8; c++)
                    *reinterpret_cast<float4*>(dst + ((c ^ (row & 7)) << 4)) =
                        make_float4((o[4 * c] + o2[4 * c]) * inv, (o[4 * c + 1] + o2[4 * c + 1]) * inv,
                                    (o[4 * c + 2] + o2[4 * c + 2]) * inv, (o[4 * c + 3] + o2[4 * c + 3]) * inv);
                tc::fence_proxy_async();
                tc::mbar_arrive(&bar->o_staged);
                if (threadIdx.x == 0 && ii == 0) TRACE(19);
            } else {
                tc::tc_fence_before();
                tc::mbar_arrive(&bar->o_free);
                tc::mbar_arrive(&bar->o_staged);
            }
            if (threadIdx.x == 0 && ii == 0) TRACE(32);
            x = xn;
        }
    } else if (warp == W_S) {
        // ======================= S issuer (+ Q loads) =======================
        if (lane == 0) {
            constexpr uint32_t id_s = tc::idesc_tf32(BQ, 2 * BKV, false, false);
            // the lo x lo product is below FP32 resolution: the lo operand multiplies only
            // the hi half of B (N = 64)
            constexpr uint32_t id_s_lo = tc::idesc_tf32(BQ, BKV, false, false);
            auto load_q = [&](const Item& q) {
                const CUtensorMap* maps = gmaps ? gmaps + NMAPS * q.b : pm.m;
                if (gmaps) tc::tmap_acquire(maps);
                const int cb = gmaps ? 0 : q.b;
                tc::mbar_expect_tx(&bar->q_full, Q_STAGE);
                tma_load_4d(qst, maps, &bar->q_full, 0, q.h, q.q0, cb);
                tma_load_4d(qst + BQ * 128, maps, &bar->q_full, 32, q.h, q.q0, cb);
            };
            bool ok = true;
            int gt = 0, ii = 0;
            for (int x = x0; x < n_slots && ok; ii++) {
                const Item it = get_item(x, table, base, bstride, B, H, nqt, S, causal);
                const int xn = next_valid(x, n_slots, per, nqt);
                if (ii == 0) load_q(it);
                if (!bwait(&bar->q_ready, ii & 1, abort, &g_attn_watchdog, 21)) { ok = false; break; }
                // this item's rows are in TMEM: the stage takes the next item's now (after the
                // first item, once the previous item's O store has read it: below)
                if (ii == 0 && xn < n_slots) load_q(get_item(xn, table, base, bstride, B, H, nqt, S, causal));
                for (int j = 0; j < it.T; j++, gt++) {
                    const int st = gt % NSK, b = gt % NBUF, use = gt / NBUF;
                    // buffer b is free once the PV of its previous tile (gt - NBUF) has read P
                    if (!bwait(EXACT && INSPLIT ? &bar->k_split[st] : &bar->k_full[st], (gt / NSK) & 1, abort, &g_attn_watchdog, 22) ||
                        (use >= 1 && !bwait(&bar->pv_done[b], (use - 1) & 1, abort, &g_attn_watchdog, 23))) { ok = false; break; }
                    tc::tc_fence_after();
                    if (gt < 4) TRACE(34 + 2 * gt);
                    const uint32_t kb0 = tc::smem_u32(kst + st * STAGE);
                    const uint32_t sd = tm + TM_SP + 128 * b;
#pragma unroll
                    for (int kb = 0; kb < D / 8; kb++) {
                        const uint32_t koff = (uint32_t)((kb >> 2) * (2 * BKV * 128) + (kb & 3) * 32);
                        const uint64_t bk = tc::smem_desc(kb0 + koff, 16, 1024, tc::SWZ_128B);   // [K_hi | K_lo]
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
                if (!ok) break;
                if (ii >= 1 && xn < n_slots) {
                    if (!bwait(&bar->stage_free, (ii - 1) & 1, abort, &g_attn_watchdog, 20)) { ok = false; break; }
                    load_q(get_item(xn, table, base, bstride, B, H, nqt, S, causal));
                }
                x = xn;
            }
        }
    } else if (warp == W_PV) {
        // ======================= PV issuer =======================
        if (lane == 0) {
            constexpr uint32_t id_o = tc::idesc_tf32(BQ, 2 * D, false, true);
            constexpr uint32_t id_o_lo = tc::idesc_tf32(BQ, D, false, true);
            bool ok = true;
            int gt = 0, ii = 0;
            for (int x = x0; x < n_slots && ok; x = next_valid(x, n_slots, per, nqt), ii++) {
                const Item it = get_item(x, table, base, bstride, B, H, nqt, S, causal);
                for (int j = 0; j < it.T; j++, gt++) {
                    const int st = gt % NSV, b = gt % NBUF, use = gt / NBUF;
                    if (!bwait(&bar->p_ready[b], use & 1, abort, &g_attn_watchdog, 24) ||
                        !bwait(EXACT && INSPLIT ? &bar->v_split[st] : &bar->v_full[st], (gt / NSV) & 1, abort, &g_attn_watchdog, 25)) { ok = false; break; }
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
                if (!ok) break;
                // the item's O rows, staged by the softmax threads: one TMA store per 32-d half
                // (rows past S are clipped by the map)
                if (!bwait(&bar->o_staged, ii & 1, abort, &g_attn_watchdog, 27)) { ok = false; break; }
                if (it.T > 0) {
                    const CUtensorMap* mo = (gmaps ? gmaps + NMAPS * it.b : pm.m) + 5;
                    if (gmaps) tc::tmap_acquire(mo);
                    const int cb = gmaps ? 0 : it.b;
                    for (int a = 0; a < 2; a++)
                        asm volatile("cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5}], [%1];"
                                     ::"l"(reinterpret_cast<uint64_t>(mo)), "r"(tc::smem_u32(qst + a * (BQ * 128))),
                                       "r"(32 * a), "r"(it.h), "r"(it.q0), "r"(cb) : "memory");
                    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
                    asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
                }
                tc::mbar_arrive(&bar->stage_free);
            }
            asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
        }
    } else if (warp >= W_KS) {
        // ======================= in-kernel split: warps 12-13 K, 14-15 V =======================
        // lo = x - hi(x) of each landed raw tile into the stage's lo half. Both halves share
        // the swizzle pattern (K: lo rows are hi rows + 64; V: lo chunks are hi chunks + 2),
        // so lo goes at the hi byte offset plus a constant.
        if (EXACT && INSPLIT) {
            const bool is_k = warp < W_VS;
            const int part = (warp - W_KS) % NSPLIT;      // this warp's share of the tile
            const int NSt = is_k ? NSK : NSV;
            uint8_t* base_st = is_k ? kst : vst;
            uint64_t* full = is_k ? bar->k_full : bar->v_full;
            uint64_t* done = is_k ? bar->k_split : bar->v_split;
            int gt = 0;
            bool ok = true;
            for (int x = x0; x < n_slots && ok; x = next_valid(x, n_slots, per, nqt)) {
                const Item it = get_item(x, table, base, bstride, B, H, nqt, S, causal);
                for (int j = 0; j < it.T; j++, gt++) {
                    const int st = gt % NSt;
                    if (!bwait(&full[st], (gt / NSt) & 1, abort, &g_attn_watchdog, 32)) { ok = false; break; }
                    uint8_t* dst = base_st + st * STAGE;
#pragma unroll 1
                    for (int u0 = 0; u0 < KV_HALF / 16 / 32 / NSPLIT; u0 += 8) {
                        float4 v[8];
                        uint8_t* src[8];
#pragma unroll
                        for (int u = 0; u < 8; u++) {
                            // float4 index in the 16 KB hi data
                            const int i = lane + 32 * (part * (KV_HALF / 16 / 32 / NSPLIT) + u0 + u);
                            src[u] = is_k ? dst + (i >> 9) * (2 * BKV * 128) + (i & 511) * 16 : dst + i * 16;
                            v[u] = *reinterpret_cast<const float4*>(src[u]);
                        }
#pragma unroll
                        for (int u = 0; u < 8; u++)
                            *reinterpret_cast<float4*>(src[u] + (is_k ? BKV * 128 : KV_HALF)) =
                                make_float4(v[u].x - hi_part(v[u].x), v[u].y - hi_part(v[u].y), v[u].z - hi_part(v[u].z),
                                            v[u].w - hi_part(v[u].w));
                    }
                    tc::fence_proxy_async();                  // visible to the tensor core's operand reads
                    __syncwarp();
                    if (lane == 0) tc::mbar_arrive(&done[st]);
                }
            }
        }
    } else {
        // ======================= producers: warp 10 K, warp 11 V =======================
        // One thread per operand puts each key tile in place with TMA: the raw FP32 values
        // (= the hi operand: the MMA reads only their TF32 bits) as two boxes of 32 d x 64
        // keys, swizzled as the MMA reads them; with a split pass, also their lo parts from
        // its copies.
        const bool is_k = warp == W_K;
        if ((warp == W_K || warp == W_V) && lane == 0) {
            // lo comes from the split pass this kernel may have started beside (a no-op
            // without a programmatic dependency)
            if (EXACT && !INSPLIT) asm volatile("griddepcontrol.wait;" ::: "memory");
            const int NSt = is_k ? NSK : NSV;
            uint8_t* base_st = is_k ? kst : vst;
            uint64_t* full = is_k ? bar->k_full : bar->v_full;
            uint64_t* empty = is_k ? bar->k_empty : bar->v_empty;
            int gt = 0;
            bool ok = true;
            for (int x = x0; x < n_slots && ok; x = next_valid(x, n_slots, per, nqt)) {
                const Item it = get_item(x, table, base, bstride, B, H, nqt, S, causal);
                const CUtensorMap* maps = gmaps ? gmaps + NMAPS * it.b : pm.m;
                const int cb = gmaps ? 0 : it.b;         // the batch coordinate of the map
                const CUtensorMap* mhi = maps + (is_k ? 1 : 2);
                const CUtensorMap* mlo = maps + (is_k ? 3 : 4);
                if (is_k && gt == 0) TRACE(3);
                if (gmaps) {
                    tc::tmap_acquire(mhi);
                    if (EXACT && !INSPLIT) tc::tmap_acquire(mlo);
                }
                if (is_k && gt == 0) TRACE(7);
                for (int j = 0; j < it.T; j++, gt++) {
                    const int st = gt % NSt;
                    if (gt >= NSt && !bwait(&empty[st], ((gt / NSt) - 1) & 1, abort, &g_attn_watchdog, 31)) { ok = false; break; }
                    uint8_t* dst = base_st + st * STAGE;
                    tc::mbar_expect_tx(&full[st], EXACT && !INSPLIT ? 2 * KV_HALF : KV_HALF);
                    for (int a = 0; a < 2; a++) {   // d 0-31 and 32-63
                        // K: per 32-d atom 64 hi rows then 64 lo rows; V: hi chunks, then lo chunks
                        uint8_t* h = dst + a * (is_k ? 2 * BKV * 128 : BKV * 128);
                        tma_load_4d(h, mhi, &full[st], 32 * a, it.h, j * BKV, cb);
                        if (EXACT && !INSPLIT) tma_load_4d(h + (is_k ? BKV * 128 : KV_HALF), mlo, &full[st], 32 * a, it.h, j * BKV, cb);
                    }
                    if (gt < 7) TRACE(is_k ? 50 + gt : 57 + (gt < 5 ? gt : 4));
                }
            }
        }
    }

    tc::tc_fence_before();
    __syncthreads();
    if (threadIdx.x == 0) TRACE(63);
    if (bar->abort && (warp == W_S || warp == W_PV) && lane == 0) {   // let issued MMAs retire before TMEM is released
        int never = 0;
        uint64_t* d = warp == W_S ? &bar->drain : &bar->drain_pv;
        tc::mma_commit(d);
        tc::mbar_wait(d, 0, &never, nullptr, 0);
    }
    __syncthreads();
    if (warp == W_S) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tm, TM_COLS);
    }
}

}  // namespace

namespace {
// lo = x - hi(x) (exact in FP32) of every K and V element, into lo[B][2][S][H][D]: the
// split pass of the FP32-exact attention (one read and one write of K and V in HBM).
// The attention kernel is its programmatic dependent: its CTAs start as the split's
// blocks drain from the SMs.
constexpr int SPLIT_THREADS = 256, SPLIT_UNROLL = 1;
__global__ void __launch_bounds__(SPLIT_THREADS) k_attn_split_lo(const LcuAttnGroup* __restrict__ table,
                                                                  LcuAttnGroup base, size_t bstride, int B, size_t n,
                                                                  float* __restrict__ lo) {
    // the attention kernel may start now: it waits (griddepcontrol.wait) before its
    // first read of lo, and prepares everything else meanwhile
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
#if LCU_ATTN_TRACE
    if (blockIdx.x == 0 && threadIdx.x == 0) g_trace[511][0] = gtime();
#endif
    const size_t n4 = n / 4, total = (size_t)B * 2 * n4, stride = (size_t)gridDim.x * blockDim.x;
    auto src_of = [&](size_t i, size_t& dst) -> const float4* {
        const size_t b = i / (2 * n4), r = i - b * 2 * n4, which = r / n4, e = r - which * n4;
        const float* src = table ? (which ? table[b].v : table[b].k) : (which ? base.v : base.k) + b * bstride;
        dst = (b * 2 + which) * n4 + e;
        return reinterpret_cast<const float4*>(src) + e;
    };
    auto lo4 = [](float4 x) {
        return make_float4(x.x - hi_part(x.x), x.y - hi_part(x.y), x.z - hi_part(x.z), x.w - hi_part(x.w));
    };
    float4* lo4p = reinterpret_cast<float4*>(lo);
    size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
    for (; i + (SPLIT_UNROLL - 1) * stride < total; i += SPLIT_UNROLL * stride) {
        float4 x[SPLIT_UNROLL];
        size_t d[SPLIT_UNROLL];
#pragma unroll
        for (int u = 0; u < SPLIT_UNROLL; u++) x[u] = __ldg(src_of(i + u * stride, d[u]));
#pragma unroll
        for (int u = 0; u < SPLIT_UNROLL; u++) lo4p[d[u]] = lo4(x[u]);
    }
    for (; i < total; i += stride) {
        size_t d0;
        const float4 x = __ldg(src_of(i, d0));
        lo4p[d0] = lo4(x);
    }
#if LCU_ATTN_TRACE
    if (threadIdx.x == 0) atomicMax(&g_trace[511][1], gtime());
#endif
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
                                           const float* o, const float* lo, size_t B, size_t S, size_t H) {
    const size_t n = S * H * D;
    // without lo copies (the kernel splits K and V itself) the lo slots repeat the K and V maps
    return make_qkv_map(maps + 0, q, B, S, H, 0, BQ, CU_TENSOR_MAP_SWIZZLE_128B) &&
           make_qkv_map(maps + 1, k, B, S, H, 0, BKV, CU_TENSOR_MAP_SWIZZLE_128B) &&
           make_qkv_map(maps + 2, v, B, S, H, 0, BKV, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B) &&
           (lo ? make_qkv_map(maps + 3, lo, B, S, H, 2 * n, BKV, CU_TENSOR_MAP_SWIZZLE_128B)
               : make_qkv_map(maps + 3, k, B, S, H, 0, BKV, CU_TENSOR_MAP_SWIZZLE_128B)) &&
           (lo ? make_qkv_map(maps + 4, lo + n, B, S, H, 2 * n, BKV, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B)
               : make_qkv_map(maps + 4, v, B, S, H, 0, BKV, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B)) &&
           make_qkv_map(maps + 5, o, B, S, H, 0, BQ, CU_TENSOR_MAP_SWIZZLE_128B);
}

extern "C" size_t lcu_attention_tc_lo_floats(size_t B, size_t S, size_t H) { return 2 * B * S * H * D; }

extern "C" int lcu_attention_tc_supported(size_t D_) { return D_ == (size_t)D; }

// FP32-exact: lo of K and V is made inside the attention kernel unless LCU_ATTN_SPLIT_PASS=1
// (then a split pass writes it into a lo buffer first and the kernel loads it by TMA).
static bool attn_split_pass() {
    static const bool v = [] { const char* e = getenv("LCU_ATTN_SPLIT_PASS"); return e && e[0] == '1'; }();
    return v;
}
extern "C" int lcu_attention_tc_needs_lo(void) { return attn_split_pass() ? 1 : 0; }

extern "C" lancius_error lcu_attention_tc(const LcuAttnGroup* d_table, const float* q, const float* k, const float* v,
                                          float* o, size_t B, size_t S, size_t H, int causal, int mode,
                                          const CUtensorMap* d_maps, float* lo, void* stream) {
    if (B == 0 || S == 0 || H == 0) return LANCIUS_ERROR_OK;
    AttnMaps pm{};
    const bool exact = mode != LCU_MODE_TF32, split_pass = exact && attn_split_pass();
    if (!d_table) {
        if (split_pass && !lo && !(lo = static_cast<float*>(lcu_scratch_acquire(lcu_attention_tc_lo_floats(B, S, H) * 4)))) {
            lancius_set_error(LANCIUS_ERROR_OOM);
            return LANCIUS_ERROR_OOM;
        }
        if (!lcu_attention_tc_make_maps(pm.m, q, k, v, o, lo, B, S, H)) {
            lancius_set_error(LANCIUS_ERROR_INTERNAL);
            return LANCIUS_ERROR_INTERNAL;
        }
    }
    if (d_table && (!d_maps || (split_pass && !lo))) { lancius_set_error(LANCIUS_ERROR_INTERNAL); return LANCIUS_ERROR_INTERNAL; }
    static int sms = 0;
    if (!sms) {
        int dev = 0;
        cudaGetDevice(&dev);
        if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0) sms = LCU_SMS;
    }
    if (split_pass) {
        const size_t total4 = 2 * B * S * H * D / 4;
        k_attn_split_lo<<<lcu_blocks(total4, SPLIT_THREADS, 16u * (unsigned)sms), SPLIT_THREADS, 0, lcu_as_stream(stream)>>>(
            d_table, LcuAttnGroup{q, k, v, o}, S * H * D, (int)B, S * H * D, lo);
        lcu_note_launch();
    }
    static bool configured[64] = {};   // the attribute is per device
    int dev_ = 0;
    cudaGetDevice(&dev_);
    if (dev_ >= 0 && dev_ < 64 && !configured[dev_]) {
        if (cudaFuncSetAttribute(k_attn_tc<true, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES) != cudaSuccess ||
            cudaFuncSetAttribute(k_attn_tc<true, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES) != cudaSuccess ||
            cudaFuncSetAttribute(k_attn_tc<false, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES) != cudaSuccess)
            return lcu_launch_status();
        configured[dev_] = true;
    }
    LcuAttnGroup base{q, k, v, o};
    float scale_log2 = (float)(1.4426950408889634 / 8.0);   // log2(e) / sqrt(64)
    // persistent grid: one CTA per SM (TMEM and shared memory allow no more), each walks
    // pairs of query tiles of equal total cost with stride gridDim.x. After a split pass it
    // is that pass's programmatic dependent: its CTAs start while the split runs and only
    // the loads of lo wait for it.
    const size_t pairs = ((S + BQ - 1) / BQ + 1) / 2 * H * B;
    const unsigned grid = (unsigned)(pairs < (size_t)sms ? pairs : (size_t)sms);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(THREADS);
    cfg.dynamicSmemBytes = SMEM_BYTES;
    cfg.stream = lcu_as_stream(stream);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    static const bool no_pdl = [] { const char* e = getenv("LCU_ATTN_NO_PDL"); return e && e[0] == '1'; }();
    cfg.numAttrs = split_pass && !no_pdl ? 1 : 0;
    const CUtensorMap* dm = d_table ? d_maps : nullptr;
    const size_t bstride = S * H * D;
    cudaError_t e = !exact     ? cudaLaunchKernelEx(&cfg, k_attn_tc<false, false>, d_table, base, bstride, (int)B, (int)S, (int)H,
                                                    causal, scale_log2, dm, pm)
                    : split_pass ? cudaLaunchKernelEx(&cfg, k_attn_tc<true, false>, d_table, base, bstride, (int)B, (int)S,
                                                      (int)H, causal, scale_log2, dm, pm)
                                 : cudaLaunchKernelEx(&cfg, k_attn_tc<true, true>, d_table, base, bstride, (int)B, (int)S,
                                                      (int)H, causal, scale_log2, dm, pm);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return lcu_check_cuda(e);
    }
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
