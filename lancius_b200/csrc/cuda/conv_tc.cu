// Implicit-GEMM CONV2D on the tcgen05 tensor cores without a materialised im2col
// (FP32-exact, 3xTF32). Restates kernel_conv2d_fwd (lancius_kernels.c:28-60): NCHW
// input, OIHW weights, zero padding, stride, optional fused ReLU
// (lancius_vision_ops.c:60-81).
//
//   C[Co][P] = W'[Co][K'] . X'[P][K']^T,  P = N*Ho*Wo,  K' = (kh, kw, ci)
//
// The input is rewritten once as NHWC FP32 (one pass over it, instead of the
// Kh*Kw-times larger im2col); the epilogue warps split each loaded tile into TF32
// hi/lo in shared memory while the MMAs of earlier stages run. For one k-step (kh, kw, 16 channels) the B tile
// of r whole output rows (r * Wo <= 256 pixels of one image) is ONE 4-D TMA load at
// (c, kw - pad, ho0*s - pad + kh, n) with both spatial traversal strides set to the
// conv stride, so the hardware performs the gather and the padding (out-of-range
// coordinates read zeros); pixels land as 64-byte K-major rows in the 64-byte swizzle.
// Weights are rewritten as [Co][kh][kw][ci] hi/lo and loaded as 2-D tiles.
//
//   warp 0      TMA producer (one lane)
//   warp 1      TMEM allocation + tcgen05.mma issue (one lane)
//   warps 2-5   epilogue: tcgen05.ld -> ReLU -> NCHW store
// Tile 256 (two M=128 TMEM accumulators) x r*Wo pixels x 16 channels, 3 stages.
// Requirements (else the im2col path runs): Ci % 16 == 0, Wo * stride <= 256, some
// r with r * Wo % 16 == 0, K' <= 8192.
// Every mbarrier wait is bounded; a timeout sets the watchdog word and unwinds.
#include "tc_common.cuh"
#include <algorithm>
#include <cstdlib>
#include <mutex>

namespace {

constexpr int BM = 256, BN = 256, BK = 16, STAGES = 3, THREADS = 192;
constexpr int A_TILE = BM * BK * 4;                  // 16 KB (two 128-row halves)
constexpr int B_TILE = BN * BK * 4;                  // 16 KB
constexpr int STAGE_BYTES = 2 * A_TILE + 2 * B_TILE; // hi + lo of both
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 + 256;
constexpr uint32_t TMEM_COLS = 512;

__device__ int g_conv_watchdog = 0;

struct Smem {
    uint64_t full[STAGES], empty[STAGES], conv[STAGES], accum, drain;
    uint32_t tmem;
    int abort, consumed;
};

struct ConvArgs {
    int n, ci, co, kh, kw, stride, pad, ho, wo;
    int rows;        // output rows per tile: the tile is rows x Wo pixels of one image
    int halves;      // 1 when Co <= 128
    int passes, relu;
    int raw_b;       // 1: the input map covers plain FP32 NHWC; the epilogue warps split it on chip
    int out_nhwc;    // 1 (persistent kernel only): store the output NHWC for a conv that reads it next
    int tma_out;     // with out_nhwc: the epilogue stages 32 x 32 blocks and stores them by TMA (maps to_hi/to_lo)
    float* out_lo;   // with out_nhwc: also store tf32_lo of every output there (NHWC), so the next
                     // conv loads hi (the value itself) and lo by TMA and needs no splitter
    float* gap;      // NCHW output (persistent kernel): also store each tile's per-channel sum of
                     // its outputs at gap[(img * tiles_per_img + tile) * Co + co], for a global pool
};

__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1, int c2,
                                            int c3) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6}], [%2];"
        ::"r"(tc::smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(tc::smem_u32(bar)), "r"(c0), "r"(c1),
          "r"(c2), "r"(c3)
        : "memory");
}

__global__ void __launch_bounds__(THREADS, 1)
k_conv_tc(const __grid_constant__ CUtensorMap tw_hi, const __grid_constant__ CUtensorMap tw_lo,
          const __grid_constant__ CUtensorMap tx_hi, const __grid_constant__ CUtensorMap tx_lo, float* __restrict__ out,
          ConvArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* tiles = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    Smem* sm = reinterpret_cast<Smem*>(tiles + STAGES * STAGE_BYTES);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int hw = a.ho * a.wo;
    const int tiles_per_img = (a.ho + a.rows - 1) / a.rows;
    const int img = blockIdx.x / tiles_per_img, ho0 = (blockIdx.x % tiles_per_img) * a.rows;
    const int bn = a.rows * a.wo;                    // pixels (MMA N) of this tile
    const int m0 = blockIdx.y * BM;
    const int CB = a.ci / BK, KT = a.kh * a.kw * CB;
    volatile int* abort = &sm->abort;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) {
            tc::mbar_init(&sm->full[s], 1); tc::mbar_init(&sm->empty[s], 1); tc::mbar_init(&sm->conv[s], 4);
        }
        tc::mbar_init(&sm->accum, 1);
        tc::mbar_init(&sm->drain, 1);
        sm->abort = 0;
        sm->consumed = 0;
        tc::fence_barrier_init();
        tc::prefetch_tmap(&tw_hi); tc::prefetch_tmap(&tx_hi);
        if (a.passes > 1) { tc::prefetch_tmap(&tw_lo); if (!a.raw_b) tc::prefetch_tmap(&tx_lo); }
    }
    if (warp == 1) tc::tmem_alloc(&sm->tmem, TMEM_COLS);
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = sm->tmem;
    int issued = 0;

    if (warp == 0 && lane == 0) {
        // ---------------- TMA producer ----------------
        // a box counts all of its bytes, the zero-filled out-of-range part included
        const uint32_t tx = a.raw_b ? (a.passes > 1 ? 2u : 1u) * (uint32_t)A_TILE + (uint32_t)(bn * BK * 4)
                                    : (a.passes > 1 ? 2u : 1u) * (uint32_t)(A_TILE + bn * BK * 4);
        for (int kt = 0; kt < KT; kt++) {
            const int s = kt % STAGES;
            if (kt >= STAGES && !tc::mbar_wait(&sm->empty[s], ((kt / STAGES) - 1) & 1, abort, &g_conv_watchdog, 1)) break;
            const int cb = kt % CB, r = kt / CB, kw = r % a.kw, kh = r / a.kw;
            uint8_t* st = tiles + s * STAGE_BYTES;
            tc::mbar_expect_tx(&sm->full[s], tx);
            tc::tma_load_3d(st, &tw_hi, &sm->full[s], kt * BK, m0, 0);
            if (a.passes > 1) tc::tma_load_3d(st + A_TILE, &tw_lo, &sm->full[s], kt * BK, m0, 0);
            // one box: rows x Wo output pixels, both spatial traversals at the conv stride
            const int ix = -a.pad + kw, iy = ho0 * a.stride - a.pad + kh;
            uint8_t* dst = st + 2 * A_TILE;
            tma_load_4d(dst, &tx_hi, &sm->full[s], cb * BK, ix, iy, img);
            if (a.passes > 1 && !a.raw_b) tma_load_4d(dst + B_TILE, &tx_lo, &sm->full[s], cb * BK, ix, iy, img);
            issued = kt + 1;
        }
    } else if (warp == 1 && lane == 0) {
        // ---------------- MMA issuer ----------------
        const uint32_t idesc = tc::idesc_tf32(128, bn, false, false);
        bool ok = true;
        for (int kt = 0; kt < KT; kt++) {
            const int s = kt % STAGES;
            if (!tc::mbar_wait(a.raw_b ? &sm->conv[s] : &sm->full[s], (kt / STAGES) & 1, abort, &g_conv_watchdog, 2)) {
                ok = false; break;
            }
            tc::tc_fence_after();
            const uint32_t st = tc::smem_u32(tiles + s * STAGE_BYTES);
            const uint32_t a_hi = st, a_lo = st + A_TILE, b_hi = st + 2 * A_TILE, b_lo = b_hi + B_TILE;
#pragma unroll
            for (int kb = 0; kb < BK / 8; kb++) {
                const uint64_t dbh = tc::smem_desc(b_hi + kb * 32, 16, 512, tc::SWZ_64B);
                const uint64_t dbl = tc::smem_desc(b_lo + kb * 32, 16, 512, tc::SWZ_64B);
                for (int half = 0; half < a.halves; half++) {
                    const uint32_t hoff = (uint32_t)half * (128 * BK * 4), d = tmem + (uint32_t)half * BN;
                    const uint64_t dah = tc::smem_desc(a_hi + hoff + kb * 32, 16, 512, tc::SWZ_64B);
                    const uint32_t acc = (kt | kb) ? 1u : 0u;
                    if (a.passes > 1) {
                        const uint64_t dal = tc::smem_desc(a_lo + hoff + kb * 32, 16, 512, tc::SWZ_64B);
                        tc::mma_tf32(d, dal, dbh, idesc, acc);      // small terms first
                        tc::mma_tf32(d, dah, dbl, idesc, 1u);
                        tc::mma_tf32(d, dah, dbh, idesc, 1u);
                    } else {
                        tc::mma_tf32(d, dah, dbh, idesc, acc);
                    }
                }
            }
            tc::mma_commit(&sm->empty[s]);
            sm->consumed = kt + 1;
        }
        if (ok) tc::mma_commit(&sm->accum);
    } else if (warp >= 2) {
        if (a.raw_b) {
            // ---------------- input splitter (raw-B mode) ----------------
            // the FP32 tile serves as hi as it is (the MMA reads it truncated to TF32);
            // lo = rna_tf32(x - tf32_hi(x)) goes to the stage's lo slot; the swizzle permutes
            // 16-byte chunks identically in both, so a flat pass suffices
            const int n4 = bn * BK / 4;
            for (int kt = 0; kt < KT; kt++) {
                const int s = kt % STAGES;
                if (!tc::mbar_wait(&sm->full[s], (kt / STAGES) & 1, abort, &g_conv_watchdog, 4)) break;
                float4* b4 = reinterpret_cast<float4*>(tiles + s * STAGE_BYTES + 2 * A_TILE);
#pragma unroll 4
                for (int i = threadIdx.x - 64; i < n4 && a.passes > 1; i += 128)
                    b4[i + B_TILE / 16] = tc::tf32_lo4(b4[i]);
                tc::fence_proxy_async();
                __syncwarp();
                if (lane == 0) tc::mbar_arrive(&sm->conv[s]);
            }
        }
        // ---------------- epilogue: rows = output channels, columns = pixels ----------------
        if (tc::mbar_wait(&sm->accum, 0, abort, &g_conv_watchdog, 3)) {
            tc::tc_fence_after();
            // Each warp owns 32 output channels (TMEM lanes). Per 32-pixel chunk the 32x32
            // block is staged in the drained pipeline smem and stored by channel rows: 8
            // lanes per row x 4 pixels, so every store instruction writes whole 128-byte
            // segments (coalesced) from a compact loop.
            const int q = warp & 3;
            float* sb = reinterpret_cast<float*>(tiles) + (size_t)q * 32 * 36;
            // the tile's pixels are consecutive in the image: rows ho0.. of width Wo
            const int valid = min(bn, (a.ho - ho0) * a.wo);
            const bool v4 = hw % 4 == 0 && ((size_t)ho0 * a.wo) % 4 == 0 && (reinterpret_cast<uintptr_t>(out) & 15) == 0;
            for (int half = 0; half < a.halves; half++) {
                const int co0 = m0 + half * 128 + 32 * q;
                for (int c = 0; c < bn; c += 32) {
                    float v[32];
                    tc::tmem_ld32(tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(half * BN + c), v);
#pragma unroll
                    for (int j = 0; j < 32; j += 4)
                        *reinterpret_cast<float4*>(sb + lane * 36 + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
                    __syncwarp();
                    const int px = c + 4 * (lane & 7);
#pragma unroll 2
                    for (int it = 0; it < 8; it++) {
                        const int r = 4 * it + (lane >> 3), co = co0 + r;
                        if (co >= a.co || px >= valid) continue;
                        float4 x = *reinterpret_cast<const float4*>(sb + r * 36 + 4 * (lane & 7));
                        if (a.relu) { x.x = fmaxf(x.x, 0.f); x.y = fmaxf(x.y, 0.f); x.z = fmaxf(x.z, 0.f); x.w = fmaxf(x.w, 0.f); }
                        float* o = out + ((size_t)img * a.co + co) * hw + (size_t)ho0 * a.wo + px;
                        if (v4 && px + 4 <= valid) {
                            *reinterpret_cast<float4*>(o) = x;
                        } else {
                            const float xv[4] = {x.x, x.y, x.z, x.w};
                            for (int t = 0; t < 4 && px + t < valid; t++) o[t] = xv[t];
                        }
                    }
                    __syncwarp();
                }
            }
        }
    }

    tc::tc_fence_before();
    __syncthreads();
    if (sm->abort) {
        int never = 0;
        if (warp == 0 && lane == 0)
            for (int kt = sm->consumed; kt < issued; kt++)
                if (!tc::mbar_wait(&sm->full[kt % STAGES], (kt / STAGES) & 1, &never, nullptr, 0)) break;
        if (warp == 1 && lane == 0) {
            tc::mma_commit(&sm->drain);
            tc::mbar_wait(&sm->drain, 0, &never, nullptr, 0);
        }
        __syncthreads();
    }
    if (warp == 1) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem, TMEM_COLS);
    }
}

// Persistent variant for output-channel tiles of 128: one CTA per SM walks the tiles
// (pixel tile x 128-channel tile) round-robin; the accumulator of one tile takes 256
// TMEM columns, so two of them alternate and the epilogue of a tile (TMEM -> ReLU ->
// NCHW) overlaps the MMAs of the next. Roles as in k_conv_tc; the epilogue stages its
// blocks in a dedicated XOR-swizzled buffer because the ring already holds the next
// tile's stages. The input comes as NHWC TF32 hi/lo (pre-split) or, in raw-B mode, as
// plain FP32 that warps 6-9 split on chip.
constexpr int PT_BM = 128, PT_STAGES = 4;
constexpr int PT_A_TILE = PT_BM * BK * 4;                       // 8 KB
constexpr int PT_STAGE_BYTES = 2 * PT_A_TILE + 2 * B_TILE;      // 48 KB
// epilogue staging: per epilogue warp 32 x 32 floats (NCHW transpose) or, for a TMA-stored
// NHWC output, a hi and a lo block of 32 pixels x 32 channels (128-byte swizzled rows)
constexpr int PT_EPI_FLOATS = 4 * 2 * 32 * 32;
constexpr int PT_SMEM_BYTES = PT_STAGES * PT_STAGE_BYTES + PT_EPI_FLOATS * 4 + 1024 + 256;

constexpr int PT_THREADS = 320;

struct SmemPT {
    uint64_t full[PT_STAGES], empty[PT_STAGES], conv[PT_STAGES], acc_full[2], acc_empty[2], drain;
    uint32_t tmem;
    int abort, consumed;
};

__global__ void __launch_bounds__(PT_THREADS, 1)
k_conv_pt(const __grid_constant__ CUtensorMap tw_hi, const __grid_constant__ CUtensorMap tw_lo,
          const __grid_constant__ CUtensorMap tx_hi, const __grid_constant__ CUtensorMap tx_lo, float* __restrict__ out,
          ConvArgs a, const __grid_constant__ CUtensorMap to_hi, const __grid_constant__ CUtensorMap to_lo) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* tiles = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    float* stage_f = reinterpret_cast<float*>(tiles + PT_STAGES * PT_STAGE_BYTES);
    SmemPT* sm = reinterpret_cast<SmemPT*>(stage_f + PT_EPI_FLOATS);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int hw = a.ho * a.wo;
    const int tiles_per_img = (a.ho + a.rows - 1) / a.rows;
    const int ct = (a.co + PT_BM - 1) / PT_BM;
    const int T = a.n * tiles_per_img * ct;
    const int bn = a.rows * a.wo;                    // pixels (MMA N) of a tile
    const int CB = a.ci / BK, KT = a.kh * a.kw * CB;
    volatile int* abort = &sm->abort;
    auto coords = [&](int t, int& img, int& ho0, int& m0) {
        const int pt = t / ct;
        m0 = (t - pt * ct) * PT_BM;
        img = pt / tiles_per_img;
        ho0 = (pt - img * tiles_per_img) * a.rows;
    };

    if (threadIdx.x == 0) {
        for (int s = 0; s < PT_STAGES; s++) {
            tc::mbar_init(&sm->full[s], 1); tc::mbar_init(&sm->empty[s], 1); tc::mbar_init(&sm->conv[s], 4);
        }
        for (int b = 0; b < 2; b++) { tc::mbar_init(&sm->acc_full[b], 1); tc::mbar_init(&sm->acc_empty[b], 4); }
        tc::mbar_init(&sm->drain, 1);
        sm->abort = 0;
        sm->consumed = 0;
        tc::fence_barrier_init();
        tc::prefetch_tmap(&tw_hi); tc::prefetch_tmap(&tx_hi);
        if (a.passes > 1) { tc::prefetch_tmap(&tw_lo); if (!a.raw_b) tc::prefetch_tmap(&tx_lo); }
    }
    if (warp == 1) tc::tmem_alloc(&sm->tmem, TMEM_COLS);
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = sm->tmem;
    int issued = 0;

    if (warp == 0 && lane == 0) {
        // ---------------- TMA producer ----------------
        const uint32_t tx = a.raw_b ? (a.passes > 1 ? 2u : 1u) * (uint32_t)PT_A_TILE + (uint32_t)(bn * BK * 4)
                                    : (a.passes > 1 ? 2u : 1u) * (uint32_t)(PT_A_TILE + bn * BK * 4);
        int it = 0;
        bool ok = true;
        for (int t = blockIdx.x; t < T && ok; t += gridDim.x) {
            int img, ho0, m0;
            coords(t, img, ho0, m0);
            for (int kt = 0; kt < KT; kt++, it++) {
                const int s = it % PT_STAGES;
                if (it >= PT_STAGES && !tc::mbar_wait(&sm->empty[s], ((it / PT_STAGES) - 1) & 1, abort, &g_conv_watchdog, 11)) {
                    ok = false; break;
                }
                const int cb = kt % CB, r = kt / CB, kw = r % a.kw, kh = r / a.kw;
                uint8_t* st = tiles + s * PT_STAGE_BYTES;
                tc::mbar_expect_tx(&sm->full[s], tx);
                tc::tma_load_3d(st, &tw_hi, &sm->full[s], kt * BK, m0, 0);
                if (a.passes > 1) tc::tma_load_3d(st + PT_A_TILE, &tw_lo, &sm->full[s], kt * BK, m0, 0);
                const int ix = -a.pad + kw, iy = ho0 * a.stride - a.pad + kh;
                uint8_t* dst = st + 2 * PT_A_TILE;
                tma_load_4d(dst, &tx_hi, &sm->full[s], cb * BK, ix, iy, img);
                if (a.passes > 1 && !a.raw_b) tma_load_4d(dst + B_TILE, &tx_lo, &sm->full[s], cb * BK, ix, iy, img);
                issued = it + 1;
            }
        }
    } else if (warp == 1 && lane == 0) {
        // ---------------- MMA issuer ----------------
        const uint32_t idesc = tc::idesc_tf32(128, bn, false, false);
        int it = 0, j = 0;
        bool ok = true;
        for (int t = blockIdx.x; t < T && ok; t += gridDim.x, j++) {
            const int b = j & 1;
            if (j >= 2 && !tc::mbar_wait(&sm->acc_empty[b], ((j >> 1) - 1) & 1, abort, &g_conv_watchdog, 12)) break;
            tc::tc_fence_after();
            const uint32_t d = tmem + (uint32_t)b * 256;
            for (int kt = 0; kt < KT; kt++, it++) {
                const int s = it % PT_STAGES;
                if (!tc::mbar_wait(a.raw_b ? &sm->conv[s] : &sm->full[s], (it / PT_STAGES) & 1, abort, &g_conv_watchdog, 13)) {
                    ok = false; break;
                }
                tc::tc_fence_after();
                const uint32_t st = tc::smem_u32(tiles + s * PT_STAGE_BYTES);
                const uint32_t a_hi = st, a_lo = st + PT_A_TILE, b_hi = st + 2 * PT_A_TILE, b_lo = b_hi + B_TILE;
#pragma unroll
                for (int kb = 0; kb < BK / 8; kb++) {
                    const uint64_t dbh = tc::smem_desc(b_hi + kb * 32, 16, 512, tc::SWZ_64B);
                    const uint64_t dah = tc::smem_desc(a_hi + kb * 32, 16, 512, tc::SWZ_64B);
                    const uint32_t acc = (kt | kb) ? 1u : 0u;
                    if (a.passes > 1) {
                        const uint64_t dbl = tc::smem_desc(b_lo + kb * 32, 16, 512, tc::SWZ_64B);
                        const uint64_t dal = tc::smem_desc(a_lo + kb * 32, 16, 512, tc::SWZ_64B);
                        tc::mma_tf32(d, dal, dbh, idesc, acc);      // small terms first
                        tc::mma_tf32(d, dah, dbl, idesc, 1u);
                        tc::mma_tf32(d, dah, dbh, idesc, 1u);
                    } else {
                        tc::mma_tf32(d, dah, dbh, idesc, acc);
                    }
                }
                tc::mma_commit(&sm->empty[s]);
                sm->consumed = it + 1;
            }
            if (!ok) break;
            tc::mma_commit(&sm->acc_full[b]);
        }
    } else if (warp >= 6) {
        // ---------------- input splitter (raw-B mode) ----------------
        if (a.raw_b) {
            const int n4 = bn * BK / 4;
            int it = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < T && ok; t += gridDim.x) {
                for (int kt = 0; kt < KT; kt++, it++) {
                    const int s = it % PT_STAGES;
                    if (!tc::mbar_wait(&sm->full[s], (it / PT_STAGES) & 1, abort, &g_conv_watchdog, 15)) { ok = false; break; }
                    float4* b4 = reinterpret_cast<float4*>(tiles + s * PT_STAGE_BYTES + 2 * PT_A_TILE);
#pragma unroll 4
                    for (int i = threadIdx.x - 192; i < n4 && a.passes > 1; i += 128)
                        b4[i + B_TILE / 16] = tc::tf32_lo4(b4[i]);
                    tc::fence_proxy_async();
                    __syncwarp();
                    if (lane == 0) tc::mbar_arrive(&sm->conv[s]);
                }
            }
        }
    } else if (warp >= 2) {
        // ---------------- epilogue: rows = output channels, columns = pixels ----------------
        const int q = warp & 3;
        float* sb = stage_f + q * 2 * 32 * 32;       // 32x32 block, float4 slots XOR-swizzled by row
        const bool v4base = hw % 4 == 0 && (reinterpret_cast<uintptr_t>(out) & 15) == 0;
        int j = 0;
        for (int t = blockIdx.x; t < T; t += gridDim.x, j++) {
            const int b = j & 1;
            int img, ho0, m0;
            coords(t, img, ho0, m0);
            if (!tc::mbar_wait(&sm->acc_full[b], (j >> 1) & 1, abort, &g_conv_watchdog, 14)) break;
            tc::tc_fence_after();
            const int valid = min(bn, (a.ho - ho0) * a.wo);
            const bool v4 = v4base && ((size_t)ho0 * a.wo) % 4 == 0;
            const int co0 = m0 + 32 * q;
            const uint32_t tbase = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)b * 256;
            uint32_t va[32];
            float gsum = 0.f;                            // this channel's sum over the tile's pixels
            tc::tmem_ld32_issue(tbase, va);
            for (int c = 0; c < bn; c += 32) {
                tc::tmem_ld_wait(va);
                if (a.gap) {
#pragma unroll
                    for (int px = 0; px < 32; px++) {
                        float x = __uint_as_float(va[px]);
                        if (a.relu) x = fmaxf(x, 0.f);
                        if (c + px < valid) gsum += x;
                    }
                }
                if (a.tma_out) {
                    // NHWC by TMA: lane = channel; the block is staged as 32 pixel rows of 32
                    // channels (128-byte swizzle) in hi and lo halves and stored as one box
                    // each, clipped at the image's last pixel and at Co. Plain stores of these
                    // rows were measured to cost ~120 us of the conv stack's 0.81 ms.
                    if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");   // previous block read
                    __syncwarp();
                    float* sl = sb + 32 * 32;
#pragma unroll
                    for (int px = 0; px < 32; px++) {
                        float x = __uint_as_float(va[px]);
                        if (a.relu) x = fmaxf(x, 0.f);
                        const int o = px * 32 + ((((lane >> 2) ^ (px & 7))) << 2) + (lane & 3);
                        sb[o] = x;
                        if (a.out_lo) sl[o] = tc::tf32_lo(x);
                    }
                    if (c + 32 < bn) tc::tmem_ld32_issue(tbase + (uint32_t)(c + 32), va);
                    tc::fence_proxy_async();
                    __syncwarp();
                    if (lane == 0 && c < valid) {
                        const int pix = ho0 * a.wo + c;
                        asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];"
                                     ::"l"(reinterpret_cast<uint64_t>(&to_hi)), "r"(tc::smem_u32(sb)), "r"(co0), "r"(pix), "r"(img)
                                     : "memory");
                        if (a.out_lo)
                            asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];"
                                         ::"l"(reinterpret_cast<uint64_t>(&to_lo)), "r"(tc::smem_u32(sl)), "r"(co0), "r"(pix),
                                           "r"(img) : "memory");
                        asm volatile("cp.async.bulk.commit_group;" ::: "memory");
                    }
                    continue;
                }
#pragma unroll
                for (int jj = 0; jj < 8; jj++)
                    *reinterpret_cast<float4*>(sb + lane * 32 + ((jj ^ (lane & 7)) << 2)) =
                        make_float4(__uint_as_float(va[4 * jj]), __uint_as_float(va[4 * jj + 1]),
                                    __uint_as_float(va[4 * jj + 2]), __uint_as_float(va[4 * jj + 3]));
                __syncwarp();
                if (c + 32 < bn) tc::tmem_ld32_issue(tbase + (uint32_t)(c + 32), va);
                if (a.out_nhwc) {
                    // NHWC: lane = channel, one 128-byte channel run per pixel and store
                    const int co = co0 + lane;
                    float* o = out + ((size_t)img * hw + (size_t)ho0 * a.wo + c) * a.co + co;
                    for (int pxi = 0; pxi < 32 && c + pxi < valid; pxi++) {
                        float x = sb[lane * 32 + ((((pxi >> 2) ^ (lane & 7))) << 2) + (pxi & 3)];
                        if (a.relu) x = fmaxf(x, 0.f);
                        if (co < a.co) {
                            o[(size_t)pxi * a.co] = x;
                            if (a.out_lo) a.out_lo[(o - out) + (size_t)pxi * a.co] = tc::tf32_lo(x);
                        }
                    }
                    __syncwarp();
                    continue;
                }
                const int cl4 = lane & 7, px = c + 4 * cl4;
#pragma unroll 2
                for (int it = 0; it < 8; it++) {
                    const int r = 4 * it + (lane >> 3), co = co0 + r;
                    if (co >= a.co || px >= valid) continue;
                    float4 x = *reinterpret_cast<const float4*>(sb + r * 32 + ((cl4 ^ (r & 7)) << 2));
                    if (a.relu) { x.x = fmaxf(x.x, 0.f); x.y = fmaxf(x.y, 0.f); x.z = fmaxf(x.z, 0.f); x.w = fmaxf(x.w, 0.f); }
                    float* o = out + ((size_t)img * a.co + co) * hw + (size_t)ho0 * a.wo + px;
                    if (v4 && px + 4 <= valid) {
                        *reinterpret_cast<float4*>(o) = x;
                    } else {
                        const float xv[4] = {x.x, x.y, x.z, x.w};
                        for (int u = 0; u < 4 && px + u < valid; u++) o[u] = xv[u];
                    }
                }
                __syncwarp();
            }
            if (a.gap && co0 + lane < a.co)
                a.gap[((size_t)img * tiles_per_img + ho0 / a.rows) * a.co + co0 + lane] = gsum;
            tc::tc_fence_before();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&sm->acc_empty[b]);
        }
        if (a.tma_out && lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
    }

    tc::tc_fence_before();
    __syncthreads();
    if (sm->abort) {
        int never = 0;
        if (warp == 0 && lane == 0)
            for (int kt = sm->consumed; kt < issued; kt++)
                if (!tc::mbar_wait(&sm->full[kt % PT_STAGES], (kt / PT_STAGES) & 1, &never, nullptr, 0)) break;
        if (warp == 1 && lane == 0) {
            tc::mma_commit(&sm->drain);
            tc::mbar_wait(&sm->drain, 0, &never, nullptr, 0);
        }
        __syncthreads();
    }
    if (warp == 1) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem, TMEM_COLS);
    }
}

// NCHW -> NHWC, as TF32 hi / lo (lo = 0 pointer: TF32 mode) or plain FP32 (round = 0,
// split later on chip): per (n, h) tiles of 32 channels x 64 columns through shared
// memory, float4 on both sides (C % 4 == 0).
__global__ void __launch_bounds__(256) k_nhwc_split(const float* __restrict__ in, float* __restrict__ hi,
                                                    float* __restrict__ lo, int C, int H, int W, int round) {
    __shared__ float t[32][65];
    const int nh = blockIdx.z, n = nh / H, h = nh % H;
    const int c0 = blockIdx.y * 32, w0 = blockIdx.x * 64;
    const bool vin = W % 4 == 0 && (reinterpret_cast<uintptr_t>(in) & 15) == 0;
    for (int idx = threadIdx.x; idx < 32 * 16; idx += 256) {
        const int c = idx >> 4, w = 4 * (idx & 15);
        const float* src = in + (((size_t)n * C + c0 + c) * H + h) * W + w0 + w;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (c0 + c < C) {
            if (vin && w0 + w + 3 < W) v = __ldg(reinterpret_cast<const float4*>(src));
            else {
                if (w0 + w < W) v.x = src[0];
                if (w0 + w + 1 < W) v.y = src[1];
                if (w0 + w + 2 < W) v.z = src[2];
                if (w0 + w + 3 < W) v.w = src[3];
            }
        }
        t[c][w] = v.x; t[c][w + 1] = v.y; t[c][w + 2] = v.z; t[c][w + 3] = v.w;
    }
    __syncthreads();
    for (int idx = threadIdx.x; idx < 64 * 8; idx += 256) {
        const int w = idx >> 3, c = 4 * (idx & 7);
        if (w0 + w >= W || c0 + c >= C) continue;
        float x[4] = {t[c][w], t[c + 1][w], t[c + 2][w], t[c + 3][w]}, xh[4], xl[4];
#pragma unroll
        for (int j = 0; j < 4; j++) {
            xh[j] = round ? tc::tf32_hi(x[j]) : x[j];
            xl[j] = tc::tf32_lo(x[j]);
        }
        const size_t o = (((size_t)n * H + h) * W + w0 + w) * C + c0 + c;
        *reinterpret_cast<float4*>(hi + o) = make_float4(xh[0], xh[1], xh[2], xh[3]);
        if (lo) *reinterpret_cast<float4*>(lo + o) = make_float4(xl[0], xl[1], xl[2], xl[3]);
    }
}

// NHWC -> NCHW (the layout a download hands back for a conv output kept NHWC between
// two convs), FP32 or FP64 out: per (n, h) tiles of 64 columns x 32 channels.
template <typename T>
__global__ void __launch_bounds__(256) k_nhwc_to_nchw(T* __restrict__ out, const float* __restrict__ in, int C, int H,
                                                      int W) {
    __shared__ float t[64][33];
    const int nh = blockIdx.z, n = nh / H, h = nh % H;
    const int c0 = blockIdx.y * 32, w0 = blockIdx.x * 64;
    for (int idx = threadIdx.x; idx < 64 * 32; idx += 256) {
        const int w = idx >> 5, c = idx & 31;
        t[w][c] = (w0 + w < W && c0 + c < C) ? in[(((size_t)n * H + h) * W + w0 + w) * C + c0 + c] : 0.f;
    }
    __syncthreads();
    for (int idx = threadIdx.x; idx < 32 * 64; idx += 256) {
        const int c = idx >> 6, w = idx & 63;
        if (w0 + w < W && c0 + c < C) out[(((size_t)n * C + c0 + c) * H + h) * W + w0 + w] = (T)t[w][c];
    }
}

// OIHW -> [Co][Kh][Kw][Ci] TF32 hi / lo
__global__ void k_weight_khwc_split(const float* __restrict__ w, float* __restrict__ hi, float* __restrict__ lo, int Co,
                                    int Ci, int Kh, int Kw) {
    const size_t n = (size_t)Co * Ci * Kh * Kw;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const int ci = (int)(i % Ci);
        size_t r = i / Ci;
        const int kw = (int)(r % Kw); r /= Kw;
        const int kh = (int)(r % Kh);
        const int co = (int)(r / Kh);
        const float x = w[(((size_t)co * Ci + ci) * Kh + kh) * Kw + kw];
        hi[i] = tc::tf32_hi(x);
        if (lo) lo[i] = tc::tf32_lo(x);
    }
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

size_t al256(size_t v) { return (v + 255) & ~size_t(255); }

// output rows per tile: the most rows r with r * Wo <= 256 and r * Wo % 16 == 0 (the
// MMA's N), the box spans (r - 1) * stride + 1 input rows of at most 256; 0 if none
int pick_rows(int wo, int ho, int stride) {
    if (wo <= 0 || wo * stride > 256) return 0;
    for (int r = BN / wo; r >= 1; r--)
        if ((r * wo) % 16 == 0 && r * stride <= 256 && r <= ho) return r;
    return 0;
}

bool configure() {
    static bool done[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && done[dev]) return true;
    if (cudaFuncSetAttribute(k_conv_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES) != cudaSuccess ||
        cudaFuncSetAttribute(k_conv_pt, cudaFuncAttributeMaxDynamicSharedMemorySize, PT_SMEM_BYTES) != cudaSuccess)
        return false;
    if (dev >= 0 && dev < 64) done[dev] = true;
    return true;
}

}  // namespace

extern "C" int lcu_conv_nhwc_supported(LcuConvShape cs) {
    return cs.ci % BK == 0 && cs.ci > 0 && cs.stride >= 1 && cs.stride <= 8 && pick_rows(cs.wo, cs.ho, cs.stride) &&
           cs.kh * cs.kw * cs.ci <= 8192 && (size_t)cs.n * cs.ho * cs.wo < (1u << 31);
}

extern "C" size_t lcu_conv_nhwc_scratch_bytes(LcuConvShape cs, int passes) {
    const size_t x = (size_t)cs.n * cs.h * cs.w * cs.ci * 4, w = (size_t)cs.co * cs.ci * cs.kh * cs.kw * 4;
    return (passes > 1 ? 2 : 1) * (al256(x) + al256(w));
}

extern "C" lancius_error lcu_conv2d_tc_nhwc(float* out, const float* in, const float* w, LcuConvShape cs, int relu,
                                            int mode, void* scratch, void* stream) {
    return lcu_conv2d_tc_nhwc_ex(out, in, w, cs, relu, mode, scratch, stream, 0, 0, nullptr, nullptr, nullptr, nullptr,
                                 nullptr, nullptr);
}

static bool conv_pt_enabled() {
    const char* e = getenv("LCU_CONV_NO_PT");
    return !(e && e[0] == '1');
}

extern "C" int lcu_conv_nhwc_out_ok(LcuConvShape cs) { return lcu_conv_nhwc_supported(cs) && conv_pt_enabled(); }

extern "C" lancius_error lcu_nhwc_to_nchw(void* out, const float* in, int n, int c, int h, int w, int f64, void* stream) {
    const dim3 grid((unsigned)((w + 63) / 64), (unsigned)((c + 31) / 32), (unsigned)(n * h));
    if (f64) k_nhwc_to_nchw<double><<<grid, 256, 0, lcu_as_stream(stream)>>>(static_cast<double*>(out), in, c, h, w);
    else k_nhwc_to_nchw<float><<<grid, 256, 0, lcu_as_stream(stream)>>>(static_cast<float*>(out), in, c, h, w);
    return lcu_launch_status();
}

// in_nhwc: `in` already holds the input as NHWC FP32 (written by the previous conv);
// in_lo: with in_nhwc, tf32_lo of that input (NHWC), loaded by TMA instead of split on chip;
// out_nhwc: store the output NHWC (persistent kernel only); out_lo: also its tf32_lo.
// The [Co][Kh][Kw][Ci] TF32 hi/lo copies of OIHW weights that the direct conv streams (a
// weight cache refreshes them once per upload instead of once per run).
extern "C" lancius_error lcu_conv_weight_split(const float* w, float* hi, float* lo, int co, int ci, int kh, int kw,
                                               void* stream) {
    const size_t we = (size_t)co * ci * kh * kw;
    if (!we) return LANCIUS_ERROR_OK;
    k_weight_khwc_split<<<lcu_blocks(we, 256), 256, 0, lcu_as_stream(stream)>>>(w, hi, lo, co, ci, kh, kw);
    lcu_note_launch();
    return lcu_launch_status();
}

// Per-channel tile sums for a global average pool after the conv: the tiles of an image and
// their [img][tile][Co] sums (lcu_conv2d_tc_nhwc_ex's gap buffer).
extern "C" int lcu_conv_tiles_per_image(LcuConvShape cs) {
    const int rows = pick_rows(cs.wo, cs.ho, cs.stride);
    return rows ? (cs.ho + rows - 1) / rows : 0;
}

__global__ void k_sum_tile_partials(float* __restrict__ out, const float* __restrict__ part, int n, int co, int tiles) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n * co) return;
    const int img = i / co, c = i - img * co;
    const float* p = part + (size_t)img * tiles * co + c;
    float s = 0.f;
    for (int t = 0; t < tiles; t++) s += p[(size_t)t * co];
    out[i] = s;
}

// out[img * Co + c] = sum over the image's tiles of gap[(img * tiles + t) * Co + c]
extern "C" lancius_error lcu_conv_gap_sum(float* out, const float* gap, int n, int co, int tiles, void* stream) {
    if (n <= 0 || co <= 0) return LANCIUS_ERROR_OK;
    k_sum_tile_partials<<<(unsigned)((n * co + 255) / 256), 256, 0, lcu_as_stream(stream)>>>(out, gap, n, co, tiles);
    lcu_note_launch();
    return lcu_launch_status();
}

// w_hi / w_lo: the weights already split (lcu_conv_weight_split), or NULL to split them here.
// gap: where the persistent kernel with an NCHW output also stores per-tile channel sums
// ([img][tile][Co], lcu_conv_tiles_per_image tiles); *gap_written tells whether it did.
extern "C" lancius_error lcu_conv2d_tc_nhwc_ex(float* out, const float* in, const float* w, LcuConvShape cs, int relu,
                                               int mode, void* scratch, void* stream, int in_nhwc, int out_nhwc,
                                               const float* in_lo, float* out_lo, const float* w_hi, const float* w_lo,
                                               float* gap, int* gap_written) {
    if (gap_written) *gap_written = 0;
    const int passes = mode == LCU_MODE_TF32 ? 1 : 3;
    if (!lcu_conv_nhwc_supported(cs) || !scratch) { lancius_set_error(LANCIUS_ERROR_UNSUPPORTED_OP); return LANCIUS_ERROR_UNSUPPORTED_OP; }
    cudaStream_t st = lcu_as_stream(stream);
    const size_t xe = (size_t)cs.n * cs.h * cs.w * cs.ci, K = (size_t)cs.ci * cs.kh * cs.kw, we = (size_t)cs.co * K;
    char* s = static_cast<char*>(scratch);
    // persistent kernel (128-channel tiles, pre-split NHWC input) unless disabled; the
    // one-launch-per-tile kernel takes the input NHWC as plain FP32 and splits it on chip
    static int n_sm = 0;
    if (!n_sm) { int dev = 0; cudaGetDevice(&dev); cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev); }
    const bool pt = conv_pt_enabled() && n_sm > 0;
    if (out_nhwc && !pt) {
        lancius_set_error(LANCIUS_ERROR_UNSUPPORTED_OP); return LANCIUS_ERROR_UNSUPPORTED_OP;
    }
    // the persistent kernel takes its input pre-split unless it reads a conv's NHWC output
    // in place (its 128-channel tiles leave little shared-memory bandwidth for a splitter)
    const int raw = in_nhwc ? (in_lo && passes > 1 ? 0 : 1) : (lcu_no_raw_a() || pt) ? 0 : 1;
    float* xh = reinterpret_cast<float*>(s); s += al256(xe * 4);
    float* xl = passes > 1 && !raw ? reinterpret_cast<float*>(s) : nullptr; if (passes > 1) s += al256(xe * 4);
    float* wh = reinterpret_cast<float*>(s); s += al256(we * 4);
    float* wl = passes > 1 ? reinterpret_cast<float*>(s) : nullptr;

    if (in_nhwc) {
        xh = const_cast<float*>(in);                  // read in place (the MMA truncates it to hi)
        if (!raw) xl = const_cast<float*>(in_lo);     // lo written by the producer; else split on chip
    } else {
        k_nhwc_split<<<dim3((unsigned)((cs.w + 63) / 64), (unsigned)((cs.ci + 31) / 32), (unsigned)(cs.n * cs.h)), 256, 0, st>>>(
            in, xh, xl, cs.ci, cs.h, cs.w, raw ? 0 : 1);
        lcu_note_launch();
    }
    if (w_hi && (w_lo || passes == 1)) {
        wh = const_cast<float*>(w_hi);
        wl = const_cast<float*>(w_lo);
    } else {
        k_weight_khwc_split<<<lcu_blocks(we, 256), 256, 0, st>>>(w, wh, wl, cs.co, cs.ci, cs.kh, cs.kw);
        lcu_note_launch();
    }
    lancius_error e = lcu_launch_status();
    if (e != LANCIUS_ERROR_OK) return e;

    EncodeTiledFn fn = encode_fn();
    if (!fn || !configure()) { lancius_set_error(LANCIUS_ERROR_INTERNAL); return LANCIUS_ERROR_INTERNAL; }
    const int rows = pick_rows(cs.wo, cs.ho, cs.stride);
    CUtensorMap mw_hi, mw_lo, mx_hi, mx_lo;
    bool ok = true;
    {   // weights: [1][Co][K] rows of K floats, box {16, 256} (128 rows for the persistent kernel)
        cuuint64_t dims[3] = {K, (cuuint64_t)cs.co, 1};
        cuuint64_t strides[2] = {K * 4, we * 4};
        cuuint32_t box[3] = {BK, pt ? (cuuint32_t)PT_BM : (cuuint32_t)BM, 1}, es[3] = {1, 1, 1};
        ok = ok && fn(&mw_hi, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, wh, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                      CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
        if (passes > 1)
            ok = ok && fn(&mw_lo, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, wl, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                          CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
        else mw_lo = mw_hi;
    }
    {   // input NHWC: dims {C, W, H, N}; box {16 channels, Wo x rows pixels at the conv stride, 1 image}
        cuuint64_t dims[4] = {(cuuint64_t)cs.ci, (cuuint64_t)cs.w, (cuuint64_t)cs.h, (cuuint64_t)cs.n};
        cuuint64_t strides[3] = {(cuuint64_t)cs.ci * 4, (cuuint64_t)cs.w * cs.ci * 4, (cuuint64_t)cs.h * cs.w * cs.ci * 4};
        cuuint32_t box[4] = {BK, (cuuint32_t)(cs.wo * cs.stride), (cuuint32_t)(rows * cs.stride), 1};
        cuuint32_t es[4] = {1, (cuuint32_t)cs.stride, (cuuint32_t)cs.stride, 1};
        ok = ok && fn(&mx_hi, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, xh, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                      CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
        if (xl)
            ok = ok && fn(&mx_lo, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, xl, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                          CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
        else mx_lo = mx_hi;
    }
    if (!ok) { lancius_set_error(LANCIUS_ERROR_INTERNAL); return LANCIUS_ERROR_INTERNAL; }
    // NHWC output by TMA stores of 32 x 32 blocks (LCU_CONV_NO_TMA_OUT=1: plain stores)
    CUtensorMap mo_hi, mo_lo;
    int tma_out = 0;
    if (out_nhwc) {
        const char* env = getenv("LCU_CONV_NO_TMA_OUT");
        tma_out = !(env && env[0] == '1') && cs.co % 4 == 0 && !(reinterpret_cast<uintptr_t>(out) & 15) &&
                  !(reinterpret_cast<uintptr_t>(out_lo) & 15);
        if (tma_out) {
            cuuint64_t dims[3] = {(cuuint64_t)cs.co, (cuuint64_t)cs.ho * cs.wo, (cuuint64_t)cs.n};
            cuuint64_t strides[2] = {(cuuint64_t)cs.co * 4, (cuuint64_t)cs.ho * cs.wo * cs.co * 4};
            cuuint32_t box[3] = {32, 32, 1}, es[3] = {1, 1, 1};
            tma_out = fn(&mo_hi, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, out, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
            if (tma_out && out_lo)
                tma_out = fn(&mo_lo, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, out_lo, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                             CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
        }
    }
    if (!tma_out) mo_hi = mw_hi;
    if (!tma_out || !out_lo) mo_lo = mo_hi;
    ConvArgs a{cs.n, cs.ci, cs.co, cs.kh, cs.kw, cs.stride, cs.pad, cs.ho, cs.wo, rows, cs.co > 128 ? 2 : 1, passes, relu, raw,
               out_nhwc, tma_out, out_nhwc ? out_lo : nullptr, nullptr};
    if (pt && !out_nhwc && gap) {
        a.gap = gap;
        if (gap_written) *gap_written = 1;
    }
    if (pt) {
        const long long T = (long long)cs.n * ((cs.ho + rows - 1) / rows) * ((cs.co + PT_BM - 1) / PT_BM);
        k_conv_pt<<<(unsigned)std::min<long long>(T, n_sm), PT_THREADS, PT_SMEM_BYTES, st>>>(mw_hi, mw_lo, mx_hi, mx_lo, out, a, mo_hi, mo_lo);
        lcu_note_launch();
        return lcu_launch_status();
    }
    dim3 grid((unsigned)(cs.n * ((cs.ho + rows - 1) / rows)), (unsigned)((cs.co + BM - 1) / BM));
    k_conv_tc<<<grid, THREADS, SMEM_BYTES, st>>>(mw_hi, mw_lo, mx_hi, mx_lo, out, a);
    lcu_note_launch();
    return lcu_launch_status();
}

// ---------------------------------------------------------------------------------
// Short-reduction conv (K = Ci*Kh*Kw <= 32, e.g. the 3-channel stem) on the tensor cores,
// writing NHWC FP32 plus its tf32_lo copy for a tensor-core conv that reads it next.
//   D[px][co] = A[px][k] . B[co][k]^T, 128 output pixels per tile (MMA M), K padded to 32
//   (one 128-byte swizzle row per pixel), FP32-exact as A_hi*[B_hi|B_lo] (N = 2 Co) +
//   A_lo*B_hi (N = Co): the left Co accumulator columns hold hi*hi + lo*hi, the right
//   hi*lo.
//   warps 0-3, 10-13  builders, two groups taking even and odd tiles (A buffer 0 and 1), so
//              two tiles' gathers are in flight: one pixel per thread; gather its Ci*Kh*Kw
//              inputs (zero padding) and write them as TF32 hi/lo rows of its A buffer
//   warps 4-7  epilogue: TMEM -> sum of both halves -> ReLU -> hi and tf32_lo, staged as
//              128-byte swizzled 32-channel blocks for the TMA store
//   warp 8     TMEM allocation + MMA issue (one lane)
//   warp 9     TMA store of the staged tile (one lane)
// Per tile the tensor work is 8 MMAs; the kernel is bound by the output stores (2 x 4 Co
// bytes per pixel), which the copy engine performs off the threads' path.
namespace {
constexpr int C1_BM = 128, C1_KP = 32, C1_THREADS = 448;
constexpr int C1_A = C1_BM * C1_KP * 4;            // 16 KB: one of A hi / A lo
constexpr int C1_B = 256 * C1_KP * 4;              // B hi rows then B lo rows (2 Co <= 256)
constexpr int C1_STG = 128 * 128;                  // one 32-channel block of 128 pixels
constexpr int C1_SMEM_BYTES = 2 * 2 * C1_A + C1_B + 8 * C1_STG + 1024 + 1024;   // staging: 2 x 64 KB or 1 x 128 KB

struct SmemC1 {
    uint64_t a_full[2], a_empty[2], acc_full[2], acc_empty[2], stg_full[2], stg_free[2], drain;
    uint32_t tmem;
    int abort;
};

__device__ __forceinline__ uint32_t c1_swz(int row, int chunk) { return (uint32_t)(row * 128 + ((chunk ^ (row & 7)) << 4)); }

template <int CI, int KH, int KW>
__global__ void __launch_bounds__(C1_THREADS, 1)
k_conv_small_tc(const __grid_constant__ CUtensorMap m_hi, const __grid_constant__ CUtensorMap m_lo,
                const float* __restrict__ in, const float* __restrict__ w, int N, int H, int W, int Co, int stride,
                int pad, int Ho, int Wo, int relu, int exact, int with_lo, uint32_t tmem_cols) {
    constexpr int K = CI * KH * KW;
    static_assert(K <= C1_KP, "reduction fits one 128-byte row");
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* abuf = base;                            // [2][hi | lo]
    uint8_t* bsm = base + 4 * C1_A;                  // [2 Co rows][128 B]
    uint8_t* stg0 = bsm + C1_B;                      // nstg x [hi | lo][Co / 32 blocks][128 px][128 B]
    SmemC1* sm = reinterpret_cast<SmemC1*>(stg0 + 8 * C1_STG);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const long long P = (long long)N * Ho * Wo;
    const int T = (int)((P + C1_BM - 1) / C1_BM);
    const int nblk = Co / 32;
    // two staging buffers when they fit (Co <= 64): the epilogue of tile j fills one while
    // the copy engine drains tile j-1's from the other
    const int nstg = Co <= 64 ? 2 : 1;
    const int stg_bytes = 2 * nblk * C1_STG;
    volatile int* abort = &sm->abort;

    if (threadIdx.x == 0) {
        for (int b = 0; b < 2; b++) {
            tc::mbar_init(&sm->a_full[b], 128); tc::mbar_init(&sm->a_empty[b], 1);
            tc::mbar_init(&sm->acc_full[b], 1); tc::mbar_init(&sm->acc_empty[b], 128);
        }
        for (int b = 0; b < 2; b++) { tc::mbar_init(&sm->stg_full[b], 128); tc::mbar_init(&sm->stg_free[b], 1); }
        tc::mbar_init(&sm->drain, 1);
        sm->abort = 0;
        tc::fence_barrier_init();
        tc::prefetch_tmap(&m_hi);
        if (with_lo) tc::prefetch_tmap(&m_lo);
    }
    // weights -> B rows: hi (the value; the MMA reads its TF32 bits) for co, lo for Co + co
    for (int i = threadIdx.x; i < Co * C1_KP; i += C1_THREADS) {
        const int co = i / C1_KP, k = i - co * C1_KP;
        const float x = k < K ? w[(size_t)co * K + k] : 0.f;
        reinterpret_cast<float*>(bsm + c1_swz(co, k >> 2))[k & 3] = x;
        reinterpret_cast<float*>(bsm + c1_swz(Co + co, k >> 2))[k & 3] = tc::tf32_lo(x);
    }
    tc::fence_proxy_async();
    if (warp == 8) tc::tmem_alloc(&sm->tmem, tmem_cols);
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = sm->tmem;

    if (warp < 4 || warp >= 10) {
        // ---------------- builders ----------------
        const int g = warp >= 10 ? 1 : 0;            // tiles j with j % 2 == g, A buffer g
        const int r = threadIdx.x - 320 * g;         // pixel row of the tile
        int j = g;
        for (int t = blockIdx.x + g * gridDim.x; t < T; t += 2 * gridDim.x, j += 2) {
            const int b = g;
            if (j >= 2 && !tc::mbar_wait(&sm->a_empty[b], ((j >> 1) - 1) & 1, abort, &g_conv_watchdog, 41)) break;
            const long long p = (long long)t * C1_BM + r;
            float v[C1_KP];
#pragma unroll
            for (int k = 0; k < C1_KP; k++) v[k] = 0.f;
            if (p < P) {
                const int n = (int)(p / ((long long)Ho * Wo));
                const int rem = (int)(p - (long long)n * Ho * Wo), ho = rem / Wo, wo = rem - ho * Wo;
                const int y0 = ho * stride - pad, x0 = wo * stride - pad;
                const float* src = in + (size_t)n * CI * H * W;
#pragma unroll
                for (int ci = 0; ci < CI; ci++)
#pragma unroll
                    for (int kh = 0; kh < KH; kh++)
#pragma unroll
                        for (int kw = 0; kw < KW; kw++) {
                            const int iy = y0 + kh, ix = x0 + kw;
                            if (iy >= 0 && iy < H && ix >= 0 && ix < W)
                                v[(ci * KH + kh) * KW + kw] = __ldg(src + ((size_t)ci * H + iy) * W + ix);
                        }
            }
            uint8_t* ah = abuf + b * 2 * C1_A;
#pragma unroll
            for (int c = 0; c < C1_KP / 4; c++) {
                const float4 x = make_float4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
                *reinterpret_cast<float4*>(ah + c1_swz(r, c)) = x;
                *reinterpret_cast<float4*>(ah + C1_A + c1_swz(r, c)) = tc::tf32_lo4(x);
            }
            tc::fence_proxy_async();
            tc::mbar_arrive(&sm->a_full[b]);
        }
    } else if (warp < 8) {
        // ---------------- epilogue ----------------
        const int q = warp & 3, row = 32 * q + lane;
        int j = 0;
        for (int t = blockIdx.x; t < T; t += gridDim.x, j++) {
            const int b = j & 1;
            const int sb = j % nstg, su = j / nstg;
            if (!tc::mbar_wait(&sm->acc_full[b], (j >> 1) & 1, abort, &g_conv_watchdog, 42)) break;
            if (j >= nstg && !tc::mbar_wait(&sm->stg_free[sb], (su - 1) & 1, abort, &g_conv_watchdog, 43)) break;
            tc::tc_fence_after();
            uint8_t* stg = stg0 + sb * stg_bytes;
            const uint32_t d = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)b * 2 * Co;
            for (int blk = 0; blk < nblk; blk++) {
                float x[32], x2[32];
                tc::tmem_ld32(d + blk * 32, x);
                if (exact) tc::tmem_ld32(d + Co + blk * 32, x2);
                else {
#pragma unroll
                    for (int c = 0; c < 32; c++) x2[c] = 0.f;
                }
                uint8_t* sh = stg + blk * C1_STG;
                uint8_t* sl = stg + (nblk + blk) * C1_STG;
#pragma unroll
                for (int c = 0; c < 8; c++) {
                    float4 y = make_float4(x[4 * c] + x2[4 * c], x[4 * c + 1] + x2[4 * c + 1], x[4 * c + 2] + x2[4 * c + 2],
                                           x[4 * c + 3] + x2[4 * c + 3]);
                    if (relu) { y.x = fmaxf(y.x, 0.f); y.y = fmaxf(y.y, 0.f); y.z = fmaxf(y.z, 0.f); y.w = fmaxf(y.w, 0.f); }
                    *reinterpret_cast<float4*>(sh + c1_swz(row, c)) = y;
                    if (with_lo) *reinterpret_cast<float4*>(sl + c1_swz(row, c)) = tc::tf32_lo4(y);
                }
            }
            tc::tc_fence_before();
            tc::mbar_arrive(&sm->acc_empty[b]);
            tc::fence_proxy_async();
            tc::mbar_arrive(&sm->stg_full[sb]);
        }
    } else if (warp == 8) {
        // ---------------- MMA issue ----------------
        if (lane == 0) {
            const uint32_t id_2 = tc::idesc_tf32(C1_BM, 2 * Co, false, false);
            const uint32_t id_1 = tc::idesc_tf32(C1_BM, Co, false, false);
            const uint32_t bb = tc::smem_u32(bsm);
            int j = 0;
            for (int t = blockIdx.x; t < T; t += gridDim.x, j++) {
                const int b = j & 1;
                if (!tc::mbar_wait(&sm->a_full[b], (j >> 1) & 1, abort, &g_conv_watchdog, 44)) break;
                if (j >= 2 && !tc::mbar_wait(&sm->acc_empty[b], ((j >> 1) - 1) & 1, abort, &g_conv_watchdog, 45)) break;
                tc::tc_fence_after();
                const uint32_t ah = tc::smem_u32(abuf + b * 2 * C1_A), d = tmem + (uint32_t)b * 2 * Co;
#pragma unroll
                for (int kb = 0; kb < C1_KP / 8; kb++) {
                    const uint64_t db = tc::smem_desc(bb + kb * 32, 16, 1024, tc::SWZ_128B);
                    const uint64_t da = tc::smem_desc(ah + kb * 32, 16, 1024, tc::SWZ_128B);
                    if (exact) {
                        tc::mma_tf32(d, da, db, id_2, kb ? 1u : 0u);                      // hi x [hi | lo]
                        tc::mma_tf32(d, tc::smem_desc(ah + C1_A + kb * 32, 16, 1024, tc::SWZ_128B), db, id_1, 1u);   // lo x hi
                    } else {
                        tc::mma_tf32(d, da, db, id_1, kb ? 1u : 0u);
                    }
                }
                tc::mma_commit(&sm->a_empty[b]);
                tc::mma_commit(&sm->acc_full[b]);
            }
        }
    } else if (warp == 9) {
        // ---------------- TMA store ----------------
        if (lane == 0) {
            int j = 0;
            for (int t = blockIdx.x; t < T; t += gridDim.x, j++) {
                const int sb = j % nstg;
                if (!tc::mbar_wait(&sm->stg_full[sb], (j / nstg) & 1, abort, &g_conv_watchdog, 46)) break;
                const uint8_t* stg = stg0 + sb * stg_bytes;
                for (int blk = 0; blk < nblk; blk++) {
                    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];"
                                 ::"l"(reinterpret_cast<uint64_t>(&m_hi)), "r"(tc::smem_u32(stg + blk * C1_STG)),
                                   "r"(32 * blk), "r"(t * C1_BM) : "memory");
                    if (with_lo)
                        asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];"
                                     ::"l"(reinterpret_cast<uint64_t>(&m_lo)), "r"(tc::smem_u32(stg + (nblk + blk) * C1_STG)),
                                       "r"(32 * blk), "r"(t * C1_BM) : "memory");
                }
                asm volatile("cp.async.bulk.commit_group;" ::: "memory");
                if (nstg == 2) {   // the previous tile's buffer is free once its copies read it
                    asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
                    if (j >= 1) tc::mbar_arrive(&sm->stg_free[(j - 1) & 1]);
                } else {
                    asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
                    tc::mbar_arrive(&sm->stg_free[0]);
                }
            }
            asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
        }
    }

    tc::tc_fence_before();
    __syncthreads();
    if (sm->abort && warp == 8 && lane == 0) {   // let issued MMAs retire before TMEM is released
        int never = 0;
        tc::mma_commit(&sm->drain);
        tc::mbar_wait(&sm->drain, 0, &never, nullptr, 0);
    }
    __syncthreads();
    if (warp == 8) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem, tmem_cols);
    }
}

bool make_nhwc_out_map(CUtensorMap* m, float* out, long long P, int Co) {
    EncodeTiledFn fn = encode_fn();
    if (!fn || (reinterpret_cast<uintptr_t>(out) & 15)) return false;
    cuuint64_t dims[2] = {(cuuint64_t)Co, (cuuint64_t)P};
    cuuint64_t strides[1] = {(cuuint64_t)Co * 4};
    cuuint32_t box[2] = {32, C1_BM}, es[2] = {1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, out, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
              CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}
}  // namespace

// The stem geometries instantiated above; Co a multiple of 32 up to 128.
extern "C" int lcu_conv_small_tc_ok(size_t N, size_t Ci, size_t H, size_t W, size_t Co, size_t Kh, size_t Kw,
                                    size_t stride, size_t pad) {
    const char* e = getenv("LCU_CONV_SMALL_SIMT");
    if (e && e[0] == '1') return 0;
    const bool geo = (Ci == 3 && Kh == 3 && Kw == 3) || (Ci == 1 && Kh == 3 && Kw == 3) || (Ci == 3 && Kh == 1 && Kw == 1);
    if (!geo || Co % 32 || Co == 0 || Co > 128 || stride < 1 || H + 2 * pad < Kh || W + 2 * pad < Kw) return 0;
    const size_t Ho = (H + 2 * pad - Kh) / stride + 1, Wo = (W + 2 * pad - Kw) / stride + 1;
    return N * Ho * Wo < (1ull << 31) && N * Ci * H * W < (1ull << 31);
}

// out (and out_lo, when given) NHWC [N][Ho][Wo][Co]; in NCHW; w [Co][Ci][Kh][Kw].
// mode LCU_MODE_TF32: one pass; otherwise 3xTF32 (FP32-exact).
extern "C" lancius_error lcu_conv2d_small_tc_nhwc(float* out, float* out_lo, const float* in, const float* w, size_t N,
                                                  size_t Ci, size_t H, size_t W, size_t Co, size_t Kh, size_t Kw,
                                                  size_t stride, size_t pad, int relu, int mode, void* stream) {
    if (!lcu_conv_small_tc_ok(N, Ci, H, W, Co, Kh, Kw, stride, pad)) {
        lancius_set_error(LANCIUS_ERROR_UNSUPPORTED_OP);
        return LANCIUS_ERROR_UNSUPPORTED_OP;
    }
    const int Ho = (int)((H + 2 * pad - Kh) / stride + 1), Wo = (int)((W + 2 * pad - Kw) / stride + 1);
    const long long P = (long long)N * Ho * Wo;
    if (P == 0) return LANCIUS_ERROR_OK;
    CUtensorMap mh, ml;
    if (!make_nhwc_out_map(&mh, out, P, (int)Co) || (out_lo && !make_nhwc_out_map(&ml, out_lo, P, (int)Co))) {
        lancius_set_error(LANCIUS_ERROR_INTERNAL);
        return LANCIUS_ERROR_INTERNAL;
    }
    if (!out_lo) ml = mh;
    static int n_sm = 0;
    if (!n_sm) { int dev = 0; cudaGetDevice(&dev); cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev); }
    const long long T = (P + C1_BM - 1) / C1_BM;
    const unsigned grid = (unsigned)std::min<long long>(T, n_sm > 0 ? n_sm : LCU_SMS);
    uint32_t cols = 32;
    while (cols < 4 * Co) cols <<= 1;
    const int exact = mode == LCU_MODE_TF32 ? 0 : 1;
    cudaStream_t st = lcu_as_stream(stream);
#define LCU_C1(ci, kh, kw)                                                                                          \
    if (Ci == ci && Kh == kh && Kw == kw) {                                                                         \
        static bool conf[64] = {};                                                                                  \
        int dev = 0;                                                                                                \
        cudaGetDevice(&dev);                                                                                        \
        if (dev >= 0 && dev < 64 && !conf[dev]) {                                                                   \
            if (cudaFuncSetAttribute(k_conv_small_tc<ci, kh, kw>, cudaFuncAttributeMaxDynamicSharedMemorySize,      \
                                     C1_SMEM_BYTES) != cudaSuccess)                                                 \
                return lcu_launch_status();                                                                         \
            conf[dev] = true;                                                                                       \
        }                                                                                                           \
        k_conv_small_tc<ci, kh, kw><<<grid, C1_THREADS, C1_SMEM_BYTES, st>>>(                                       \
            mh, ml, in, w, (int)N, (int)H, (int)W, (int)Co, (int)stride, (int)pad, Ho, Wo, relu, exact,             \
            out_lo ? 1 : 0, cols);                                                                                  \
        lcu_note_launch();                                                                                          \
        return lcu_launch_status();                                                                                 \
    }
    LCU_C1(3, 3, 3) LCU_C1(1, 3, 3) LCU_C1(3, 1, 1)
#undef LCU_C1
    lancius_set_error(LANCIUS_ERROR_UNSUPPORTED_OP);
    return LANCIUS_ERROR_UNSUPPORTED_OP;
}

extern "C" int lcu_conv_watchdog_read_and_clear(void) {
    int v = 0, z = 0;
    cudaMemcpyFromSymbol(&v, g_conv_watchdog, sizeof(int));
    if (v) cudaMemcpyToSymbol(g_conv_watchdog, &z, sizeof(int));
    return v;
}

// Device address of this file's watchdog word on the current device (0 if unavailable).
extern "C" int* lcu_conv_watchdog_addr(void) {
    void* p = nullptr;
    return cudaGetSymbolAddress(&p, g_conv_watchdog) == cudaSuccess ? static_cast<int*>(p) : nullptr;
}
