// FP32 GEMM on the 5th-generation tensor cores (tcgen05, kind::tf32) with the
// 3xTF32 split for FP32-exact results:
//     A*B ~= Ahi*Bhi + Ahi*Blo + Alo*Bhi,   hi = x truncated to TF32, lo = rna_tf32(x - hi),
// accumulated in FP32 in TMEM. A split pass writes hi/lo copies of both operands
// into scratch with 16-byte-aligned row pitches (any M, N, K is then TMA-legal);
// the GEMM kernel streams them with TMA through a 4-stage mbarrier ring:
//
//   warp 0      TMA producer (one elected lane)
//   warp 1      TMEM allocation + tcgen05.mma issue for rows 0-127 (one lane)
//   warp 10     tcgen05.mma issue for rows 128-255 (one lane): one thread's MMAs complete
//               one after another; two issuing threads overlap on the tensor pipe
//   warps 2-9   epilogue: tcgen05.ld -> +bias -> ReLU/GELU -> +residual -> global
//               (two warps per TMEM lane quadrant; in raw-A mode they also split A)
//
// Tile 128 x 256 x 16: A K-major in 64-byte swizzle, B N-major in the 128-byte
// swizzle with 32-byte atoms (the only N-major layout tcgen05 accepts for TF32;
// eight 32-column chunks), accumulator 128 lanes x 256 TMEM columns.
// Every mbarrier wait is bounded (tc::kSpinLimit); a timeout sets the watchdog
// word, unwinds the CTA and frees its TMEM.
#include "tc_common.cuh"
#include <cuda_bf16.h>
#include <cstdio>
#ifndef LCU_GEMM_DEBUG
#define LCU_GEMM_DEBUG 0
#endif
#include <algorithm>
#include <mutex>
#include <vector>

namespace {

constexpr int BM = 256, BN = 256, BK = 16, STAGES = 3;
constexpr int EPI_WARPS = 8;                         // two per TMEM lane quadrant
constexpr int THREADS = 64 + 32 * EPI_WARPS + 32;     // + the second MMA issuer (warp 10)
constexpr int MMA_WARP2 = 2 + EPI_WARPS;
constexpr int A_TILE = BM * BK * 4;                  // 16 KB (two 128-row halves)
constexpr int B_CHUNK = BK * 32 * 4;                 // 2 KB: 16 k-rows x 32 n
constexpr uint32_t TMEM_COLS = 512;   // two 128x256 FP32 accumulators (rows 0-127, 128-255) at columns 0 and 256

__device__ int g_gemm_watchdog = 0;

// Optional per-CTA phase timestamps (%globaltimer) for tuning; compiled out unless built
// with -DLCU_GEMM_TRACE=1 (then lcu_gemm_trace_dump copies them out).
#ifndef LCU_GEMM_TRACE
#define LCU_GEMM_TRACE 0
#endif
#if LCU_GEMM_TRACE
__device__ unsigned long long g_gtrace[2048][8];
__device__ __forceinline__ unsigned long long gtime() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
#define GTRACE(slot) do { unsigned cta_ = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z); \
    if (cta_ < 2048) g_gtrace[cta_][slot] = gtime(); } while (0)
#else
#define GTRACE(slot) do {} while (0)
#endif

struct Smem {
    uint64_t full[STAGES];
    uint64_t empty[STAGES];
    uint64_t conv[STAGES];     // raw-A mode: the stage's A tile has been split in place
    uint64_t accum;
    uint64_t drain, drain2;
    uint32_t tmem_base;
    int abort;
    int consumed;
};

// Dynamic shared memory of a launch with TBN-column tiles.
constexpr int smem_bytes(int tbn) { return STAGES * (2 * A_TILE + 2 * tbn * BK * 4) + 1024 + 256 + tbn * 4; }

// DST: the epilogue stores into LcuColDest's destinations. TBN: tile columns, 256 or 192
// (192 for products whose 256-wide tiles would leave SMs idle in the last round, e.g.
// 8192 x 768: 96 tiles of 256 x 256 against 128 of 256 x 192 on 148 SMs; N = 192 MMAs run
// at ~3/4 of the time of N = 256 ones).
template <bool DST, int TBN>
__global__ void __launch_bounds__(THREADS, 1)
k_gemm_tc(const __grid_constant__ CUtensorMap ta_hi, const __grid_constant__ CUtensorMap ta_lo,
          const __grid_constant__ CUtensorMap tb_hi, const __grid_constant__ CUtensorMap tb_lo,
          const LcuGemmGroup* __restrict__ groups, int M, int N, int K, int epi, int passes,
          int splits, int kchunk, float* __restrict__ partial, int conv_hw, LcuColDest dst,
          const CUtensorMap* __restrict__ a_maps) {
    constexpr int BN = TBN, B_TILE = BN * BK * 4, STAGE_BYTES = 2 * A_TILE + 2 * B_TILE;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* tiles = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    Smem* sm = reinterpret_cast<Smem*>(tiles + STAGES * STAGE_BYTES);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // blockIdx.z = group * splits + split; a split covers k in [k_begin, k_begin + kchunk)
    const int g = blockIdx.z / splits, split = blockIdx.z % splits;
    const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
    const int k_begin = split * kchunk;
    const int k_end = min(K, k_begin + kchunk);
    // passes == 0: BF16 operands (kind::f16, K = 16 per MMA): a stage holds 32 k of them in
    // the same 64-byte rows that hold 16 k of TF32
    const bool bf = passes == 0;
    const int KSTEP = bf ? 2 * BK : BK;
    const int KT = (k_end - k_begin + KSTEP - 1) / KSTEP;
    volatile int* abort = &sm->abort;
    if (threadIdx.x == 0) GTRACE(0);

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) {
            tc::mbar_init(&sm->full[s], 1); tc::mbar_init(&sm->empty[s], 2); tc::mbar_init(&sm->conv[s], EPI_WARPS);
        }
        tc::mbar_init(&sm->accum, 2);
        tc::mbar_init(&sm->drain, 1);
        tc::mbar_init(&sm->drain2, 1);
        sm->abort = 0;
        sm->consumed = 0;
        tc::fence_barrier_init();
        if (a_maps) { tc::tmap_acquire(a_maps + groups[g].aidx); tc::prefetch_tmap(a_maps + groups[g].aidx); }
        else { tc::prefetch_tmap(&ta_hi); if (passes > 1) tc::prefetch_tmap(&ta_lo); }
        tc::prefetch_tmap(&tb_hi);
        if (passes > 1) tc::prefetch_tmap(&tb_lo);
    }
    if (warp == 1) tc::tmem_alloc(&sm->tmem_base, TMEM_COLS);
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = sm->tmem_base;
    int issued = 0;

    if (warp == 0 && lane == 0) {
        // ---------------- TMA producer ----------------
        // raw-A mode: only the FP32 A tile arrives; the epilogue warps split it into hi/lo in place
        const uint32_t tx = a_maps ? (passes > 1 ? A_TILE + 2 * B_TILE : A_TILE + B_TILE)
                                   : (passes > 1 ? STAGE_BYTES : A_TILE + B_TILE);   // BF16: A_TILE + B_TILE too
        const int ga = groups[g].aidx, gb = groups[g].bidx;      // scratch slots of this group's operands
        const CUtensorMap* ma = a_maps ? a_maps + ga : &ta_hi;
        for (int kt = 0; kt < KT; kt++) {
            int s = kt % STAGES;
            if (kt >= STAGES && !tc::mbar_wait(&sm->empty[s], ((kt / STAGES) - 1) & 1, abort, &g_gemm_watchdog, 1)) break;
            uint8_t* st = tiles + s * STAGE_BYTES;
            tc::mbar_expect_tx(&sm->full[s], tx);
            int k0 = k_begin + kt * KSTEP;
            tc::tma_load_3d(st, ma, &sm->full[s], k0, m0, a_maps ? 0 : ga);               // A: two 128-row boxes
            tc::tma_load_3d(st + A_TILE / 2, ma, &sm->full[s], k0, m0 + 128, a_maps ? 0 : ga);
            if (bf)   // B^T, K-major like A: one box of 256 rows of 32 k
                tc::tma_load_3d(st + 2 * A_TILE, &tb_hi, &sm->full[s], k0, n0, gb);
            else
                for (int j = 0; j < BN / 32; j++)
                    tc::tma_load_3d(st + 2 * A_TILE + j * B_CHUNK, &tb_hi, &sm->full[s], n0 + 32 * j, k0, gb);
            if (passes > 1) {
                if (!a_maps) {
                    tc::tma_load_3d(st + A_TILE, &ta_lo, &sm->full[s], k0, m0, ga);
                    tc::tma_load_3d(st + A_TILE + A_TILE / 2, &ta_lo, &sm->full[s], k0, m0 + 128, ga);
                }
                for (int j = 0; j < BN / 32; j++)
                    tc::tma_load_3d(st + 2 * A_TILE + B_TILE + j * B_CHUNK, &tb_lo, &sm->full[s], n0 + 32 * j, k0, gb);
            }
            issued = kt + 1;
        }
    } else if ((warp == 1 || warp == MMA_WARP2) && lane == 0) {
        // ---------------- MMA issuers: warp 1 rows 0-127, warp 10 rows 128-255 ----------------
        constexpr uint32_t idesc = tc::idesc_tf32(128, BN, false, true);
        const int half = warp == 1 ? 0 : 1;
        bool ok = true;
        for (int kt = 0; kt < KT && ok; kt++) {
            int s = kt % STAGES;
            if (!tc::mbar_wait(a_maps ? &sm->conv[s] : &sm->full[s], (kt / STAGES) & 1, abort, &g_gemm_watchdog, 2)) {
                ok = false; break;
            }
            if (kt == 0) GTRACE(1);
            tc::tc_fence_after();
            if (LCU_GEMM_DEBUG && blockIdx.x == 0 && blockIdx.y == 0 && kt == 0) {
                const float* fa = reinterpret_cast<const float*>(tiles + s * STAGE_BYTES);
                const float* fb = reinterpret_cast<const float*>(tiles + s * STAGE_BYTES + 2 * A_TILE);
                printf("tmem=%08x A[0..7]=%g %g %g %g %g %g %g %g  A[16..19]=%g %g %g %g\n", tmem, fa[0], fa[1], fa[2], fa[3], fa[4], fa[5], fa[6], fa[7], fa[16], fa[17], fa[18], fa[19]);
                printf("B[0..7]=%g %g %g %g %g %g %g %g B[32..35]=%g %g %g %g B[512]=%g\n", fb[0], fb[1], fb[2], fb[3], fb[4], fb[5], fb[6], fb[7], fb[32], fb[33], fb[34], fb[35], fb[512]);
            }
            uint32_t st = tc::smem_u32(tiles + s * STAGE_BYTES);
            uint32_t a_hi = st, a_lo = st + A_TILE, b_hi = st + 2 * A_TILE, b_lo = st + 2 * A_TILE + B_TILE;
            if (bf) {
                constexpr uint32_t idb = tc::idesc_bf16(128, BN);
                const uint32_t hoff = (uint32_t)half * (128 * BK * 4), d = tmem + (uint32_t)half * 256;
#pragma unroll
                for (int kb = 0; kb < 2; kb++) {             // 16 k (32 bytes) per MMA
                    const uint64_t da = tc::smem_desc(a_hi + hoff + kb * 32, 16, 512, tc::SWZ_64B);
                    const uint64_t db = tc::smem_desc(b_hi + kb * 32, 16, 512, tc::SWZ_64B);
                    tc::mma_bf16(d, da, db, idb, (kt | kb) ? 1u : 0u);
                }
            }
#pragma unroll
            for (int kb = 0; kb < BK / 8 && !bf; kb++) {
                uint64_t dbh = tc::smem_desc(b_hi + kb * 1024, B_CHUNK, 512, tc::SWZ_128B_BASE32B);
                uint64_t dbl = tc::smem_desc(b_lo + kb * 1024, B_CHUNK, 512, tc::SWZ_128B_BASE32B);
                {                                            // rows 0-127 and 128-255 share the B tile
                    const uint32_t hoff = (uint32_t)half * (128 * BK * 4), d = tmem + (uint32_t)half * 256;
                    uint64_t dah = tc::smem_desc(a_hi + hoff + kb * 32, 16, 512, tc::SWZ_64B);
                    uint32_t acc = (kt | kb) ? 1u : 0u;
                    if (passes > 1) {
                        uint64_t dal = tc::smem_desc(a_lo + hoff + kb * 32, 16, 512, tc::SWZ_64B);
                        tc::mma_tf32(d, dal, dbh, idesc, acc);      // small terms first
                        tc::mma_tf32(d, dah, dbl, idesc, 1u);
                        tc::mma_tf32(d, dah, dbh, idesc, 1u);
                    } else {
                        tc::mma_tf32(d, dah, dbh, idesc, acc);
                    }
                }
            }
            tc::mma_commit(&sm->empty[s]);          // stage s is free once both issuers' MMAs retire
            if (half == 0) sm->consumed = kt + 1;
        }
        if (ok) tc::mma_commit(&sm->accum);
    } else if (warp >= 2 && warp < MMA_WARP2) {
        if (a_maps) {
            // ---------------- A splitter (raw-A mode) ----------------
            // The FP32 tile serves as hi as it is (the MMA reads it truncated to TF32);
            // lo = rna_tf32(x - tf32_hi(x)) goes to the stage's lo slot. The swizzle permutes
            // 16-byte chunks identically in both slots, so this is a flat elementwise pass.
            for (int kt = 0; kt < KT; kt++) {
                const int s = kt % STAGES;
                if (!tc::mbar_wait(&sm->full[s], (kt / STAGES) & 1, abort, &g_gemm_watchdog, 4)) break;
                float4* a4 = reinterpret_cast<float4*>(tiles + s * STAGE_BYTES);
                if (passes > 1) {
#pragma unroll 4
                    for (int i = threadIdx.x - 64; i < A_TILE / 16; i += 32 * EPI_WARPS)
                        a4[i + A_TILE / 16] = tc::tf32_lo4(a4[i]);
                }
                tc::fence_proxy_async();           // generic-proxy writes -> visible to the tensor core
                __syncwarp();
                if (lane == 0) tc::mbar_arrive(&sm->conv[s]);
            }
        }
        // ---------------- epilogue ----------------
        // Set-up that needs no accumulator runs while the last MMAs retire: the tile's bias
        // slice goes to shared memory and the first residual rows are put in flight.
        LcuGemmGroup gr = groups[g];
        if (splits > 1) {   // raw partial sums; the reduction applies the epilogue
            gr.c = partial + (size_t)blockIdx.z * M * N;
            gr.bias = nullptr; gr.resid = nullptr;
        }
        const int epi_here = splits > 1 ? LCU_EPI_NONE : epi;
        float* sbias = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(sm) + 256);
        for (int i = threadIdx.x - 64; i < BN; i += 32 * EPI_WARPS)
            sbias[i] = (gr.bias && n0 + i < N) ? __ldg(gr.bias + n0 + i) : 0.f;
        asm volatile("bar.sync 1, %0;" ::"n"(32 * EPI_WARPS) : "memory");      // the epilogue warps
        // Each warp owns 32 TMEM lanes (rows) and every other 32-column chunk of them (two
        // warps per lane quadrant). Per chunk it stages the 32x32 block in shared memory
        // (the drained pipeline buffers) and writes it back by rows: every store
        // instruction covers whole 128-byte row segments (coalesced). The warp's next
        // chunk's TMEM load and residual rows are in flight meanwhile.
        const int q = warp & 3;                    // TMEM lane quadrant of this warp
        constexpr int PARTS = EPI_WARPS / 4;       // warps sharing a quadrant
        const int part = (warp - 2) >> 2;
        // float4 path: every pointer 16-byte aligned and rows a multiple of 4 floats
        const bool v4 = N % 4 == 0 && !conv_hw && ((reinterpret_cast<uintptr_t>(gr.c) | reinterpret_cast<uintptr_t>(gr.resid) |
                                                    reinterpret_cast<uintptr_t>(gr.bias)) & 15) == 0 &&
                        (!DST || (dst.ldc % 4 == 0 && dst.col_off % 4 == 0));
        // residual rows of a chunk, 8 per lane (the float4 path's lane mapping)
        auto load_res = [&](int row0, int cc, float4 (&rv)[8]) {
            const int col = n0 + cc + 4 * (lane & 7);
#pragma unroll
            for (int it = 0; it < 8; it++) {
                const int row = row0 + 4 * it + (lane >> 3);
                rv[it] = (gr.resid && v4 && row < M && col < N)
                             ? *reinterpret_cast<const float4*>(gr.resid + (size_t)row * N + col)
                             : make_float4(0.f, 0.f, 0.f, 0.f);
            }
        };
        const int nh = m0 + 128 < M ? 2 : 1;                         // row halves present
        const int nc = (min(BN, N - n0) + 31) / 32;                   // 32-column chunks present
        float4 rv[8];
        if (part < nh * nc) load_res(m0 + (part / nc) * 128 + 32 * q, (part % nc) * 32, rv);
        if (threadIdx.x == 64) GTRACE(2);
        if (tc::mbar_wait(&sm->accum, 0, abort, &g_gemm_watchdog, 3)) {
            if (threadIdx.x == 64) GTRACE(3);
            tc::tc_fence_after();
            float* sb = reinterpret_cast<float*>(tiles) + (size_t)(warp - 2) * 32 * 36;
            auto taddr = [&](int i) {
                return tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)((i / nc) * 256 + (i % nc) * 32);
            };
            const int total = nh * nc;
            uint32_t va[32];
            if (part < total) tc::tmem_ld32_issue(taddr(part), va);
            for (int i = part; i < total; i += PARTS) {
                const int half = i / nc, c = (i % nc) * 32;
                const int row0 = m0 + half * 128 + 32 * q;
                tc::tmem_ld_wait(va);
#pragma unroll
                for (int j = 0; j < 32; j += 4)
                    *reinterpret_cast<float4*>(sb + lane * 36 + j) =
                        make_float4(__uint_as_float(va[j]), __uint_as_float(va[j + 1]), __uint_as_float(va[j + 2]),
                                    __uint_as_float(va[j + 3]));
                __syncwarp();
                float4 rn[8];
                const int nx = i + PARTS;
                if (nx < total) {
                    tc::tmem_ld32_issue(taddr(nx), va);
                    load_res(m0 + (nx / nc) * 128 + 32 * q, (nx % nc) * 32, rn);
                }
                if (v4) {
                    // 8 lanes per row, 4 columns each: 4 rows (128-byte segments) per step
                    const int cl = c + 4 * (lane & 7), col = n0 + cl;
                    if (col < N) {
                        const float4 bv = *reinterpret_cast<const float4*>(sbias + cl);
#pragma unroll
                        for (int it = 0; it < 8; it++) {
                            const int r = 4 * it + (lane >> 3), row = row0 + r;
                            if (row >= M) break;
                            float4 x = *reinterpret_cast<const float4*>(sb + r * 36 + 4 * (lane & 7));
                            x.x = lcu_apply_epi(x.x + bv.x, epi_here); x.y = lcu_apply_epi(x.y + bv.y, epi_here);
                            x.z = lcu_apply_epi(x.z + bv.z, epi_here); x.w = lcu_apply_epi(x.w + bv.w, epi_here);
                            x.x += rv[it].x; x.y += rv[it].y; x.z += rv[it].z; x.w += rv[it].w;   // zeros without a residual
                            if (DST && splits == 1) {
                                const size_t o = (size_t)row * dst.ldc + dst.col_off + col;
                                for (int k = 0; k < dst.n_dst; k++) *reinterpret_cast<float4*>(dst.ptr[k] + o) = x;
                            } else {
                                *reinterpret_cast<float4*>(gr.c + (size_t)row * N + col) = x;
                            }
                        }
                    }
                } else {
                    // any shape: lane j takes column j of each row (coalesced per row)
                    const int col = n0 + c + lane;
                    if (col < N) {
                        const float bv = sbias[c + lane];
#pragma unroll 4
                        for (int r = 0; r < 32; r++) {
                            const int row = row0 + r;
                            if (row >= M) break;
                            float x = lcu_apply_epi(sb[r * 36 + lane] + bv, epi_here);
                            if (conv_hw && splits == 1) {
                                // implicit-GEMM conv: row = output channel, column = n*HoWo + pixel -> NCHW
                                gr.c[(size_t)(col / conv_hw) * M * conv_hw + (size_t)row * conv_hw + col % conv_hw] = x;
                                continue;
                            }
                            if (gr.resid) x += gr.resid[(size_t)row * N + col];
                            if (DST && splits == 1) {   // fused all-gather: straight into every rank's C
                                const size_t o = (size_t)row * dst.ldc + dst.col_off + col;
                                for (int k = 0; k < dst.n_dst; k++) dst.ptr[k][o] = x;
                            } else {
                                gr.c[(size_t)row * N + col] = x;
                            }
                        }
                    }
                }
                __syncwarp();
                if (nx < total) {
#pragma unroll
                    for (int it = 0; it < 8; it++) rv[it] = rn[it];
                }
            }
            if (DST) __threadfence_system();   // peer stores complete before the kernel does
            if (threadIdx.x == 64) GTRACE(4);
        }
    }

    tc::tc_fence_before();
    __syncthreads();
    if (sm->abort) {
        // unwind: let in-flight TMA copies land and in-flight MMAs retire before the
        // CTA's shared memory and TMEM go away (both waits bounded as well)
        int never = 0;
        if (warp == 0 && lane == 0)
            for (int kt = sm->consumed; kt < issued; kt++)
                if (!tc::mbar_wait(&sm->full[kt % STAGES], (kt / STAGES) & 1, &never, nullptr, 0)) break;
        if ((warp == 1 || warp == MMA_WARP2) && lane == 0) {
            uint64_t* d = warp == 1 ? &sm->drain : &sm->drain2;
            tc::mma_commit(d);
            tc::mbar_wait(d, 0, &never, nullptr, 0);
        }
        __syncthreads();
    }
    if (warp == 1) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem, TMEM_COLS);
    }
    if (threadIdx.x == 0) GTRACE(5);
}




// hi/lo split of `count` row-major [rows, cols] operands into pitched scratch. Rows are
// walked by the grid and columns by the block: float4 in and out when cols % 4 == 0 and
// the source is 16-byte aligned (the pitch always is), no per-element division.
__device__ __forceinline__ void split_rows(const float* __restrict__ src, size_t rows, size_t cols, size_t pitch,
                                           float* __restrict__ hi, float* __restrict__ lo) {
    const bool v4 = cols % 4 == 0 && (reinterpret_cast<uintptr_t>(src) & 15) == 0;
    for (size_t r = blockIdx.x; r < rows; r += gridDim.x) {
        const float* s_row = src + r * cols;
        float* h_row = hi + r * pitch;
        float* l_row = lo ? lo + r * pitch : nullptr;
        if (v4) {
            for (size_t c = 4 * threadIdx.x; c < cols; c += 4 * blockDim.x) {
                const float4 x = __ldg(reinterpret_cast<const float4*>(s_row + c));
                *reinterpret_cast<float4*>(h_row + c) = make_float4(tc::tf32_hi(x.x), tc::tf32_hi(x.y), tc::tf32_hi(x.z),
                                                                    tc::tf32_hi(x.w));
                if (l_row) *reinterpret_cast<float4*>(l_row + c) = tc::tf32_lo4(x);
            }
        } else {
            for (size_t c = threadIdx.x; c < cols; c += blockDim.x) {
                const float x = s_row[c];
                h_row[c] = tc::tf32_hi(x);
                if (l_row) l_row[c] = tc::tf32_lo(x);
            }
        }
    }
}

__global__ void k_split(const LcuGemmGroup* __restrict__ groups, int which, size_t rows, size_t cols, size_t pitch,
                        float* __restrict__ hi, float* __restrict__ lo) {
    const LcuGemmGroup& gr = groups[blockIdx.y];
    if (which == 0 ? gr.adup : gr.bdup) return;          // an earlier group already split this operand
    const size_t base = (size_t)(which == 0 ? gr.aidx : gr.bidx) * rows * pitch;
    split_rows(which == 0 ? gr.a : gr.b, rows, cols, pitch, hi + base, lo ? lo + base : nullptr);
}

// BF16 (round to nearest even) copies of the GEMM operands: A row-major into [M][pitch],
// B [K][N] transposed into [N][pitch] (K-major, as the kernel reads both). Zero padding.
__global__ void k_to_bf16_a(const LcuGemmGroup* __restrict__ groups, size_t M, size_t K, size_t pitch,
                            __nv_bfloat16* __restrict__ dst) {
    const LcuGemmGroup& gr = groups[blockIdx.y];
    if (gr.adup) return;
    __nv_bfloat16* out = dst + (size_t)gr.aidx * M * pitch;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < M * pitch; i += (size_t)gridDim.x * blockDim.x) {
        const size_t r = i / pitch, c = i - r * pitch;
        out[i] = __float2bfloat16_rn(c < K ? gr.a[r * K + c] : 0.f);
    }
}
__global__ void k_to_bf16_bt(const LcuGemmGroup* __restrict__ groups, size_t K, size_t N, size_t pitch,
                             __nv_bfloat16* __restrict__ dst) {
    __shared__ float t[32][33];
    const LcuGemmGroup& gr = groups[blockIdx.z];
    if (gr.bdup) return;
    __nv_bfloat16* out = dst + (size_t)gr.bidx * N * pitch;
    const size_t k0 = (size_t)blockIdx.y * 32, n0 = (size_t)blockIdx.x * 32;
    for (int r = threadIdx.y; r < 32; r += blockDim.y) {
        const size_t k = k0 + r, n = n0 + threadIdx.x;
        t[r][threadIdx.x] = (k < K && n < N) ? gr.b[k * N + n] : 0.f;
    }
    __syncthreads();
    for (int r = threadIdx.y; r < 32; r += blockDim.y) {
        const size_t n = n0 + r, k = k0 + threadIdx.x;
        if (n < N && k < pitch) out[n * pitch + k] = __float2bfloat16_rn(t[threadIdx.x][r]);
    }
}

__global__ void k_split_one(const float* __restrict__ src, size_t rows, size_t cols, size_t pitch, float* __restrict__ hi,
                            float* __restrict__ lo) {
    split_rows(src, rows, cols, pitch, hi, lo);
}

// hi/lo im2col of an NCHW input into pitched [K = Ci*Kh*Kw][P = N*Ho*Wo] scratch
// (zero padding), the B operand of the implicit-GEMM conv; reads groups[0].b.
__global__ void k_im2col_split(const LcuGemmGroup* __restrict__ groups, LcuConvShape cs, size_t pitch,
                               float* __restrict__ hi, float* __restrict__ lo) {
    // grid.y = k (one im2col row), grid.x strides over the N*Ho*Wo columns (32-bit index math)
    const float* in = groups[0].b;
    const int k = blockIdx.y;
    const int kw = k % cs.kw, kh = (k / cs.kw) % cs.kh, ci = k / (cs.kw * cs.kh);
    const int hw = cs.ho * cs.wo, P = cs.n * hw;
    float* hrow = hi + (size_t)k * pitch;
    float* lrow = lo ? lo + (size_t)k * pitch : nullptr;
    for (int p = blockIdx.x * blockDim.x + threadIdx.x; p < P; p += gridDim.x * blockDim.x) {
        const int n = p / hw, r = p - n * hw;
        const int ho = r / cs.wo, wo = r - ho * cs.wo;
        const int ih = ho * cs.stride - cs.pad + kh, iw = wo * cs.stride - cs.pad + kw;
        float x = 0.f;
        if (ih >= 0 && iw >= 0 && ih < cs.h && iw < cs.w)
            x = __ldg(in + (((size_t)n * cs.ci + ci) * cs.h + ih) * (size_t)cs.w + iw);
        hrow[p] = tc::tf32_hi(x);
        if (lrow) lrow[p] = tc::tf32_lo(x);
    }
}

// out = act(sum over splits of the partials + bias) + resid, splits summed in order
__global__ void k_splitk_reduce(const LcuGemmGroup* __restrict__ groups, const float* __restrict__ partial, int splits,
                                size_t M, size_t N, int epi, size_t conv_hw, LcuColDest dst) {
    const LcuGemmGroup gr = groups[blockIdx.y];
    const float* p = partial + (size_t)blockIdx.y * splits * M * N;
    size_t n = M * N;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        float acc = 0.f;
        for (int s = 0; s < splits; s++) acc += p[(size_t)s * n + i];
        if (gr.bias) acc += __ldg(gr.bias + i % N);
        acc = lcu_apply_epi(acc, epi);
        if (gr.resid) acc += gr.resid[i];
        if (dst.n_dst > 0) {
            const size_t o = (i / N) * dst.ldc + dst.col_off + i % N;
            for (int q = 0; q < dst.n_dst; q++) dst.ptr[q][o] = acc;
        } else if (conv_hw) {
            size_t r = i / N, c = i % N;
            gr.c[(c / conv_hw) * M * conv_hw + r * conv_hw + c % conv_hw] = acc;
        } else {
            gr.c[i] = acc;
        }
    }
    if (dst.n_dst > 0) __threadfence_system();
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

// 3D map over [G][rows][pitch] floats, box {box_inner, box_rows, 1}
bool make_map(CUtensorMap* m, const float* base, size_t inner, size_t rows, size_t groups, size_t pitch,
              uint32_t box_inner, uint32_t box_rows, CUtensorMapSwizzle swz) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[3] = {inner, rows, groups};
    cuuint64_t strides[2] = {pitch * 4, rows * pitch * 4};
    cuuint32_t box[3] = {box_inner, box_rows, 1};
    cuuint32_t es[3] = {1, 1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(base), dims, strides, box, es,
              CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

size_t pad4(size_t v) { return (v + 3) & ~size_t(3); }

// 3D map over [G][rows][pitch] BF16, box {32 k (64 bytes), box_rows}, 64-byte swizzle (K-major)
bool make_map_bf16(CUtensorMap* m, const void* base, size_t inner, size_t rows, size_t groups, size_t pitch,
                   uint32_t box_rows) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[3] = {inner, rows, groups};
    cuuint64_t strides[2] = {pitch * 2, rows * pitch * 2};
    cuuint32_t box[3] = {32, box_rows, 1};
    cuuint32_t es[3] = {1, 1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, es,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}
size_t al256(size_t v) { return (v + 255) & ~size_t(255); }

}  // namespace

// ---------------------------------------------------------------------------
// Prepared launch: tensor maps over a scratch region, built once (the executor
// binds them at plan time; the per-op entry point builds them per call).

// K is cut into chunks of at most kMaxChunk: the tensor core's FP32 accumulation
// error grows with the reduction length, and per-chunk partials summed in FP32 keep
// the 3xTF32 result within 1e-4 at K = 16384 (measured normwise: 3e-5 at K = 4096,
// 6.3e-5 at 8192, 1.1e-4 at 16384 without the split, 3e-5 with 4096-chunks).
constexpr int kMaxChunk = 8192;
int split_count(size_t K) { return K > (size_t)kMaxChunk ? (int)((K + kMaxChunk - 1) / kMaxChunk) : 1; }

extern "C" size_t lcu_gemm_tc_scratch_bytes(size_t M, size_t N, size_t K, int G, int Ga, int Gb, int passes) {
    if (passes == 0) {   // BF16: A [Ga][M][pad8(K)] and B^T [Gb][N][pad8(K)]
        const size_t kp = (K + 7) & ~size_t(7);
        int sp = split_count(K);
        return al256((size_t)Ga * M * kp * 2) + al256((size_t)Gb * N * kp * 2) + (sp > 1 ? al256((size_t)G * sp * M * N * 4) : 0);
    }
    size_t a = al256((size_t)Ga * M * pad4(K) * 4), b = al256((size_t)Gb * K * pad4(N) * 4);
    int sp = split_count(K);
    size_t part = sp > 1 ? al256((size_t)G * sp * M * N * 4) : 0;
    return (passes > 1 ? 2 * (a + b) : a + b) + part;
}

extern "C" lancius_error lcu_gemm_tc_prepare(LcuTcGemmPlan* p, void* scratch, size_t M, size_t N, size_t K, int G,
                                             int Ga, int Gb, int passes) {
    p->M = M; p->N = N; p->K = K; p->Kp = pad4(K); p->Np = pad4(N); p->G = G; p->Ga = Ga; p->Gb = Gb; p->passes = passes;
    p->conv = LcuConvShape{};
    p->b_presplit = 0;
    p->d_amaps = nullptr;
    if (passes == 0) {   // BF16 operands, both K-major: A [Ga][M][Kp], B^T [Gb][N][Kp]
        p->Kp = (K + 7) & ~size_t(7);
        char* s = static_cast<char*>(scratch);
        p->s_ahi = (float*)s; s += al256((size_t)Ga * M * p->Kp * 2);
        p->s_bhi = (float*)s; s += al256((size_t)Gb * N * p->Kp * 2);
        p->s_alo = p->s_blo = nullptr;
        p->splits = split_count(K);
        p->kchunk = p->splits > 1 ? (int)(((K + p->splits - 1) / p->splits + 2 * BK - 1) / (2 * BK) * (2 * BK)) : (int)(K ? K : 1);
        p->partial = p->splits > 1 ? (float*)s : nullptr;
        bool ok = make_map_bf16(&p->a_hi, p->s_ahi, K, M, Ga, p->Kp, 128) && make_map_bf16(&p->b_hi, p->s_bhi, K, N, Gb, p->Kp, BN);
        if (!ok) { lancius_set_error(LANCIUS_ERROR_INTERNAL); return LANCIUS_ERROR_INTERNAL; }
        p->a_lo = p->a_hi; p->b_lo = p->b_hi;
        return LANCIUS_ERROR_OK;
    }
    size_t a = al256((size_t)Ga * M * p->Kp * 4), b = al256((size_t)Gb * K * p->Np * 4);
    char* s = static_cast<char*>(scratch);
    p->s_ahi = (float*)s; s += a;
    p->s_bhi = (float*)s; s += b;
    p->s_alo = passes > 1 ? (float*)s : nullptr; if (passes > 1) s += a;
    p->s_blo = passes > 1 ? (float*)s : nullptr; if (passes > 1) s += b;
    p->splits = split_count(K);
    p->kchunk = p->splits > 1 ? (int)(((K + p->splits - 1) / p->splits + BK - 1) / BK * BK) : (int)(K ? K : 1);
    p->partial = p->splits > 1 ? (float*)s : nullptr;
    bool ok = make_map(&p->a_hi, p->s_ahi, K, M, Ga, p->Kp, BK, 128, CU_TENSOR_MAP_SWIZZLE_64B) &&
              make_map(&p->b_hi, p->s_bhi, N, K, Gb, p->Np, 32, BK, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B);
    if (ok && passes > 1)
        ok = make_map(&p->a_lo, p->s_alo, K, M, Ga, p->Kp, BK, 128, CU_TENSOR_MAP_SWIZZLE_64B) &&
             make_map(&p->b_lo, p->s_blo, N, K, Gb, p->Np, 32, BK, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B);
    else if (ok) { p->a_lo = p->a_hi; p->b_lo = p->b_hi; }
    if (!ok) { lancius_set_error(LANCIUS_ERROR_INTERNAL); return LANCIUS_ERROR_INTERNAL; }
    return LANCIUS_ERROR_OK;
}

extern "C" lancius_error lcu_gemm_tc_use_presplit_b(LcuTcGemmPlan* p, float* b_hi, float* b_lo) {
    if (p->conv.n || !b_hi || (p->passes > 1 && !b_lo)) { lancius_set_error(LANCIUS_ERROR_INTERNAL); return LANCIUS_ERROR_INTERNAL; }
    bool ok = make_map(&p->b_hi, b_hi, p->N, p->K, p->Gb, p->Np, 32, BK, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B);
    if (ok && p->passes > 1) ok = make_map(&p->b_lo, b_lo, p->N, p->K, p->Gb, p->Np, 32, BK, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B);
    else if (ok) p->b_lo = p->b_hi;
    if (!ok) { lancius_set_error(LANCIUS_ERROR_INTERNAL); return LANCIUS_ERROR_INTERNAL; }
    p->s_bhi = b_hi; p->s_blo = p->passes > 1 ? b_lo : nullptr;
    p->b_presplit = 1;
    return LANCIUS_ERROR_OK;
}

extern "C" bool lcu_gemm_tc_make_raw_a_map(CUtensorMap* m, const float* a, size_t M, size_t K) {
    if (K % 4 || (reinterpret_cast<uintptr_t>(a) & 15) || !M || !K) return false;
    return make_map(m, a, K, M, 1, K, BK, 128, CU_TENSOR_MAP_SWIZZLE_64B);   // 128-row boxes
}

extern "C" lancius_error lcu_gemm_tc_use_raw_a(LcuTcGemmPlan* p, const CUtensorMap* d_maps) {
    if (p->conv.n || !d_maps) { lancius_set_error(LANCIUS_ERROR_INTERNAL); return LANCIUS_ERROR_INTERNAL; }
    p->d_amaps = d_maps;
    return LANCIUS_ERROR_OK;
}

#if LCU_GEMM_TRACE
extern "C" int lcu_gemm_trace_dump(unsigned long long* host, int ctas) {
    return cudaMemcpyFromSymbol(host, g_gtrace, (size_t)ctas * 8 * sizeof(unsigned long long)) == cudaSuccess ? 0 : -1;
}
#endif

extern "C" lancius_error lcu_tf32_split_rows(const float* src, size_t rows, size_t cols, size_t pitch, float* hi, float* lo,
                                             void* stream) {
    if (!rows || !cols) return LANCIUS_ERROR_OK;
    k_split_one<<<(unsigned)(rows < 65535 ? rows : 65535), 256, 0, lcu_as_stream(stream)>>>(src, rows, cols, pitch, hi, lo);
    return lcu_launch_status();
}

extern "C" lancius_error lcu_gemm_tc_run(const LcuTcGemmPlan* p, const LcuGemmGroup* d_groups, int epi, void* stream) {
    LcuColDest none{};
    return lcu_gemm_tc_run_dst(p, d_groups, epi, none, stream);
}

extern "C" lancius_error lcu_gemm_tc_run_dst(const LcuTcGemmPlan* p, const LcuGemmGroup* d_groups, int epi,
                                             LcuColDest dst, void* stream) {
    static bool configured[64] = {};     // the attribute is per device
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) { lancius_set_error(LANCIUS_ERROR_INTERNAL); return LANCIUS_ERROR_INTERNAL; }
    if (!configured[dev]) {
        if (cudaFuncSetAttribute(k_gemm_tc<false, 256>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes(256)) != cudaSuccess ||
            cudaFuncSetAttribute(k_gemm_tc<true, 256>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes(256)) != cudaSuccess ||
            cudaFuncSetAttribute(k_gemm_tc<false, 192>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes(192)) != cudaSuccess)
            return lcu_launch_status();
        configured[dev] = true;
    }
    cudaStream_t st = lcu_as_stream(stream);
    float* lo_a = p->passes > 1 ? p->s_alo : nullptr;
    float* lo_b = p->passes > 1 ? p->s_blo : nullptr;
    if (p->K > 0 && p->passes == 0) {
        __nv_bfloat16* a16 = reinterpret_cast<__nv_bfloat16*>(p->s_ahi);
        __nv_bfloat16* b16 = reinterpret_cast<__nv_bfloat16*>(p->s_bhi);
        k_to_bf16_a<<<dim3(lcu_blocks(p->M * p->Kp, 256), p->G), 256, 0, st>>>(d_groups, p->M, p->K, p->Kp, a16);
        k_to_bf16_bt<<<dim3((unsigned)((p->N + 31) / 32), (unsigned)((p->Kp + 31) / 32), p->G), dim3(32, 8), 0, st>>>(
            d_groups, p->K, p->N, p->Kp, b16);
        lcu_note_launch();
        lcu_note_launch();
    } else if (p->K > 0) {
        if (!p->d_amaps) {
            k_split<<<dim3((unsigned)(p->M < 65535 ? p->M : 65535), p->G), 256, 0, st>>>(d_groups, 0, p->M, p->K, p->Kp, p->s_ahi, lo_a);
            lcu_note_launch();
        }
        if (p->conv.n)
            k_im2col_split<<<dim3((unsigned)((p->N + 1023) / 1024 < 64 ? (p->N + 1023) / 1024 : 64), (unsigned)p->K), 256, 0, st>>>(
                d_groups, p->conv, p->Np, p->s_bhi, lo_b);
        else if (!p->b_presplit)
            k_split<<<dim3((unsigned)(p->K < 65535 ? p->K : 65535), p->G), 256, 0, st>>>(d_groups, 1, p->K, p->N, p->Np, p->s_bhi, lo_b);
        if (p->conv.n || !p->b_presplit) lcu_note_launch();
    }
    // tile width: 192 where it takes fewer tile-column-rounds of the SMs (a tile's time is
    // about proportional to its width); BF16 and the fused all-gather keep 256
    const size_t mt = (p->M + BM - 1) / BM, gz = (size_t)p->G * p->splits;
    auto cost = [&](size_t bn) { return ((mt * ((p->N + bn - 1) / bn) * gz + LCU_SMS - 1) / LCU_SMS) * bn; };
    const char* bn_env = getenv("LCU_GEMM_BN");
    const bool narrow = p->passes > 0 && dst.n_dst == 0 && !(bn_env && atoi(bn_env) == 256) &&
                        ((bn_env && atoi(bn_env) == 192) || cost(192) < cost(256));
    const unsigned tbn = narrow ? 192u : 256u;
    dim3 grid((unsigned)((p->N + tbn - 1) / tbn), (unsigned)((p->M + BM - 1) / BM), (unsigned)(p->G * p->splits));
    if (narrow)
        k_gemm_tc<false, 192><<<grid, THREADS, smem_bytes(192), st>>>(p->a_hi, p->a_lo, p->b_hi, p->b_lo, d_groups, (int)p->M,
                                                                      (int)p->N, (int)p->K, epi, p->passes, p->splits,
                                                                      p->kchunk, p->partial,
                                                                      p->conv.n ? p->conv.ho * p->conv.wo : 0, dst, p->d_amaps);
    else if (dst.n_dst > 0)
        k_gemm_tc<true, 256><<<grid, THREADS, smem_bytes(256), st>>>(p->a_hi, p->a_lo, p->b_hi, p->b_lo, d_groups, (int)p->M, (int)p->N,
                                                           (int)p->K, epi, p->passes, p->splits, p->kchunk, p->partial,
                                                           p->conv.n ? p->conv.ho * p->conv.wo : 0, dst, p->d_amaps);
    else
        k_gemm_tc<false, 256><<<grid, THREADS, smem_bytes(256), st>>>(p->a_hi, p->a_lo, p->b_hi, p->b_lo, d_groups, (int)p->M, (int)p->N,
                                                            (int)p->K, epi, p->passes, p->splits, p->kchunk, p->partial,
                                                            p->conv.n ? p->conv.ho * p->conv.wo : 0, dst, p->d_amaps);
    lcu_note_launch();
    if (p->splits > 1) {
        k_splitk_reduce<<<dim3(lcu_blocks(p->M * p->N, 256 * 4, 148 * 8), p->G), 256, 0, st>>>(d_groups, p->partial, p->splits,
                                                                                               p->M, p->N, epi,
                                                                                               p->conv.n ? (size_t)p->conv.ho * p->conv.wo : 0,
                                                                                               dst);
        lcu_note_launch();
    }
    return lcu_launch_status();
}

// Watchdog word of the tensor-core kernels: 0 = no timeout, else the role that gave up.
extern "C" int lcu_gemm_watchdog_read_and_clear(void) {
    int v = 0, z = 0;
    cudaMemcpyFromSymbol(&v, g_gemm_watchdog, sizeof(int));
    if (v) cudaMemcpyToSymbol(g_gemm_watchdog, &z, sizeof(int));
    return v;
}

// ---------------------------------------------------------------------------
// Per-op entry: scratch comes from a per-device cache that grows on demand.

namespace {
struct ScratchCache { void* p = nullptr; size_t bytes = 0; };
std::mutex g_scratch_mu;
std::vector<ScratchCache> g_scratch;
}

static void* acquire_from(std::vector<ScratchCache>& cache, size_t bytes) {
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lk(g_scratch_mu);
    if ((int)cache.size() <= dev) cache.resize(dev + 1);
    ScratchCache& c = cache[dev];
    if (c.bytes < bytes) {
        if (c.p) { cudaDeviceSynchronize(); cudaFree(c.p); c.p = nullptr; c.bytes = 0; }
        if (cudaMalloc(&c.p, bytes) != cudaSuccess) { cudaGetLastError(); c.p = nullptr; return nullptr; }
        c.bytes = bytes;
    }
    return c.p;
}

namespace { std::vector<ScratchCache> g_gather, g_decode; }
// Per-device cached buffers that grow on demand: GEMM/conv operand scratch, and a
// second one for the column-split all-gather (both alive during one colsplit call).
extern "C" void* lcu_scratch_acquire(size_t bytes) { return acquire_from(g_scratch, bytes); }
extern "C" void* lcu_scratch_acquire_gather(size_t bytes) { return acquire_from(g_gather, bytes); }
// split-KV partials of the decode attention
extern "C" void* lcu_scratch_acquire_decode(size_t bytes) { return acquire_from(g_decode, bytes); }

extern "C" lancius_error lcu_gemm_tc(float* c, const float* a, const float* b, size_t M, size_t K, size_t N,
                                     const float* bias, int epi, int mode, void* stream) {
    int passes = lcu_gemm_passes(mode);
    size_t need = lcu_gemm_tc_scratch_bytes(M, N, K, 1, 1, 1, passes) + 256;
    char* scratch = static_cast<char*>(lcu_scratch_acquire(need));
    if (!scratch) { lancius_set_error(LANCIUS_ERROR_OOM); return LANCIUS_ERROR_OOM; }
    // the one-entry group table lives at the end of the scratch region
    LcuGemmGroup* d_group = reinterpret_cast<LcuGemmGroup*>(scratch + need - 256);
    LcuGemmGroup h{a, b, c, bias, nullptr};
    cudaStream_t st = lcu_as_stream(stream);
    cudaError_t ce = cudaMemcpyAsync(d_group, &h, sizeof(h), cudaMemcpyHostToDevice, st);
    if (ce != cudaSuccess) return lcu_check_cuda(ce);
    LcuTcGemmPlan p;
    lancius_error e = lcu_gemm_tc_prepare(&p, scratch, M, N, K, 1, 1, 1, passes);
    if (e != LANCIUS_ERROR_OK) return e;
    e = lcu_gemm_tc_run(&p, d_group, epi, stream);
    // the host-side group record must stay valid until the copy ran
    if (e == LANCIUS_ERROR_OK) e = lcu_check_stream(st);
    return e;
}

// Implicit-GEMM conv on the tensor cores: C[Co, N*Ho*Wo] = W[Co, Ci*Kh*Kw] * im2col(in),
// stored straight into NCHW by the epilogue (ReLU fused). Scratch from the per-device cache.
extern "C" lancius_error lcu_conv2d_tc(float* out, const float* in, const float* w, LcuConvShape cs, int relu, int mode,
                                       void* stream) {
    const int passes = lcu_gemm_passes(lcu_contraction_mode(mode));
    const size_t M = cs.co, K = (size_t)cs.ci * cs.kh * cs.kw, N = (size_t)cs.n * cs.ho * cs.wo;
    const size_t need = lcu_gemm_tc_scratch_bytes(M, N, K, 1, 1, 1, passes) + 256;
    char* scratch = static_cast<char*>(lcu_scratch_acquire(need));
    if (!scratch) { lancius_set_error(LANCIUS_ERROR_OOM); return LANCIUS_ERROR_OOM; }
    LcuGemmGroup* d_group = reinterpret_cast<LcuGemmGroup*>(scratch + need - 256);
    LcuGemmGroup h{w, in, out, nullptr, nullptr};
    cudaStream_t st = lcu_as_stream(stream);
    cudaError_t ce = cudaMemcpyAsync(d_group, &h, sizeof(h), cudaMemcpyHostToDevice, st);
    if (ce != cudaSuccess) return lcu_check_cuda(ce);
    LcuTcGemmPlan p;
    lancius_error e = lcu_gemm_tc_prepare(&p, scratch, M, N, K, 1, 1, 1, passes);
    if (e != LANCIUS_ERROR_OK) return e;
    p.conv = cs;
    e = lcu_gemm_tc_run(&p, d_group, relu ? LCU_EPI_RELU : LCU_EPI_NONE, stream);
    if (e == LANCIUS_ERROR_OK) e = lcu_check_stream(st);
    return e;
}

// Device address of this file's watchdog word on the current device (0 if unavailable).
extern "C" int* lcu_gemm_watchdog_addr(void) {
    void* p = nullptr;
    return cudaGetSymbolAddress(&p, g_gemm_watchdog) == cudaSuccess ? static_cast<int*>(p) : nullptr;
}

// Self-test of the timeout path: one thread waits on an mbarrier that nothing arrives on,
// with a short poll limit, then records a timeout in this file's watchdog word exactly as
// the GEMM's own waits do. No fault, no hang: the kernel returns after the limit.
namespace {
__global__ void k_watchdog_selftest(int where) {
    __shared__ uint64_t bar;
    if (threadIdx.x != 0) return;
    tc::mbar_init(&bar, 1);
    tc::fence_barrier_init();
    for (int i = 0; i < 1024; i++)
        if (tc::mbar_try(&bar, 0)) return;       // phase 0 never completes
    atomicCAS(&g_gemm_watchdog, 0, where);
}
}  // namespace

extern "C" lancius_error lcu_watchdog_selftest(void* stream) {
    k_watchdog_selftest<<<1, 32, 0, lcu_as_stream(stream)>>>(99);
    lcu_note_launch();
    return lcu_launch_status();
}
