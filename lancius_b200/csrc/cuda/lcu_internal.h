// Internal launcher interface shared by the executor and the per-op C ABI.
// Group tables (device-resident arrays of per-instance pointers) let one launch
// cover every same-shaped node of a wave.
#pragma once
#include "common.cuh"
#include <cuda.h>

// tensor-core GEMM passes of a precision mode: 3 (3xTF32), 1 (TF32), 0 (BF16 operands)
static inline int lcu_gemm_passes(int mode) { return mode == LCU_MODE_BF16 ? 0 : mode == LCU_MODE_TF32 ? 1 : 3; }
// conv and attention have no BF16 form: the BF16 mode runs them as one TF32 pass
static inline int lcu_contraction_mode(int mode) { return mode == LCU_MODE_BF16 ? (int)LCU_MODE_TF32 : mode; }

struct LcuGemmGroup {        // one independent product C = act(A*B + bias) + resid
    const float* a;
    const float* b;
    float* c;
    const float* bias;   // [N] row vector added to every row, or NULL
    const float* resid;  // [M,N] added after the activation, or NULL
    // tensor-core path: scratch slot of this group's hi/lo A and B copies; a group whose
    // operand equals an earlier group's (adup/bdup = 1) reuses that slot and skips the split
    int aidx, bidx, adup, bdup;
};
struct LcuAttnGroup { const float* q; const float* k; const float* v; float* o; };
struct LcuEltGroup { float* out; const float* a; const float* b; };
struct LcuRowGroup { float* out; const float* in; const float* gamma; const float* beta; };

struct LcuConvShape { int n, ci, h, w, co, kh, kw, stride, pad, ho, wo; };   // n == 0: not a conv

// Extra destinations of a GEMM result (the column-split GEMM's fused all-gather): element
// (m, n) of the [M, N] product is stored at ptr[i][m * ldc + col_off + n] for every i < n_dst,
// local and peer (NVLink) memory alike, instead of into the group's own C.
struct LcuColDest { float* ptr[8]; int n_dst; size_t ldc, col_off; };

// A prepared tensor-core GEMM: TMA maps over the hi/lo scratch copies of A and B.
struct LcuTcGemmPlan {
    CUtensorMap a_hi, a_lo, b_hi, b_lo;
    float *s_ahi, *s_alo, *s_bhi, *s_blo;
    size_t M, N, K, Kp, Np;
    int G, Ga, Gb, passes;       // groups, distinct A operands, distinct B operands
    int splits, kchunk;          // K cut into `splits` chunks of kchunk (multiple of 16)
    float* partial;              // [G][splits][M][N] partial sums when splits > 1
    LcuConvShape conv;           // conv.n > 0: B is the im2col of groups[0].b, C is stored NCHW
    int b_presplit;              // 1: b maps point at persistent hi/lo weight copies; no B split per run
    const CUtensorMap* d_amaps;  // raw-A mode: per-distinct-A maps (device memory) over the FP32 operands
                                 // themselves, split into hi/lo inside the GEMM; no A split pass
};

// Internal epilogue of the CUDA-core small-product GEMM: bias, then a row softmax over
// all N <= 32 columns held by one tile (a MATMUL -> ADD(bias) -> SOFTMAX chain)
constexpr int LCU_EPI_SOFTMAX_ROW = 16;
int lcu_gemm_softmax_fold_ok(size_t M, size_t N, size_t K);
// Two chained small products in one launch (gemm_simt.cu, k_mlp2): H = epi1(A1 B1 + bias1),
// then Y = epi2(H B2 + bias2) with N2 <= 32; tickets: ceil(M / 16) zeroed words, left zeroed.
int lcu_mlp2_ok(size_t M, size_t N1, size_t K1, size_t N2);
lancius_error lcu_mlp2(const LcuGemmGroup* d_l1, const LcuGemmGroup* d_l2, size_t M, size_t N1, size_t K1, int epi1,
                       size_t N2, int epi2, unsigned* d_tickets, void* stream);

extern "C" {
size_t lcu_gemm_tc_scratch_bytes(size_t M, size_t N, size_t K, int G, int Ga, int Gb, int passes);
lancius_error lcu_gemm_tc_prepare(LcuTcGemmPlan* p, void* scratch, size_t M, size_t N, size_t K, int G, int Ga, int Gb,
                                  int passes);
// Points a prepared plan's B maps at persistent [Gb][K][pad4(N)] hi/lo copies (made by
// lcu_tf32_split_rows) so runs skip the per-call B split; undone by the next prepare.
lancius_error lcu_gemm_tc_use_presplit_b(LcuTcGemmPlan* p, float* b_hi, float* b_lo);
// Raw-A mode: a map over the FP32 A operand itself ([M][K] row-major; K % 4 == 0, 16-byte
// aligned, false otherwise), one per distinct A, stored in device memory and handed to the plan.
bool lcu_gemm_tc_make_raw_a_map(CUtensorMap* m, const float* a, size_t M, size_t K);
lancius_error lcu_gemm_tc_use_raw_a(LcuTcGemmPlan* p, const CUtensorMap* d_maps);
// hi = rna_tf32(x), lo = rna_tf32(x - hi) of a row-major [rows, cols] matrix into rows of `pitch` floats
lancius_error lcu_tf32_split_rows(const float* src, size_t rows, size_t cols, size_t pitch, float* hi, float* lo,
                                  void* stream);
lancius_error lcu_gemm_tc_run(const LcuTcGemmPlan* p, const LcuGemmGroup* d_groups, int epi, void* stream);
lancius_error lcu_gemm_tc_run_dst(const LcuTcGemmPlan* p, const LcuGemmGroup* d_groups, int epi, LcuColDest dst,
                                  void* stream);
lancius_error lcu_gemm_simt_grouped(const LcuGemmGroup* d_groups, int count, size_t M, size_t N, size_t K, int epi,
                                    void* stream);
lancius_error lcu_gemm_simt(float* c, const float* a, const float* b, size_t M, size_t K, size_t N, const float* bias,
                            int epi, void* stream);
lancius_error lcu_conv2d_simt(float* out, const float* in, const float* w, size_t N, size_t Ci, size_t H, size_t W,
                              size_t Co, size_t Kh, size_t Kw, size_t stride, size_t pad, int relu, void* stream);
lancius_error lcu_attention_simt(const LcuAttnGroup* d_table, const float* q, const float* k, const float* v, float* o,
                                 size_t B, size_t S, size_t H, size_t D, int causal, void* stream);
lancius_error lcu_eltwise_grouped(int op, const LcuEltGroup* d_table, int count, size_t n, int vec, void* s);
lancius_error lcu_layernorm_grouped(const LcuRowGroup* d_table, int count, LcuRowGroup one, size_t rows, size_t hidden,
                                    float eps, int vec, void* s);
lancius_error lcu_copy_f32(float* o, const float* a, size_t n, void* s);
lancius_error lcu_convert_f64_to_f32(float* o, const double* a, size_t n, void* s);
lancius_error lcu_convert_f32_to_f64(double* o, const float* a, size_t n, void* s);
lancius_error lcu_gemm_tc(float* c, const float* a, const float* b, size_t M, size_t K, size_t N, const float* bias,
                          int epi, int mode, void* stream);
int lcu_gemm_watchdog_read_and_clear(void);
int lcu_use_tensor_cores(size_t M, size_t N, size_t K);
int lcu_attention_tc_supported(size_t D);
int lcu_force_simt(void);
int lcu_no_weight_cache(void);
int lcu_no_raw_a(void);
lancius_error lcu_conv2d_tc(float* out, const float* in, const float* w, LcuConvShape cs, int relu, int mode, void* stream);
// direct implicit-GEMM conv over NHWC hi/lo copies (conv_tc.cu); scratch of
// lcu_conv_nhwc_scratch_bytes(cs, passes) bytes
int lcu_conv_nhwc_supported(LcuConvShape cs);
size_t lcu_conv_nhwc_scratch_bytes(LcuConvShape cs, int passes);
lancius_error lcu_conv2d_tc_nhwc(float* out, const float* in, const float* w, LcuConvShape cs, int relu, int mode,
                                 void* scratch, void* stream);
// in_nhwc: the input already is NHWC FP32 (a previous conv's output); out_nhwc: write the
// output NHWC (needs lcu_conv_nhwc_out_ok)
lancius_error lcu_conv_weight_split(const float* w, float* hi, float* lo, int co, int ci, int kh, int kw, void* stream);
lancius_error lcu_conv2d_tc_nhwc_ex(float* out, const float* in, const float* w, LcuConvShape cs, int relu, int mode,
                                   void* scratch, void* stream, int in_nhwc, int out_nhwc, const float* in_lo,
                                   float* out_lo, const float* w_hi, const float* w_lo, float* gap, int* gap_written);
int lcu_conv_tiles_per_image(LcuConvShape cs);
lancius_error lcu_conv_gap_sum(float* out, const float* gap, int n, int co, int tiles, void* stream);
int lcu_conv_nhwc_out_ok(LcuConvShape cs);
// NHWC FP32 -> NCHW FP32 (f64 = 0) or FP64 (f64 = 1)
lancius_error lcu_nhwc_to_nchw(void* out, const float* in, int n, int c, int h, int w, int f64, void* stream);
// short-reduction conv writing NHWC (out_nhwc) where lcu_conv_smallk_nhwc_ok holds
lancius_error lcu_conv2d_smallk_ex(float* out, const float* in, const float* w, size_t N, size_t Ci, size_t H, size_t W,
                                   size_t Co, size_t Kh, size_t Kw, size_t stride, size_t pad, int relu, int out_nhwc,
                                   void* stream, float* out_lo);
// tensor-core short-reduction conv (Ci*Kh*Kw <= 32 stems, Co % 32 == 0, Co <= 128) writing
// NHWC (+ its tf32_lo copy when out_lo is given)
int lcu_conv_small_tc_ok(size_t N, size_t Ci, size_t H, size_t W, size_t Co, size_t Kh, size_t Kw, size_t stride,
                         size_t pad);
lancius_error lcu_conv2d_small_tc_nhwc(float* out, float* out_lo, const float* in, const float* w, size_t N, size_t Ci,
                                       size_t H, size_t W, size_t Co, size_t Kh, size_t Kw, size_t stride, size_t pad,
                                       int relu, int mode, void* stream);
int lcu_conv_smallk_nhwc_ok(size_t N, size_t Ci, size_t H, size_t W, size_t Co, size_t Kh, size_t Kw, size_t stride,
                            size_t pad);
int lcu_conv_force_im2col(void);
// direct CUDA-core conv for Ci*Kh*Kw <= 32 (first layers), any stride and padding
int lcu_conv_smallk_supported(size_t Ci, size_t Kh, size_t Kw, size_t Co);
int lcu_force_tc_conv(void);
lancius_error lcu_conv2d_smallk(float* out, const float* in, const float* w, size_t N, size_t Ci, size_t H, size_t W,
                                size_t Co, size_t Kh, size_t Kw, size_t stride, size_t pad, int relu, void* stream);   // LCU_CONV_IM2COL=1: keep the materialised-im2col conv
int lcu_conv_watchdog_read_and_clear(void);
void* lcu_scratch_acquire(size_t bytes);
// INT8 weights: tensor cores (gemm_i8.cu) above lcu_int8_use_tc's size, CUDA cores below;
// scratch = the *_scratch_bytes() of device memory, or NULL for a library buffer.
int lcu_int8_use_tc(size_t M, size_t N, size_t K);
size_t lcu_matmul_int8_scratch_bytes(size_t M, size_t K, size_t N);
size_t lcu_conv2d_int8_scratch_bytes(size_t N, size_t Ci, size_t H, size_t W, size_t Co, size_t Kh, size_t Kw,
                                     size_t stride, size_t pad);
// b_packed: the weights already K-major ([N][Kp], lcu_int8_pack_kmajor), or NULL
lancius_error lcu_matmul_int8(float* out, const float* a, const int8_t* b, double scale_b, size_t M, size_t K, size_t N,
                              const int8_t* b_packed, float* amax_scratch, void* scratch, void* s);
lancius_error lcu_int8_pack_kmajor(int8_t* dst, const int8_t* b, size_t K, size_t N, size_t Kp, void* s);
lancius_error lcu_conv2d_int8(float* out, const float* in, const int8_t* w, double scale_w, size_t N, size_t Ci, size_t H,
                              size_t W, size_t Co, size_t Kh, size_t Kw, size_t stride, size_t pad, int relu,
                              float* amax_scratch, void* scratch, void* s);
lancius_error lcu_matmul_int8_simt(float* out, const float* a, const int8_t* b, double scale_b, size_t M, size_t K,
                                   size_t N, float* amax_scratch, void* s);
lancius_error lcu_conv2d_int8_simt(float* out, const float* in, const int8_t* w, double scale_w, size_t N, size_t Ci,
                                   size_t H, size_t W, size_t Co, size_t Kh, size_t Kw, size_t stride, size_t pad,
                                   int relu, float* amax_scratch, void* s);
int lcu_int8_watchdog_read_and_clear(void);
int* lcu_attention_watchdog_addr(void);
int* lcu_conv_watchdog_addr(void);
int* lcu_int8_watchdog_addr(void);
int* lcu_gemm_watchdog_addr(void);
void* lcu_scratch_acquire_gather(size_t bytes);
void* lcu_scratch_acquire_decode(size_t bytes);
// mode: LCU_MODE_FP32_EXACT (3xTF32) or LCU_MODE_TF32 (one pass)
// d_table: a grouped launch over `B` operand sets, whose tensor maps (made by
// lcu_attention_tc_make_maps with B = 1) are at d_maps in device memory; else q/k/v/o are
// [B][S][H][D] and the maps are built per call.
// lo: lcu_attention_tc_lo_floats(B, S, H) floats for the K/V lo copies (NULL on the per-op
// path: the per-device scratch is used); a grouped launch's maps (LCU_ATTN_TC_MAPS per set:
// Q, K, V, K lo, V lo, O) must point into that buffer at set i's [2][S][H][D] block.
#define LCU_ATTN_TC_MAPS 6
lancius_error lcu_attention_tc(const LcuAttnGroup* d_table, const float* q, const float* k, const float* v, float* o,
                               size_t B, size_t S, size_t H, int causal, int mode, const CUtensorMap* d_maps,
                               float* lo, void* stream);
bool lcu_attention_tc_make_maps(CUtensorMap* maps, const float* q, const float* k, const float* v, const float* o,
                                const float* lo, size_t B, size_t S, size_t H);
size_t lcu_attention_tc_lo_floats(size_t B, size_t S, size_t H);
int lcu_attention_tc_needs_lo(void);   // 0: the kernel splits K and V itself, lo may be NULL
int lcu_attention_watchdog_read_and_clear(void);
void lcu_reset_launch_count(void);
int lcu_launch_count(void);
// cudaStreamSynchronize + report (and clear) tensor-core watchdog trips as LANCIUS_ERROR_INTERNAL
lancius_error lcu_check_stream(void* stream);
void lcu_ctx_retarget_schedule(lcu_ctx* c, lancius_schedule* s);
}
