/*
 * lcu_oracle.h -- TEST INFRASTRUCTURE ONLY (parity checker, never the product).
 *
 * FP64 CPU restatement of the Lancius reference's dense kernels and of its
 * arena-mode graph executor. Only tests/, __graft_entry__.smoke() and bench.py's
 * CPU-baseline leg load this library. Each function names the reference lines it
 * restates (paths inside the reference project, tree bleeding/v11A1 unless noted).
 */
#ifndef LCU_ORACLE_H
#define LCU_ORACLE_H
#include <stddef.h>
#include "lancius/lancius_ir.h"

void orc_matmul(double* out, const double* a, const double* b, size_t M, size_t K, size_t N);
void orc_conv2d(double* out, const double* in, const double* w, size_t N, size_t C_in, size_t H_in,
                size_t W_in, size_t C_out, size_t K_h, size_t K_w, size_t stride, size_t pad, int relu);
void orc_maxpool2d(double* out, const double* in, size_t N, size_t C, size_t H_in, size_t W_in, size_t K, size_t stride);
void orc_layernorm(double* out, const double* in, const double* gamma, const double* beta, size_t rows, size_t hidden, double eps);
void orc_gelu(double* out, const double* in, size_t n);
void orc_softmax(double* out, const double* in, size_t rows, size_t cols);
void orc_attention(double* out, const double* q, const double* k, const double* v, size_t S, size_t H, size_t D, int causal);
void orc_naive_attention(double* out, const double* q, const double* k, const double* v, size_t S, size_t H, size_t D);
void orc_sum_axis1(double* out, const double* in, size_t rows, size_t cols);
void orc_swiglu(double* out, const double* gate, const double* up, size_t n);
void orc_attention_kv_cache(double* out, const double* q, const double* kc, const double* vc, size_t S, size_t H,
                            size_t D);
void orc_conv2d_int8(double* out, const double* in, const int8_t* w, double scale_w, size_t N, size_t Ci, size_t H,
                     size_t W, size_t Co, size_t Kh, size_t Kw, size_t stride, size_t pad, int relu);
void orc_gqa(double* out, const double* q, const double* k, const double* v, size_t S, size_t Hq, size_t Hkv, size_t D);
void orc_rope(double* q, double* k, size_t B, size_t S, size_t H, size_t D, int pos_offset);
void orc_conv2d_bwd_in(double* out, const double* grad, const double* w, size_t N, size_t Ci, size_t H, size_t W,
                       size_t Co, size_t Ho, size_t Wo, size_t Kh, size_t Kw, size_t stride, size_t pad);
void orc_conv2d_bwd_w(double* out, const double* grad, const double* in, size_t N, size_t Ci, size_t H, size_t W,
                      size_t Co, size_t Ho, size_t Wo, size_t Kh, size_t Kw, size_t stride, size_t pad);
void orc_maxpool2d_bwd(double* out, const double* grad, const double* in, size_t N, size_t C, size_t H, size_t W,
                       size_t Ho, size_t Wo, size_t K, size_t stride);
void orc_matmul_int8(double* out, const double* a, const int8_t* b, double scale_b, size_t M, size_t K, size_t N);
void orc_rmsnorm(double* out, const double* in, const double* gamma, size_t rows, size_t hidden, double eps);

/* Executes the graph on the CPU in arena mode (every node its own buffer).
 * Returns a table indexed by node id (NULL for NOP nodes); INPUT entries point at
 * the node's bound runtime_data. Free with orc_free_results(). */
double** orc_run_graph(const lancius_graph* g);
void orc_free_results(const lancius_graph* g, double** results);

#endif
