/*
 * TEST INFRASTRUCTURE ONLY -- FP64 CPU restatement of the Lancius reference's
 * hot-path math, used as the parity checker. Not linked by the product.
 * Loop orders follow the reference so that sums accumulate in the same order.
 */
#include "lcu_oracle.h"
#include <math.h>
#include <stdlib.h>
#include <string.h>

/* src/math/lancius_kernels.c:15-26 and the executor MATMUL at
 * src/runtime/lancius_scheduler.c:222-234: zero, then i-k-j accumulation. */
void orc_matmul(double* out, const double* a, const double* b, size_t M, size_t K, size_t N) {
    #pragma omp parallel for schedule(static)
    for (size_t r = 0; r < M; r++) {
        double* o = out + r * N;
        for (size_t c = 0; c < N; c++) o[c] = 0.0;
        for (size_t k = 0; k < K; k++) {
            double av = a[r * K + k];
            const double* br = b + k * N;
            for (size_t c = 0; c < N; c++) o[c] += av * br[c];
        }
    }
}

/* lancius_kernels.c:28-60 (relu=0) and :140-173 (relu=1): direct NCHW/OIHW conv,
 * zero padding, sum over (ci, kh, kw) in that order. */
void orc_conv2d(double* out, const double* in, const double* w, size_t N, size_t C_in, size_t H_in,
                size_t W_in, size_t C_out, size_t K_h, size_t K_w, size_t stride, size_t pad, int relu) {
    size_t H_out = (H_in + 2 * pad - K_h) / stride + 1, W_out = (W_in + 2 * pad - K_w) / stride + 1;
    #pragma omp parallel for collapse(2) schedule(static)
    for (size_t n = 0; n < N; n++)
        for (size_t co = 0; co < C_out; co++)
            for (size_t ho = 0; ho < H_out; ho++)
                for (size_t wo = 0; wo < W_out; wo++) {
                    double s = 0.0;
                    for (size_t ci = 0; ci < C_in; ci++)
                        for (size_t kh = 0; kh < K_h; kh++)
                            for (size_t kw = 0; kw < K_w; kw++) {
                                long ih = (long)(ho * stride) - (long)pad + (long)kh;
                                long iw = (long)(wo * stride) - (long)pad + (long)kw;
                                if (ih < 0 || iw < 0 || ih >= (long)H_in || iw >= (long)W_in) continue;
                                s += in[((n * C_in + ci) * H_in + (size_t)ih) * W_in + (size_t)iw] *
                                     w[((co * C_in + ci) * K_h + kh) * K_w + kw];
                            }
                    out[((n * C_out + co) * H_out + ho) * W_out + wo] = (relu && !(s > 0.0)) ? 0.0 : s;
                }
}

/* src/runtime/lancius_vision_ops.c:82-112: max over a KxK window, no padding, start -1e9 */
void orc_maxpool2d(double* out, const double* in, size_t N, size_t C, size_t H_in, size_t W_in, size_t K, size_t stride) {
    size_t H_out = (H_in - K) / stride + 1, W_out = (W_in - K) / stride + 1;
    for (size_t p = 0; p < N * C; p++)
        for (size_t ho = 0; ho < H_out; ho++)
            for (size_t wo = 0; wo < W_out; wo++) {
                double m = -1e9;
                for (size_t kh = 0; kh < K; kh++)
                    for (size_t kw = 0; kw < K; kw++) {
                        double v = in[(p * H_in + ho * stride + kh) * W_in + wo * stride + kw];
                        if (v > m) m = v;
                    }
                out[(p * H_out + ho) * W_out + wo] = m;
            }
}

/* lancius_kernels.c:217-236: two-pass mean / biased variance per row */
void orc_layernorm(double* out, const double* in, const double* gamma, const double* beta, size_t rows, size_t hidden, double eps) {
    for (size_t r = 0; r < rows; r++) {
        const double* x = in + r * hidden;
        double mean = 0.0, var = 0.0;
        for (size_t i = 0; i < hidden; i++) mean += x[i];
        mean /= (double)hidden;
        for (size_t i = 0; i < hidden; i++) var += (x[i] - mean) * (x[i] - mean);
        var /= (double)hidden;
        double inv = 1.0 / sqrt(var + eps);
        for (size_t i = 0; i < hidden; i++) out[r * hidden + i] = (x[i] - mean) * inv * gamma[i] + beta[i];
    }
}

/* lancius_kernels.c:238-246: tanh-form GELU with the input clamped to [-100, 100] */
void orc_gelu(double* out, const double* in, size_t n) {
    const double c = 0.7978845608028654;
    for (size_t i = 0; i < n; i++) {
        double x = in[i];
        if (x > 100.0) x = 100.0;
        if (x < -100.0) x = -100.0;
        out[i] = 0.5 * x * (1.0 + tanh(c * (x + 0.044715 * x * x * x)));
    }
}

/* src/runtime/lancius_scheduler.c:284-294 */
void orc_softmax(double* out, const double* in, size_t rows, size_t cols) {
    for (size_t r = 0; r < rows; r++) {
        const double* x = in + r * cols;
        double* y = out + r * cols;
        double m = x[0], s = 0.0;
        for (size_t c = 1; c < cols; c++) if (x[c] > m) m = x[c];
        for (size_t c = 0; c < cols; c++) { y[c] = exp(x[c] - m); s += y[c]; }
        for (size_t c = 0; c < cols; c++) y[c] /= s;
    }
}

/* lancius_kernels.c:278-332: per (row i, head h) one streaming pass over all j with
 * the online-softmax recurrence, m starting at -1e9, scale 1/sqrt(D); causal=1
 * replaces scores of j > i by -1e9 (line 307). causal=0 is the same recurrence
 * without that line (the unmasked encoder case). */
void orc_attention(double* out, const double* q, const double* k, const double* v, size_t S, size_t H, size_t D, int causal) {
    double scale = 1.0 / sqrt((double)D);
    #pragma omp parallel for collapse(2) schedule(static)
    for (size_t i = 0; i < S; i++)
        for (size_t h = 0; h < H; h++) {
            double acc[1024];
            double m = -1e9, l = 0.0;
            const double* qr = q + (i * H + h) * D;
            for (size_t d = 0; d < D; d++) acc[d] = 0.0;
            for (size_t j = 0; j < S; j++) {
                const double* kr = k + (j * H + h) * D;
                const double* vr = v + (j * H + h) * D;
                double s = 0.0;
                for (size_t d = 0; d < D; d++) s += qr[d] * kr[d];
                s *= scale;
                if (causal && j > i) s = -1e9;
                double mn = s > m ? s : m;
                double corr = exp(m - mn), p = exp(s - mn);
                l = l * corr + p;
                for (size_t d = 0; d < D; d++) acc[d] = acc[d] * corr + p * vr[d];
                m = mn;
            }
            double inv = 1.0 / l;
            for (size_t d = 0; d < D; d++) out[(i * H + h) * D + d] = acc[d] * inv;
        }
}

/* stable/v9S/examples/audit_flash_attention.c:9-49: materialised causal softmax */
void orc_naive_attention(double* out, const double* q, const double* k, const double* v, size_t S, size_t H, size_t D) {
    double* sc = (double*)malloc(S * sizeof(double));
    double scale = 1.0 / sqrt((double)D);
    for (size_t i = 0; i < S; i++)
        for (size_t h = 0; h < H; h++) {
            double mx = -1e9, sum = 0.0;
            for (size_t j = 0; j < S; j++) {
                double s = 0.0;
                for (size_t d = 0; d < D; d++) s += q[(i * H + h) * D + d] * k[(j * H + h) * D + d];
                s *= scale;
                if (j > i) s = -1e9;
                sc[j] = s;
                if (s > mx) mx = s;
            }
            for (size_t j = 0; j < S; j++) { sc[j] = exp(sc[j] - mx); sum += sc[j]; }
            for (size_t j = 0; j < S; j++) sc[j] /= sum;
            for (size_t d = 0; d < D; d++) {
                double a = 0.0;
                for (size_t j = 0; j < S; j++) a += sc[j] * v[(j * H + h) * D + d];
                out[(i * H + h) * D + d] = a;
            }
        }
    free(sc);
}

/* src/runtime/lancius_scheduler.c:263-267 */
void orc_sum_axis1(double* out, const double* in, size_t rows, size_t cols) {
    for (size_t r = 0; r < rows; r++) {
        double s = 0.0;
        for (size_t c = 0; c < cols; c++) s += in[r * cols + c];
        out[r] = s;
    }
}

/* lancius_kernels.c:381-396 */
void orc_rmsnorm(double* out, const double* in, const double* gamma, size_t rows, size_t hidden, double eps) {
    for (size_t r = 0; r < rows; r++) {
        double sq = 0.0;
        for (size_t j = 0; j < hidden; j++) sq += in[r * hidden + j] * in[r * hidden + j];
        double inv = 1.0 / sqrt(sq / (double)hidden + eps);
        for (size_t j = 0; j < hidden; j++) out[r * hidden + j] = in[r * hidden + j] * inv * gamma[j];
    }
}


/* lancius_kernels.c:398-405 */
void orc_swiglu(double* out, const double* gate, const double* up, size_t n) {
    for (size_t i = 0; i < n; i++) { double g = gate[i]; out[i] = g / (1.0 + exp(-g)) * up[i]; }
}

/* lancius_kernels.c:407-448: causal attention, query head hq reads kv head hq / (Hq / Hkv) */
void orc_gqa(double* out, const double* q, const double* k, const double* v, size_t S, size_t Hq, size_t Hkv, size_t D) {
    size_t grp = Hq / Hkv;
    double scale = 1.0 / sqrt((double)D);
    for (size_t i = 0; i < S; i++)
        for (size_t hq = 0; hq < Hq; hq++) {
            double acc[1024], m = -1e9, l = 0.0;
            size_t hk = hq / grp;
            for (size_t d = 0; d < D; d++) acc[d] = 0.0;
            for (size_t j = 0; j < S; j++) {
                double s = 0.0;
                for (size_t d = 0; d < D; d++) s += q[(i * Hq + hq) * D + d] * k[(j * Hkv + hk) * D + d];
                s *= scale;
                if (j > i) s = -1e9;
                double mn = s > m ? s : m, corr = exp(m - mn), p = exp(s - mn);
                l = l * corr + p;
                for (size_t d = 0; d < D; d++) acc[d] = acc[d] * corr + p * v[(j * Hkv + hk) * D + d];
                m = mn;
            }
            for (size_t d = 0; d < D; d++) out[(i * Hq + hq) * D + d] = acc[d] / l;
        }
}

/* lancius_kernels.c:338-379: decode attention of one query token against [S][H][D]
 * caches, no mask; the row max starts at -1e9 as in the reference */
void orc_attention_kv_cache(double* out, const double* q, const double* kc, const double* vc, size_t S, size_t H,
                            size_t D) {
    double scale = 1.0 / sqrt((double)D);
    double* p = (double*)malloc(S * sizeof(double));
    for (size_t h = 0; h < H; h++) {
        double mx = -1e9, sum = 0.0;
        for (size_t j = 0; j < S; j++) {
            double s = 0.0;
            for (size_t d = 0; d < D; d++) s += q[h * D + d] * kc[(j * H + h) * D + d];
            p[j] = s * scale;
            if (p[j] > mx) mx = p[j];
        }
        for (size_t j = 0; j < S; j++) { p[j] = exp(p[j] - mx); sum += p[j]; }
        for (size_t d = 0; d < D; d++) {
            double acc = 0.0;
            for (size_t j = 0; j < S; j++) acc += p[j] / sum * vc[(j * H + h) * D + d];
            out[h * D + d] = acc;
        }
    }
    free(p);
}

/* lancius_kernels.c:248-272: rotary embedding on interleaved pairs, in place */
void orc_rope(double* q, double* k, size_t B, size_t S, size_t H, size_t D, int pos_offset) {
    for (size_t b = 0; b < B; b++)
        for (size_t s = 0; s < S; s++)
            for (size_t h = 0; h < H; h++)
                for (size_t d = 0; d < D; d += 2) {
                    double freq = 1.0 / pow(10000.0, (double)d / (double)D), ang = (double)((long)s + pos_offset) * freq;
                    double c = cos(ang), sn = sin(ang);
                    size_t i = ((b * S + s) * H + h) * D + d;
                    double q0 = q[i], q1 = q[i + 1], k0 = k[i], k1 = k[i + 1];
                    q[i] = q0 * c - q1 * sn; q[i + 1] = q0 * sn + q1 * c;
                    k[i] = k0 * c - k1 * sn; k[i + 1] = k0 * sn + k1 * c;
                }
}

/* lancius_kernels.c:62-91 */
void orc_conv2d_bwd_in(double* out, const double* grad, const double* w, size_t N, size_t Ci, size_t H, size_t W,
                       size_t Co, size_t Ho, size_t Wo, size_t Kh, size_t Kw, size_t stride, size_t pad) {
    memset(out, 0, N * Ci * H * W * sizeof(double));
    for (size_t n = 0; n < N; n++)
        for (size_t co = 0; co < Co; co++)
            for (size_t ho = 0; ho < Ho; ho++)
                for (size_t wo = 0; wo < Wo; wo++) {
                    double g = grad[((n * Co + co) * Ho + ho) * Wo + wo];
                    for (size_t ci = 0; ci < Ci; ci++)
                        for (size_t kh = 0; kh < Kh; kh++)
                            for (size_t kw = 0; kw < Kw; kw++) {
                                long ih = (long)(ho * stride) - (long)pad + (long)kh, iw = (long)(wo * stride) - (long)pad + (long)kw;
                                if (ih < 0 || iw < 0 || ih >= (long)H || iw >= (long)W) continue;
                                out[((n * Ci + ci) * H + (size_t)ih) * W + (size_t)iw] += g * w[((co * Ci + ci) * Kh + kh) * Kw + kw];
                            }
                }
}

/* lancius_kernels.c:93-136 (the per-thread accumulators there only change summation order) */
void orc_conv2d_bwd_w(double* out, const double* grad, const double* in, size_t N, size_t Ci, size_t H, size_t W,
                      size_t Co, size_t Ho, size_t Wo, size_t Kh, size_t Kw, size_t stride, size_t pad) {
    memset(out, 0, Co * Ci * Kh * Kw * sizeof(double));
    for (size_t n = 0; n < N; n++)
        for (size_t co = 0; co < Co; co++)
            for (size_t ho = 0; ho < Ho; ho++)
                for (size_t wo = 0; wo < Wo; wo++) {
                    double g = grad[((n * Co + co) * Ho + ho) * Wo + wo];
                    for (size_t ci = 0; ci < Ci; ci++)
                        for (size_t kh = 0; kh < Kh; kh++)
                            for (size_t kw = 0; kw < Kw; kw++) {
                                long ih = (long)(ho * stride) - (long)pad + (long)kh, iw = (long)(wo * stride) - (long)pad + (long)kw;
                                if (ih < 0 || iw < 0 || ih >= (long)H || iw >= (long)W) continue;
                                out[((co * Ci + ci) * Kh + kh) * Kw + kw] += g * in[((n * Ci + ci) * H + (size_t)ih) * W + (size_t)iw];
                            }
                }
}

/* lancius_vision_ops.c:149-190: gradient routed to the first maximum of each window */
void orc_maxpool2d_bwd(double* out, const double* grad, const double* in, size_t N, size_t C, size_t H, size_t W,
                       size_t Ho, size_t Wo, size_t K, size_t stride) {
    memset(out, 0, N * C * H * W * sizeof(double));
    for (size_t p = 0; p < N * C; p++)
        for (size_t ho = 0; ho < Ho; ho++)
            for (size_t wo = 0; wo < Wo; wo++) {
                double m = -1e9;
                size_t bi = 0, bj = 0;
                for (size_t kh = 0; kh < K; kh++)
                    for (size_t kw = 0; kw < K; kw++) {
                        size_t ih = ho * stride + kh, iw = wo * stride + kw;
                        double v = in[(p * H + ih) * W + iw];
                        if (v > m) { m = v; bi = ih; bj = iw; }
                    }
                out[(p * H + bi) * W + bj] += grad[(p * Ho + ho) * Wo + wo];
            }
}

/* lancius_scheduler.c:195-220: dynamic symmetric INT8 quantisation of A (scale max|a|/127,
 * round half away from zero), int8 x int8 -> int32 products, result * scale_a * scale_b */
void orc_matmul_int8(double* out, const double* a, const int8_t* b, double scale_b, size_t M, size_t K, size_t N) {
    double mx = 0.0;
    for (size_t i = 0; i < M * K; i++) { double v = fabs(a[i]); if (v > mx) mx = v; }
    double sa = mx > 0.0 ? mx / 127.0 : 1e-8;
    for (size_t r = 0; r < M; r++)
        for (size_t c = 0; c < N; c++) {
            int32_t acc = 0;
            for (size_t k = 0; k < K; k++) acc += (int32_t)(int8_t)round(a[r * K + k] / sa) * (int32_t)b[k * N + c];
            out[r * N + c] = (double)acc * (sa * scale_b);
        }
}

/* vision_ops.c:16-57 + lancius_kernels.c:176-210: the input quantised as in
 * orc_matmul_int8 (per tensor, on first execution), int8 x int8 -> int32 direct conv
 * (zero padding contributes nothing), result * scale_in * scale_w, then the fused ReLU */
void orc_conv2d_int8(double* out, const double* in, const int8_t* w, double scale_w, size_t N, size_t Ci, size_t H,
                     size_t W, size_t Co, size_t Kh, size_t Kw, size_t stride, size_t pad, int relu) {
    size_t E = N * Ci * H * W, Ho = (H + 2 * pad - Kh) / stride + 1, Wo = (W + 2 * pad - Kw) / stride + 1;
    double mx = 0.0;
    for (size_t i = 0; i < E; i++) { double v = fabs(in[i]); if (v > mx) mx = v; }
    double sa = mx > 0.0 ? mx / 127.0 : 1e-8;
    int8_t* q = (int8_t*)malloc(E ? E : 1);
    for (size_t i = 0; i < E; i++) q[i] = (int8_t)round(in[i] / sa);
    for (size_t n = 0; n < N; n++)
        for (size_t co = 0; co < Co; co++)
            for (size_t ho = 0; ho < Ho; ho++)
                for (size_t wo = 0; wo < Wo; wo++) {
                    int32_t acc = 0;
                    for (size_t ci = 0; ci < Ci; ci++)
                        for (size_t kh = 0; kh < Kh; kh++)
                            for (size_t kw = 0; kw < Kw; kw++) {
                                long ih = (long)(ho * stride) - (long)pad + (long)kh;
                                long iw = (long)(wo * stride) - (long)pad + (long)kw;
                                if (ih < 0 || iw < 0 || ih >= (long)H || iw >= (long)W) continue;
                                acc += (int32_t)q[((n * Ci + ci) * H + ih) * W + iw] *
                                       (int32_t)w[((co * Ci + ci) * Kh + kh) * Kw + kw];
                            }
                    double v = (double)acc * (sa * scale_w);
                    out[((n * Co + co) * Ho + ho) * Wo + wo] = relu && v < 0.0 ? 0.0 : v;
                }
    free(q);
}

/* ---- arena-mode graph executor: src/runtime/lancius_scheduler.c:61-362 ----- */

static size_t elems(const lancius_node* n) { return lancius_node_elements(n); }

static void run_node(const lancius_node* n, double* o, double** R) {
    size_t E = elems(n);
    const double* a = n->input_count > 0 ? R[n->inputs[0]->id] : NULL;
    const double* b = n->input_count > 1 ? R[n->inputs[1]->id] : NULL;
    const double* c = n->input_count > 2 ? R[n->inputs[2]->id] : NULL;
    const lancius_node* i0 = n->input_count > 0 ? n->inputs[0] : NULL;
    const lancius_node* i1 = n->input_count > 1 ? n->inputs[1] : NULL;
    switch (n->op) {
    case LANCIUS_OP_CONST: for (size_t e = 0; e < E; e++) o[e] = n->attr_val; break;      /* :330-342 */
    case LANCIUS_OP_ADD: for (size_t e = 0; e < E; e++) o[e] = a[e] + b[e]; break;       /* :169-189 */
    case LANCIUS_OP_SUB: for (size_t e = 0; e < E; e++) o[e] = a[e] - b[e]; break;       /* :241-245 */
    case LANCIUS_OP_MUL: for (size_t e = 0; e < E; e++) o[e] = a[e] * b[e]; break;       /* :236-240 */
    case LANCIUS_OP_RELU: for (size_t e = 0; e < E; e++) o[e] = a[e] > 0.0 ? a[e] : 0.0; break; /* :305-308 */
    case LANCIUS_OP_TANH: for (size_t e = 0; e < E; e++) o[e] = tanh(a[e]); break;
    case LANCIUS_OP_MATMUL:
        if (i1->runtime_data_int8 && i1->dtype == LANCIUS_DTYPE_INT8)
            orc_matmul_int8(o, a, i1->runtime_data_int8, i1->scale, i0->shape[0], i0->shape[1], i1->shape[1]);
        else
            orc_matmul(o, a, b, i0->shape[0], i0->shape[1], i1->shape[1]);
        break;
    case LANCIUS_OP_SOFTMAX: orc_softmax(o, a, n->shape[0], n->shape[1]); break;
    case LANCIUS_OP_SUM: { double s = 0.0; for (size_t e = 0; e < elems(i0); e++) s += a[e]; o[0] = s; } break;
    case LANCIUS_OP_SUM_AXIS0: {                                                          /* :257-262 */
        size_t Rr = i0->shape[0], C = i0->shape[1];
        for (size_t cc = 0; cc < C; cc++) o[cc] = 0.0;
        for (size_t r = 0; r < Rr; r++) for (size_t cc = 0; cc < C; cc++) o[cc] += a[r * C + cc];
    } break;
    case LANCIUS_OP_SUM_AXIS1: orc_sum_axis1(o, a, i0->shape[0], i0->shape[1]); break;
    case LANCIUS_OP_TRANSPOSE: {                                                          /* :246-250 */
        size_t Rr = i0->shape[0], C = i0->shape[1];
        for (size_t r = 0; r < Rr; r++) for (size_t cc = 0; cc < C; cc++) o[cc * Rr + r] = a[r * C + cc];
    } break;
    case LANCIUS_OP_BROADCAST:                                                           /* :268-278 */
        if (elems(i0) == 1) { for (size_t e = 0; e < E; e++) o[e] = a[0]; }
        else { for (size_t r = 0; r < n->shape[0]; r++) for (size_t cc = 0; cc < n->shape[1]; cc++) o[r * n->shape[1] + cc] = a[cc]; }
        break;
    case LANCIUS_OP_LAYERNORM: orc_layernorm(o, a, b, c, n->shape[0], n->shape[1], 1e-5); break; /* :109-115 */
    case LANCIUS_OP_GELU: orc_gelu(o, a, E); break;
    case LANCIUS_OP_RMSNORM: orc_rmsnorm(o, a, b, n->shape[0], n->shape[1], 1e-5); break;
    case LANCIUS_OP_SWIGLU: orc_swiglu(o, a, b, E); break;
    case LANCIUS_OP_GQA: orc_gqa(o, a, b, c, n->shape[0], n->kernel_h, n->kernel_w, n->shape[2]); break;
    case LANCIUS_OP_RELU_BWD: for (size_t e = 0; e < E; e++) o[e] = b[e] > 0.0 ? a[e] : 0.0; break;   /* :279-283 */
    case LANCIUS_OP_SOFTMAX_BWD: {                                                                    /* :295-304 */
        size_t Rr = n->shape[0], Cc = n->shape[1];
        for (size_t r = 0; r < Rr; r++) {
            double dot = 0.0;
            for (size_t cc = 0; cc < Cc; cc++) dot += a[r * Cc + cc] * b[r * Cc + cc];
            for (size_t cc = 0; cc < Cc; cc++) o[r * Cc + cc] = b[r * Cc + cc] * (a[r * Cc + cc] - dot);
        }
    } break;
    case LANCIUS_OP_CROSS_ENTROPY: {                                                                  /* :68-86 */
        size_t Rr = i0->shape[0], Cc = i0->shape[1];
        double tot = 0.0;
        for (size_t r = 0; r < Rr; r++) {
            double mx = a[r * Cc];
            for (size_t cc = 1; cc < Cc; cc++) if (a[r * Cc + cc] > mx) mx = a[r * Cc + cc];
            double se = 0.0;
            for (size_t cc = 0; cc < Cc; cc++) se += exp(a[r * Cc + cc] - mx);
            double lse = log(se) + mx;
            for (size_t cc = 0; cc < Cc; cc++) if (b[r * Cc + cc] == 1.0) tot -= a[r * Cc + cc] - lse;
        }
        o[0] = fabs(tot / (double)Rr);
    } break;
    case LANCIUS_OP_CROSS_ENTROPY_BWD: {                                                              /* :90-106 */
        size_t Rr = n->shape[0], Cc = n->shape[1];
        double sc = c[0] / (double)Rr;
        for (size_t r = 0; r < Rr; r++) {
            double mx = a[r * Cc];
            for (size_t cc = 1; cc < Cc; cc++) if (a[r * Cc + cc] > mx) mx = a[r * Cc + cc];
            double se = 0.0;
            for (size_t cc = 0; cc < Cc; cc++) se += exp(a[r * Cc + cc] - mx);
            for (size_t cc = 0; cc < Cc; cc++) o[r * Cc + cc] = (exp(a[r * Cc + cc] - mx) / se - b[r * Cc + cc]) * sc;
        }
    } break;
    case LANCIUS_OP_MAXPOOL2D_BWD: {
        const lancius_node* g0 = n->inputs[0];
        orc_maxpool2d_bwd(o, a, b, i1->shape[0], i1->shape[1], i1->shape[2], i1->shape[3], g0->shape[2], g0->shape[3],
                          n->kernel_h, n->stride);
    } break;
    case LANCIUS_OP_CONV2D_BWD: {                                                                      /* vision_ops.c:126-137 */
        const lancius_node* wn = n->inputs[2];
        orc_conv2d_bwd_in(o, a, c, i1->shape[0], i1->shape[1], i1->shape[2], i1->shape[3], wn->shape[0], i0->shape[2],
                          i0->shape[3], wn->shape[2], wn->shape[3], n->stride, n->pad);
    } break;
    case LANCIUS_OP_CONV2D_BWD_W:                                                                      /* vision_ops.c:138-148 */
        orc_conv2d_bwd_w(o, a, b, i1->shape[0], i1->shape[1], i1->shape[2], i1->shape[3], n->shape[0], i0->shape[2],
                         i0->shape[3], n->shape[2], n->shape[3], n->stride, n->pad);
        break;
    case LANCIUS_OP_ATTENTION: orc_attention(o, a, b, c, n->shape[0], n->shape[1], n->shape[2], n->attr_val != 1.0); break;
    case LANCIUS_OP_CONV2D: case LANCIUS_OP_CONV2D_RELU_FUSED:                           /* vision_ops.c:60-81 */
        if (i1->runtime_data_int8 && i1->dtype == LANCIUS_DTYPE_INT8) {
            orc_conv2d_int8(o, a, i1->runtime_data_int8, i1->scale, i0->shape[0], i0->shape[1], i0->shape[2],
                            i0->shape[3], i1->shape[0], i1->shape[2], i1->shape[3], n->stride, n->pad,
                            n->op == LANCIUS_OP_CONV2D_RELU_FUSED);
            break;
        }
        orc_conv2d(o, a, b, i0->shape[0], i0->shape[1], i0->shape[2], i0->shape[3], i1->shape[0],
                   i1->shape[2], i1->shape[3], n->stride, n->pad, n->op == LANCIUS_OP_CONV2D_RELU_FUSED);
        break;
    case LANCIUS_OP_MAXPOOL2D:
        orc_maxpool2d(o, a, i0->shape[0], i0->shape[1], i0->shape[2], i0->shape[3], n->kernel_h, n->stride);
        break;
    case LANCIUS_OP_FLATTEN: case LANCIUS_OP_RESHAPE: memcpy(o, a, E * sizeof(double)); break; /* vision_ops.c:113-125 */
    default: for (size_t e = 0; e < E; e++) o[e] = NAN; break;
    }
}

double** orc_run_graph(const lancius_graph* g) {
    double** R = (double**)calloc(g->next_id, sizeof(double*));
    unsigned char* done = (unsigned char*)calloc(g->next_id, 1);
    uint32_t left = g->node_count;
    /* inputs-before-consumers order (same data dependencies as the wave order) */
    while (left) {
        uint32_t progressed = 0;
        for (uint32_t i = 0; i < g->node_count; i++) {
            const lancius_node* n = g->nodes[i];
            if (done[n->id]) continue;
            int ready = 1;
            for (uint32_t j = 0; j < n->input_count; j++) ready &= done[n->inputs[j]->id];
            if (!ready) continue;
            if (n->op == LANCIUS_OP_INPUT) R[n->id] = n->runtime_data;
            else if (n->op != LANCIUS_OP_NOP) {
                R[n->id] = (double*)malloc((elems(n) ? elems(n) : 1) * sizeof(double));
                run_node(n, R[n->id], R);
            }
            done[n->id] = 1; left--; progressed++;
        }
        if (!progressed) break;
    }
    free(done);
    return R;
}

void orc_free_results(const lancius_graph* g, double** R) {
    if (!R) return;
    for (uint32_t i = 0; i < g->node_count; i++) {
        const lancius_node* n = g->nodes[i];
        if (n->op != LANCIUS_OP_INPUT) free(R[n->id]);
    }
    free(R);
}

