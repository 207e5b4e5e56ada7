/*
 * lancius_cuda.h -- C ABI of the B200 (sm_100a) execution backend for Lancius.
 *
 * Replaces, below the unchanged IR / scheduler / memory-plan contract, the
 * reference's CPU math:
 *   execute_node_math()             bleeding/v11A1/src/runtime/lancius_scheduler.c:61-309
 *   lancius_schedule_execute()      bleeding/v11A1/src/runtime/lancius_scheduler.c:311-362
 *   lancius_execute_vision_op()     bleeding/v11A1/src/runtime/lancius_vision_ops.c:10-191
 *   kernel_*()                      bleeding/v11A1/include/lancius/lancius_kernels.h:14-50
 *
 * Plain C types only (no CUDA or torch types): streams are passed as void*
 * (a cudaStream_t, NULL = the context's stream for ctx calls / the legacy default
 * stream for per-op calls); device buffers are float* device pointers.
 * Every call reports failure through lancius_set_error() and its return value;
 * nothing aborts. All device math is FP32 storage with one of the precision
 * modes below.
 */
#ifndef LANCIUS_CUDA_H
#define LANCIUS_CUDA_H

#include "lancius/lancius_ir.h"
#include "lancius/lancius_scheduler.h"
#include "lancius/lancius_memory_planner.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Contraction precision (GEMM, conv, attention).
 *  FP32_EXACT: 3xTF32 split on tcgen05 (a_hi*b_hi + a_hi*b_lo + a_lo*b_hi), FP32
 *              accumulate; parity bar normwise rel 1e-4 vs the FP64 reference.
 *  TF32:       one tcgen05 kind::tf32 pass; parity bar 2e-2.
 *  BF16:       tensor-core GEMMs (lcu_matmul, graph MATMULs) on BF16 copies of both
 *              operands (round to nearest even), tcgen05 kind::f16, FP32 accumulate;
 *              conv and attention run the TF32 pass; parity bar 2e-2. The column-split
 *              and allocation-free GEMMs take FP32_EXACT and TF32 only.              */
typedef enum { LCU_MODE_FP32_EXACT = 0, LCU_MODE_TF32 = 1, LCU_MODE_BF16 = 2 } lcu_mode;

/* Epilogue fused into GEMM / conv stores. */
typedef enum { LCU_EPI_NONE = 0, LCU_EPI_RELU = 1, LCU_EPI_GELU = 2 } lcu_epilogue;

typedef struct lcu_ctx lcu_ctx;

/* ---- context: one per GPU, one host thread drives it ------------------- */
lcu_ctx* lcu_create(int device);
void lcu_destroy(lcu_ctx* ctx);
lancius_error lcu_set_mode(lcu_ctx* ctx, lcu_mode mode);
void* lcu_stream(lcu_ctx* ctx);                 /* the context's cudaStream_t */
lancius_error lcu_synchronize(lcu_ctx* ctx);     /* also reports device watchdog flags */
/* Waits for a stream (NULL = legacy default) and reports a tensor-core watchdog trip
 * (a bounded mbarrier wait that gave up) as LANCIUS_ERROR_INTERNAL, clearing it. The
 * per-op launchers that return before the work is done (lcu_attention, lcu_layernorm
 * ...) report trips here; the blocking ones (lcu_matmul, lcu_conv2d, the INT8 and
 * column-split GEMMs, lcu_matmul_noalloc) check before they return. */
lancius_error lcu_check_stream(void* stream);
/* Test hook (no reference counterpart): launches a kernel whose bounded wait on an
 * mbarrier nothing arrives on gives up and sets the GEMM watchdog word, so the next
 * lcu_synchronize returns LANCIUS_ERROR_INTERNAL (and clears the word). */
lancius_error lcu_watchdog_selftest(void* stream);

/* ---- graph binding: the memory plan's offsets map onto one device allocation.
 * plan == NULL: the backend plans the FP32 device pool itself
 * (lancius_build_memory_plan_ex(sched, g, 4, 256, 1)). A caller-supplied plan is
 * validated first (lancius_memory_plan_validate with 4-byte elements) and
 * rejected with LANCIUS_ERROR_INVALID_MODEL when live tensors would overlap.
 * INPUT and CONST nodes get their own persistent slots after the pool.        */
lancius_error lcu_bind_plan(lcu_ctx* ctx, lancius_schedule* sched, lancius_graph* g,
                            const lancius_memory_plan* plan);

/* Host <-> device copies of one node's slot. host_dtype is LANCIUS_DTYPE_FP64
 * (reference-style double buffers, converted on the device), FP32, or INT8 for
 * quantized weights (bytes, uploaded as they are). */
lancius_error lcu_upload(lcu_ctx* ctx, const lancius_node* n, const void* host, lancius_dtype host_dtype);
lancius_error lcu_download(lcu_ctx* ctx, const lancius_node* n, void* host, lancius_dtype host_dtype);
/* FP32 download queued on the context's stream without waiting (complete after
 * lcu_synchronize); for pipelining requests over two contexts. The reference has no
 * device copies, so no counterpart. */
lancius_error lcu_download_async(lcu_ctx* ctx, const lancius_node* n, void* host);
/* Uploads every INPUT node whose runtime_data (FP64) is bound on the host. */
lancius_error lcu_upload_bound_inputs(lcu_ctx* ctx);
float* lcu_node_device_ptr(lcu_ctx* ctx, const lancius_node* n);
/* Tensor-core MATMULs whose weights are INPUT nodes read TF32 hi/lo copies made once
 * per lcu_upload of the weight (not per run). After writing a weight slot through
 * lcu_node_device_ptr, call this to remake the copies. No reference counterpart:
 * the reference's CPU kernels read the FP64 weights directly. */
lancius_error lcu_refresh_weights(lcu_ctx* ctx);

/* Runs every wave of the bound schedule on the context's stream (asynchronous;
 * lcu_synchronize() or a download waits). Same shape as the reference's
 * lancius_schedule_execute(schedule, scratch): the second argument is the
 * device context instead of a host arena. Errors: lancius_get_error(). */
void lancius_schedule_execute_cuda(lancius_schedule* sched, lcu_ctx* ctx);
/* Text of the last CUDA status this thread turned into LANCIUS_ERROR_INTERNAL/OOM
 * ("no error" if none); a diagnostic companion of lancius_get_error(). */
const char* lcu_last_cuda_error(void);
/* Number of kernels the last lancius_schedule_execute_cuda call launched. */
int lcu_last_launch_count(lcu_ctx* ctx);
/* 1 = replay the schedule through a captured CUDA graph after the first run. */
lancius_error lcu_set_graph_replay(lcu_ctx* ctx, int enable);
/* 1 (default) = fold MATMUL -> ADD(BROADCAST bias) -> RELU|GELU -> ADD(residual)
 * chains into one GEMM epilogue when the backend plans memory itself. Nodes inside
 * a folded chain share the chain's output slot (a download returns the chain's
 * final value); a BROADCAST read only by a folded ADD is never materialised.
 * Takes effect at the next lcu_bind_plan. */
lancius_error lcu_set_fusion(lcu_ctx* ctx, int enable);

/* Page-locked host buffers for fast lcu_upload / lcu_download. */
void* lcu_host_alloc(size_t bytes);
void lcu_host_free(void* p);

/* ---- per-op launchers: argument order mirrors the reference kernel_* ------ */
/* C[M,N] = A[M,K] * B[K,N] (+ bias[N]) (epilogue); row-major.
 * Mirrors kernel_matmul (lancius_kernels.c:15-26) / executor MATMUL (scheduler.c:190-235). */
lancius_error lcu_matmul(float* out, const float* a, const float* b, size_t M, size_t K, size_t N,
                         const float* bias, int epilogue, int mode, void* stream);
/* Causal (causal=1, kernel_attention lancius_kernels.c:278-332) or unmasked
 * attention over B independent [S, H, D] blocks (heads concatenated). */
lancius_error lcu_attention(float* out, const float* q, const float* k, const float* v,
                            size_t B, size_t S, size_t H, size_t D, int causal, int mode, void* stream);
/* NCHW input, OIHW weights, zero padding (kernel_conv2d_fwd / kernel_conv2d_relu_fwd,
 * lancius_kernels.c:28-60,140-173). relu = 1 applies ReLU in the store. */
lancius_error lcu_conv2d(float* out, const float* in, const float* w, size_t N, size_t C_in,
                         size_t H_in, size_t W_in, size_t C_out, size_t K_h, size_t K_w,
                         size_t stride, size_t pad, int relu, int mode, void* stream);
/* kernel_layernorm (lancius_kernels.c:217-236): biased variance, eps. */
lancius_error lcu_layernorm(float* out, const float* in, const float* gamma, const float* beta,
                            size_t rows, size_t hidden, float eps, void* stream);
lancius_error lcu_softmax(float* out, const float* in, size_t rows, size_t cols, void* stream);
lancius_error lcu_gelu(float* out, const float* in, size_t n, void* stream);
lancius_error lcu_tanh(float* out, const float* in, size_t n, void* stream);
lancius_error lcu_relu(float* out, const float* in, size_t n, void* stream);
lancius_error lcu_add(float* out, const float* a, const float* b, size_t n, void* stream);
lancius_error lcu_sub(float* out, const float* a, const float* b, size_t n, void* stream);
lancius_error lcu_mul(float* out, const float* a, const float* b, size_t n, void* stream);
/* BROADCAST (scheduler.c:268-278): in_elems == 1 fills; else row vector -> [rows, cols]. */
lancius_error lcu_broadcast(float* out, const float* in, size_t in_elems, size_t rows, size_t cols, void* stream);
lancius_error lcu_fill(float* out, float value, size_t n, void* stream);
lancius_error lcu_sum_axis1(float* out, const float* in, size_t rows, size_t cols, void* stream);
lancius_error lcu_maxpool2d(float* out, const float* in, size_t N, size_t C, size_t H_in, size_t W_in,
                            size_t K, size_t stride, void* stream);

/* ---- multi-GPU: column-split GEMM with an NCCL all-gather over NVLink -------
 * No counterpart in the reference (CPU only, distributed execution deferred,
 * KNOWN_LIMITATIONS.md:24); used to split a large square product (16384^3) by columns.
 * One process (or thread) per GPU. Rank 0 creates the id and shares its 128 bytes
 * with the others out of band (torch.distributed, a file, MPI ...). */
typedef struct lcu_comm lcu_comm;
lancius_error lcu_comm_unique_id(void* out, size_t bytes);            /* bytes >= 128 */
lcu_comm* lcu_comm_create(int nranks, int rank, const void* unique_id, int device);
void lcu_comm_destroy(lcu_comm* comm);
void lcu_comm_abort(lcu_comm* comm);      /* failure path: peers gone; never blocks */
int lcu_comm_size(const lcu_comm* comm);
/* C [M, N] on every rank = A [M, K] * [B_0 | B_1 | ...]; this rank passes its slab
 * b_slab [K, N / nranks]. N % nranks == 0. */
lancius_error lcu_gemm_colsplit(lcu_comm* comm, float* c, const float* a, const float* b_slab, size_t M, size_t K,
                                size_t N, int mode, void* stream);
/* Same result, compute and exchange fused: this rank's GEMM epilogue stores its finished
 * tiles into every rank's C over NVLink (C opened on each rank through CUDA IPC on the
 * first call with a given C; that call is collective), then a 4-byte NCCL all-gather acts
 * as the barrier. C must be 16-byte aligned device memory from cudaMalloc (or a pool on
 * top of it); nranks <= 8. Returns after the stream has drained. */
lancius_error lcu_gemm_colsplit_fused(lcu_comm* comm, float* c, const float* a, const float* b_slab, size_t M,
                                      size_t K, size_t N, int mode, void* stream);

/* lcu_matmul without device allocation (no counterpart in the reference, whose
 * kernels run on the host). For callers that may not call cudaMalloc once they are
 * running -- device memory owned by another allocator or a fixed memory budget.
 * Same arguments and results as lcu_matmul (tensor-core path, M, N, K >= 1); its
 * scratch is a 64 MiB array compiled into the library, one per GPU, kept until
 * exit: problems needing more (lcu_gemm_tc scratch ~ 16*(M*K+K*N) bytes in
 * FP32-exact mode) return LANCIUS_ERROR_OVERFLOW. All calls on a GPU share the
 * array, so calls that overlap on the GPU race; serialize them. The first call on
 * each device looks up the array's address; make it before any stream capture.
 * With CUDA's default lazy module loading the GPU reserves the array at that first
 * lookup (which can fail with LANCIUS_ERROR_OOM); with CUDA_MODULE_LOADING=EAGER at
 * context creation. Blocks until the product is written; a tensor-core watchdog
 * trip is reported as LANCIUS_ERROR_INTERNAL. */
lancius_error lcu_matmul_noalloc(float* out, const float* a, const float* b, size_t M, size_t K, size_t N,
                                 const float* bias, int epilogue, int mode, void* stream);
size_t lcu_noalloc_scratch_capacity(void);
/* Looks up (and so reserves) the array on the current device without computing:
 * call it once per GPU at start-up, before any stream capture. */
lancius_error lcu_noalloc_prepare(void);

/* ---- training, LLM and INT8 operators (the reference's kernels beyond inference) */
lancius_error lcu_sum(float* out, const float* a, size_t n, void* stream);                       /* scheduler.c:251-256 */
lancius_error lcu_sum_axis0(float* out, const float* a, size_t rows, size_t cols, void* stream); /* :257-262 */
lancius_error lcu_transpose(float* out, const float* a, size_t rows, size_t cols, void* stream); /* :246-250 */
lancius_error lcu_relu_bwd(float* out, const float* grad, const float* fwd, size_t n, void* stream); /* :279-283 */
lancius_error lcu_softmax_bwd(float* out, const float* dy, const float* y, size_t rows, size_t cols, void* stream); /* :295-304 */
lancius_error lcu_cross_entropy(float* out, const float* logits, const float* targets, size_t rows, size_t cols,
                                void* stream);                                                   /* :68-86 */
lancius_error lcu_cross_entropy_bwd(float* out, const float* logits, const float* targets, const float* grad_out,
                                    size_t rows, size_t cols, void* stream);                     /* :90-106 */
lancius_error lcu_rmsnorm(float* out, const float* in, const float* gamma, size_t rows, size_t hidden, float eps,
                          void* stream);                                                         /* lancius_kernels.c:381-396 */
lancius_error lcu_swiglu(float* out, const float* gate, const float* up, size_t n, void* stream); /* :398-405 */
lancius_error lcu_rope(float* q, float* k, size_t B, size_t S, size_t H, size_t D, int pos_offset, void* stream); /* :248-272 */
lancius_error lcu_gqa(float* out, const float* q, const float* k, const float* v, size_t S, size_t Hq, size_t Hkv,
                      size_t D, void* stream);                                                   /* :407-448 */
/* KV-cache decode attention, lancius_kernels.c:338-379 (kernel_attention_kv_cache):
 * out[H*D] = softmax(q . K^T / sqrt(D)) V over all seq_len cached rows; caches
 * [seq_len][H][D], q and out [H*D]. head_dim <= 256. The batched form takes B
 * sequences at once: q, out [B][H*D], caches [B][seq_len][H][D]. */
lancius_error lcu_attention_kv_cache(float* out, const float* q, const float* k_cache, const float* v_cache,
                                     size_t seq_len, size_t n_heads, size_t head_dim, void* stream);
lancius_error lcu_attention_kv_cache_batched(float* out, const float* q, const float* k_cache, const float* v_cache,
                                             size_t batch, size_t seq_len, size_t n_heads, size_t head_dim,
                                             void* stream);
lancius_error lcu_maxpool2d_bwd(float* out, const float* grad, const float* in, size_t N, size_t C, size_t H, size_t W,
                                size_t K, size_t stride, void* stream);                          /* vision_ops.c:149-190 */
lancius_error lcu_conv2d_bwd(float* out, const float* grad, const float* w, size_t N, size_t C_in, size_t H, size_t W,
                             size_t C_out, size_t H_out, size_t W_out, size_t K_h, size_t K_w, size_t stride, size_t pad,
                             void* stream);                                                      /* lancius_kernels.c:62-91 */
lancius_error lcu_conv2d_bwd_w(float* out, const float* grad, const float* in, size_t N, size_t C_in, size_t H, size_t W,
                               size_t C_out, size_t H_out, size_t W_out, size_t K_h, size_t K_w, size_t stride,
                               size_t pad, void* stream);                                        /* :93-136 */

/* Library self-description for tests: the names of this build's kernels. */
const char* lcu_build_info(void);

#ifdef __cplusplus
}
#endif
#endif
