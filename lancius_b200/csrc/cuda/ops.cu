// Per-op C ABI (lancius_cuda.h): argument checks and kernel selection.
#include "lcu_internal.h"
#include <string.h>
#include <stdlib.h>

static thread_local int tl_launches = 0;
extern "C" void lcu_note_launch(void) { tl_launches++; }

static thread_local int tl_cuda_error = 0;
extern "C" void lcu_note_cuda_error(int e) { tl_cuda_error = e; }
extern "C" const char* lcu_last_cuda_error(void) {
    return tl_cuda_error ? cudaGetErrorString((cudaError_t)tl_cuda_error) : "no error";
}
extern "C" void lcu_reset_launch_count(void) { tl_launches = 0; }
extern "C" int lcu_launch_count(void) { return tl_launches; }

// Tensor-core path from 2^24 multiply-adds up (below that the CUDA-core kernel's
// single launch beats split + GEMM); LCU_FORCE_SIMT=1 / LCU_FORCE_TC=1 override.
static int force_mode() {
    static int force = -1;
    if (force < 0) {
        const char* s = getenv("LCU_FORCE_SIMT");
        const char* t = getenv("LCU_FORCE_TC");
        force = (s && s[0] == '1') ? 0 : (t && t[0] == '1') ? 1 : 2;
    }
    return force;
}
extern "C" int lcu_force_simt(void) { return force_mode() == 0; }
// LCU_FORCE_TC=1 also sends short-reduction convs to the tensor cores (tests)
extern "C" int lcu_force_tc_conv(void) { return force_mode() == 1; }
// LCU_NO_WEIGHT_CACHE=1: split MATMUL weights into TF32 hi/lo on every run instead of once
// per upload (read at each bind, so tests can compare both paths in one process)
extern "C" int lcu_no_weight_cache(void) {
    const char* e = getenv("LCU_NO_WEIGHT_CACHE");
    return e && e[0] == '1';
}
// LCU_NO_RAW_A=1: split tensor-core GEMM A operands in a separate pass (read at each bind)
extern "C" int lcu_no_raw_a(void) {
    const char* e = getenv("LCU_NO_RAW_A");
    return e && e[0] == '1';
}
extern "C" int lcu_conv_force_im2col(void) {
    static int f = -1;
    if (f < 0) { const char* e = getenv("LCU_CONV_IM2COL"); f = e && e[0] == '1'; }
    return f;
}
extern "C" int lcu_use_tensor_cores(size_t M, size_t N, size_t K) {
    int force = force_mode();
    if (force != 2) return force && K > 0;
    return K > 0 && (double)M * (double)N * (double)K >= 16777216.0;
}

static lancius_error bad(lancius_error e) { lancius_set_error(e); return e; }

extern "C" {

lancius_error lcu_matmul(float* out, const float* a, const float* b, size_t M, size_t K, size_t N, const float* bias,
                         int epilogue, int mode, void* stream) {
    if (!out || (K && (!a || !b))) return bad(LANCIUS_ERROR_NULL_PTR);
    if (epilogue < LCU_EPI_NONE || epilogue > LCU_EPI_GELU) return bad(LANCIUS_ERROR_UNSUPPORTED_OP);
    if (mode != LCU_MODE_FP32_EXACT && mode != LCU_MODE_TF32 && mode != LCU_MODE_BF16) return bad(LANCIUS_ERROR_UNSUPPORTED_DTYPE);
    if (M == 0 || N == 0) return LANCIUS_ERROR_OK;
    // K == 0 is valid: the product is zero, bias and epilogue still apply
    if (lcu_use_tensor_cores(M, N, K)) return lcu_gemm_tc(out, a, b, M, K, N, bias, epilogue, mode, stream);
    return lcu_gemm_simt(out, a, b, M, K, N, bias, epilogue, stream);
}

lancius_error lcu_attention(float* out, const float* q, const float* k, const float* v, size_t B, size_t S, size_t H,
                            size_t D, int causal, int mode, void* stream) {
    if (!out || !q || !k || !v) return bad(LANCIUS_ERROR_NULL_PTR);
    if (mode != LCU_MODE_FP32_EXACT && mode != LCU_MODE_TF32 && mode != LCU_MODE_BF16) return bad(LANCIUS_ERROR_UNSUPPORTED_DTYPE);
    if (D != 64 && D != 128) return bad(LANCIUS_ERROR_UNSUPPORTED_OP);
    if ((((uintptr_t)q | (uintptr_t)k | (uintptr_t)v | (uintptr_t)out) & 15u)) return bad(LANCIUS_ERROR_UNSUPPORTED_DTYPE);
    if (lcu_attention_tc_supported(D) && !lcu_force_simt())
        return lcu_attention_tc(nullptr, q, k, v, out, B, S, H, causal ? 1 : 0, lcu_contraction_mode(mode), nullptr,
                                nullptr, stream);
    return lcu_attention_simt(nullptr, q, k, v, out, B, S, H, D, causal ? 1 : 0, stream);
}

lancius_error lcu_conv2d(float* out, const float* in, const float* w, size_t N, size_t C_in, size_t H_in, size_t W_in,
                         size_t C_out, size_t K_h, size_t K_w, size_t stride, size_t pad, int relu, int mode,
                         void* stream) {
    if (!out || !in || !w) return bad(LANCIUS_ERROR_NULL_PTR);
    if (mode != LCU_MODE_FP32_EXACT && mode != LCU_MODE_TF32 && mode != LCU_MODE_BF16) return bad(LANCIUS_ERROR_UNSUPPORTED_DTYPE);
    if (stride == 0 || H_in + 2 * pad < K_h || W_in + 2 * pad < K_w) return bad(LANCIUS_ERROR_SHAPE_MISMATCH);
    size_t Ho = (H_in + 2 * pad - K_h) / stride + 1, Wo = (W_in + 2 * pad - K_w) / stride + 1;
    mode = lcu_contraction_mode(mode);   // no BF16 conv: one TF32 pass
    if (lcu_conv_smallk_supported(C_in, K_h, K_w, C_out) && !lcu_force_tc_conv())
        return lcu_conv2d_smallk(out, in, w, N, C_in, H_in, W_in, C_out, K_h, K_w, stride, pad, relu, stream);
    if (N && C_in && lcu_use_tensor_cores(C_out, N * Ho * Wo, C_in * K_h * K_w)) {
        LcuConvShape cs{(int)N, (int)C_in, (int)H_in, (int)W_in, (int)C_out, (int)K_h, (int)K_w, (int)stride, (int)pad,
                        (int)Ho, (int)Wo};
        if (lcu_conv_nhwc_supported(cs) && !lcu_conv_force_im2col()) {
            void* scratch = lcu_scratch_acquire(lcu_conv_nhwc_scratch_bytes(cs, mode == LCU_MODE_TF32 ? 1 : 3));
            if (!scratch) return bad(LANCIUS_ERROR_OOM);
            lancius_error e = lcu_conv2d_tc_nhwc(out, in, w, cs, relu, mode, scratch, stream);
            // the per-device scratch is reused by the next call
            if (e == LANCIUS_ERROR_OK) e = lcu_check_stream(stream);
            return e;
        }
        return lcu_conv2d_tc(out, in, w, cs, relu, mode, stream);
    }
    return lcu_conv2d_simt(out, in, w, N, C_in, H_in, W_in, C_out, K_h, K_w, stride, pad, relu, stream);
}

const char* lcu_build_info(void) {
    return "lancius_b200 sm_100a: gemm_tcgen05_3xtf32 attention_tcgen05_3xtf32 conv_tcgen05_3xtf32 gemm_simt conv_simt attention_simt layernorm softmax sum_axis1 maxpool eltwise";
}

}  // extern "C"
