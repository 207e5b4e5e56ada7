// HBM-bound elementwise kernels: 128-bit (float4) grid-stride loops when every
// pointer is 16-byte aligned, a scalar loop otherwise. Grids are capped at a
// multiple of the SM count; each thread streams several float4s.
#include "lcu_internal.h"

namespace {

enum BinOp { OP_ADD, OP_SUB, OP_MUL };
enum UnOp { OP_RELU, OP_GELU, OP_TANH, OP_COPY };

template <int OPK>
__device__ __forceinline__ float bin(float a, float b) {
    return OPK == OP_ADD ? a + b : OPK == OP_SUB ? a - b : a * b;
}
template <int OPK>
__device__ __forceinline__ float un(float a) {
    return OPK == OP_RELU ? (a > 0.f ? a : 0.f) : OPK == OP_GELU ? lcu_gelu_f(a) : OPK == OP_TANH ? tanhf(a) : a;
}

template <int OPK>
__global__ void k_binary_v4(const LcuEltGroup* __restrict__ table, LcuEltGroup g, size_t n4) {
    if (table) g = table[blockIdx.y];
    float4* __restrict__ o = (float4*)g.out;
    const float4* __restrict__ a = (const float4*)g.a;
    const float4* __restrict__ b = (const float4*)g.b;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n4; i += (size_t)gridDim.x * blockDim.x) {
        float4 x = a[i], y = b[i];
        o[i] = make_float4(bin<OPK>(x.x, y.x), bin<OPK>(x.y, y.y), bin<OPK>(x.z, y.z), bin<OPK>(x.w, y.w));
    }
}
template <int OPK>
__global__ void k_binary(const LcuEltGroup* __restrict__ table, LcuEltGroup g, size_t n) {
    if (table) g = table[blockIdx.y];
    float* __restrict__ o = g.out;
    const float* __restrict__ a = g.a;
    const float* __restrict__ b = g.b;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        o[i] = bin<OPK>(a[i], b[i]);
}
template <int OPK>
__global__ void k_unary_v4(const LcuEltGroup* __restrict__ table, LcuEltGroup g, size_t n4) {
    if (table) g = table[blockIdx.y];
    float4* __restrict__ o = (float4*)g.out;
    const float4* __restrict__ a = (const float4*)g.a;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n4; i += (size_t)gridDim.x * blockDim.x) {
        float4 x = a[i];
        o[i] = make_float4(un<OPK>(x.x), un<OPK>(x.y), un<OPK>(x.z), un<OPK>(x.w));
    }
}
template <int OPK>
__global__ void k_unary(const LcuEltGroup* __restrict__ table, LcuEltGroup g, size_t n) {
    if (table) g = table[blockIdx.y];
    float* __restrict__ o = g.out;
    const float* __restrict__ a = g.a;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        o[i] = un<OPK>(a[i]);
}

__global__ void k_fill(float* __restrict__ o, float v, size_t n) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) o[i] = v;
}
// row vector [cols] -> [rows, cols]  (scheduler.c:275-277)
__global__ void k_broadcast_rows(float* __restrict__ o, const float* __restrict__ v, size_t rows, size_t cols) {
    size_t n = rows * cols;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        o[i] = v[i % cols];
}
__global__ void k_broadcast_scalar(float* __restrict__ o, const float* __restrict__ v, size_t n) {
    float s = v[0];
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) o[i] = s;
}
__global__ void k_f64_to_f32(float* __restrict__ o, const double* __restrict__ a, size_t n) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        o[i] = (float)a[i];
}
__global__ void k_f32_to_f64(double* __restrict__ o, const float* __restrict__ a, size_t n) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        o[i] = (double)a[i];
}

inline bool aligned16(const void* p) { return ((uintptr_t)p & 15u) == 0; }

// table != NULL: `count` groups of n elements each (grid.y = group); every pointer
// in a table built by the executor is 256-byte aligned, so `vec` is decided once.
template <int OPK>
lancius_error launch_binary(const LcuEltGroup* table, int count, LcuEltGroup g, size_t n, bool vec, void* s) {
    if (n == 0 || count <= 0) return LANCIUS_ERROR_OK;
    cudaStream_t st = lcu_as_stream(s);
    unsigned cap = table ? 148u * 4u : 148u * 16u;
    dim3 grid(vec ? lcu_blocks(n / 4, 256 * 4, cap) : lcu_blocks(n, 256 * 4, cap), (unsigned)count);
    if (vec) k_binary_v4<OPK><<<grid, 256, 0, st>>>(table, g, n / 4);
    else k_binary<OPK><<<grid, 256, 0, st>>>(table, g, n);
    lcu_note_launch();
    return lcu_launch_status();
}
template <int OPK>
lancius_error launch_unary(const LcuEltGroup* table, int count, LcuEltGroup g, size_t n, bool vec, void* s) {
    if (n == 0 || count <= 0) return LANCIUS_ERROR_OK;
    cudaStream_t st = lcu_as_stream(s);
    unsigned cap = table ? 148u * 4u : 148u * 16u;
    dim3 grid(vec ? lcu_blocks(n / 4, 256 * 4, cap) : lcu_blocks(n, 256 * 4, cap), (unsigned)count);
    if (vec) k_unary_v4<OPK><<<grid, 256, 0, st>>>(table, g, n / 4);
    else k_unary<OPK><<<grid, 256, 0, st>>>(table, g, n);
    lcu_note_launch();
    return lcu_launch_status();
}
template <int OPK>
lancius_error one_binary(float* o, const float* a, const float* b, size_t n, void* s) {
    if (!o || !a || !b) { lancius_set_error(LANCIUS_ERROR_NULL_PTR); return LANCIUS_ERROR_NULL_PTR; }
    bool vec = aligned16(o) && aligned16(a) && aligned16(b) && n % 4 == 0;
    return launch_binary<OPK>(nullptr, 1, LcuEltGroup{o, a, b}, n, vec, s);
}
template <int OPK>
lancius_error one_unary(float* o, const float* a, size_t n, void* s) {
    if (!o || !a) { lancius_set_error(LANCIUS_ERROR_NULL_PTR); return LANCIUS_ERROR_NULL_PTR; }
    bool vec = aligned16(o) && aligned16(a) && n % 4 == 0;
    return launch_unary<OPK>(nullptr, 1, LcuEltGroup{o, a, nullptr}, n, vec, s);
}

}  // namespace

extern "C" {

lancius_error lcu_add(float* o, const float* a, const float* b, size_t n, void* s) { return one_binary<OP_ADD>(o, a, b, n, s); }
lancius_error lcu_sub(float* o, const float* a, const float* b, size_t n, void* s) { return one_binary<OP_SUB>(o, a, b, n, s); }
lancius_error lcu_mul(float* o, const float* a, const float* b, size_t n, void* s) { return one_binary<OP_MUL>(o, a, b, n, s); }
lancius_error lcu_relu(float* o, const float* a, size_t n, void* s) { return one_unary<OP_RELU>(o, a, n, s); }
lancius_error lcu_gelu(float* o, const float* a, size_t n, void* s) { return one_unary<OP_GELU>(o, a, n, s); }
lancius_error lcu_tanh(float* o, const float* a, size_t n, void* s) { return one_unary<OP_TANH>(o, a, n, s); }
lancius_error lcu_copy_f32(float* o, const float* a, size_t n, void* s) { return one_unary<OP_COPY>(o, a, n, s); }

// Executor entry: one launch over `count` same-sized groups from a device table.
// op: 0 add, 1 sub, 2 mul, 3 relu, 4 gelu, 5 tanh, 6 copy.
lancius_error lcu_eltwise_grouped(int op, const LcuEltGroup* d_table, int count, size_t n, int vec, void* s) {
    LcuEltGroup none{nullptr, nullptr, nullptr};
    switch (op) {
        case 0: return launch_binary<OP_ADD>(d_table, count, none, n, vec, s);
        case 1: return launch_binary<OP_SUB>(d_table, count, none, n, vec, s);
        case 2: return launch_binary<OP_MUL>(d_table, count, none, n, vec, s);
        case 3: return launch_unary<OP_RELU>(d_table, count, none, n, vec, s);
        case 4: return launch_unary<OP_GELU>(d_table, count, none, n, vec, s);
        case 5: return launch_unary<OP_TANH>(d_table, count, none, n, vec, s);
        case 6: return launch_unary<OP_COPY>(d_table, count, none, n, vec, s);
        default: lancius_set_error(LANCIUS_ERROR_UNSUPPORTED_OP); return LANCIUS_ERROR_UNSUPPORTED_OP;
    }
}

lancius_error lcu_fill(float* o, float v, size_t n, void* s) {
    if (!o) { lancius_set_error(LANCIUS_ERROR_NULL_PTR); return LANCIUS_ERROR_NULL_PTR; }
    if (n == 0) return LANCIUS_ERROR_OK;
    k_fill<<<lcu_blocks(n, 256 * 4), 256, 0, lcu_as_stream(s)>>>(o, v, n);
    lcu_note_launch();
    return lcu_launch_status();
}

lancius_error lcu_broadcast(float* o, const float* in, size_t in_elems, size_t rows, size_t cols, void* s) {
    if (!o || !in) { lancius_set_error(LANCIUS_ERROR_NULL_PTR); return LANCIUS_ERROR_NULL_PTR; }
    if (rows * cols == 0) return LANCIUS_ERROR_OK;
    if (in_elems == 1)
        k_broadcast_scalar<<<lcu_blocks(rows * cols, 1024), 256, 0, lcu_as_stream(s)>>>(o, in, rows * cols);
    else
        k_broadcast_rows<<<lcu_blocks(rows * cols, 1024), 256, 0, lcu_as_stream(s)>>>(o, in, rows, cols);
    lcu_note_launch();
    return lcu_launch_status();
}

lancius_error lcu_convert_f64_to_f32(float* o, const double* a, size_t n, void* s) {
    if (n == 0) return LANCIUS_ERROR_OK;
    k_f64_to_f32<<<lcu_blocks(n, 1024), 256, 0, lcu_as_stream(s)>>>(o, a, n);
    lcu_note_launch();
    return lcu_launch_status();
}
lancius_error lcu_convert_f32_to_f64(double* o, const float* a, size_t n, void* s) {
    if (n == 0) return LANCIUS_ERROR_OK;
    k_f32_to_f64<<<lcu_blocks(n, 1024), 256, 0, lcu_as_stream(s)>>>(o, a, n);
    lcu_note_launch();
    return lcu_launch_status();
}

}  // extern "C"
