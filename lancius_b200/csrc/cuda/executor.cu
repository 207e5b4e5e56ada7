// Device context and graph executor: the B200 sibling of the reference's
// lancius_schedule_execute (bleeding/v11A1/src/runtime/lancius_scheduler.c:311-362).
//
// lcu_bind_plan() turns (schedule, graph, plan) into a static launch list once:
//   * every node gets a byte offset in ONE device allocation per context:
//     [ planned pool | persistent INPUT/CONST slots | launch tables ];
//   * the executor's own plan (plan == NULL) is built on a fused view of the graph:
//     MATMUL -> ADD(BROADCAST(bias)) -> RELU|GELU -> ADD(residual) chains collapse
//     into one GEMM with that epilogue, and RESHAPE/FLATTEN share their source's
//     bytes; nodes inside a chain alias the chain's storage;
//   * same-shaped nodes of one wave (the reference runs them concurrently on its
//     thread pool, :364-413) become ONE launch over a device-resident pointer table.
// lancius_schedule_execute_cuda() replays that list on the context's stream,
// optionally through a captured CUDA graph.
#include "lcu_internal.h"
#include "../host/planner_internal.h"
#include <map>
#include <string>
#include <tuple>
#include <vector>
#include <cstring>
#include <cstdio>

namespace {

constexpr size_t NPOS = (size_t)-1;
constexpr size_t SLOT_ALIGN = 256;

enum StepKind { S_GEMM, S_ATTN, S_CONV, S_LN, S_SOFTMAX, S_SUMAX1, S_ELT, S_BCAST, S_MAXPOOL, S_MISC, S_MLP2 };

struct Step {
    StepKind kind;
    int count = 1;
    size_t table_off = 0;      // byte offset of the group table inside the allocation
    size_t M = 0, N = 0, K = 0;
    int epi = 0, op = 0, vec = 0, causal = 0, relu = 0;
    int tc = 0, ga = 1, gb = 1;   // tensor-core GEMM; distinct A / B operands in the group
    int plan_idx = -1, plan_mode = -1;
    size_t S = 0, H = 0, D = 0;
    size_t cn = 0, ci = 0, h = 0, w = 0, co = 0, kh = 0, kw = 0, stride = 0, pad = 0;
    size_t out = 0, in0 = 0, in1 = 0;   // node offsets for single-instance steps
    size_t rows = 0, cols = 0, n = 0, in_elems = 0;
    size_t in2 = 0;            // third input (S_MISC)
    int lop = 0;               // lancius opcode (S_MISC); LANCIUS_OP_MATMUL / CONV2D* mean the INT8-weight forms
    double dscale = 1.0;       // INT8 weight scale
    size_t packed_off = (size_t)-1;   // INT8 MATMUL: K-major copy of the weights in ctx->packed
    size_t wsplit_off = (size_t)-1;   // tensor-core MATMUL on INPUT weights: hi/lo copies in ctx->wsplit
    int amap_idx = -1;                // tensor-core MATMUL in raw-A mode / tensor-core ATTENTION: first of its maps in ctx->amaps
    float* attn_lo = nullptr;         // tensor-core ATTENTION: K/V lo copies ([count][2][S][H][D])
    float eps = 1e-5f;
    uint32_t node_id = 0;      // S_CONV: the conv node (its output)
    uint32_t in_id = 0;        // S_CONV: the input node
    int in_nhwc = 0;           // S_CONV: the input slot holds NHWC (written by the previous conv)
    int out_nhwc = 0;          // S_CONV: store the output NHWC for the convs that read it
    size_t in_lo = (size_t)-1; // S_CONV: tf32_lo of the NHWC input in ctx->lo_buf (float offset)
    size_t out_lo = (size_t)-1;// S_CONV: where to store tf32_lo of the NHWC output
    size_t gap_off = (size_t)-1;  // S_CONV: per-tile channel sums for a global pool (ctx->gap_buf);
                                  // S_SUMAX1: the same sums, added up instead of reading the conv output
    int gap_tiles = 0;            // tiles per image of those sums
    mutable int gap_done = 0;     // S_CONV: the last run stored them (the persistent kernel ran)
    int gap_src = -1;             // S_SUMAX1: index of the conv step that stores them
    const lancius_node* node0 = nullptr;   // first node of the step's group
    size_t table2_off = 0;     // S_MLP2: the second product's group table
    size_t N2 = 0;             // S_MLP2: columns of the second product (its K is N)
    int epi2 = 0;              // S_MLP2: the second product's epilogue
    size_t ticket_off = 0;     // S_MLP2: ceil(M / 16) zeroed counters
};

struct Chain {          // a MATMUL and the epilogue nodes folded into it
    const lancius_node* bias_src = nullptr;
    const lancius_node* resid = nullptr;
    int epi = LCU_EPI_NONE;
};

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

}  // namespace

struct lcu_ctx {
    int device = 0;
    cudaStream_t stream = nullptr;
    int mode = LCU_MODE_FP32_EXACT;
    int replay = 0;
    int fusion = 1;
    lancius_graph* g = nullptr;
    lancius_schedule* s = nullptr;
    char* dmem = nullptr;
    size_t dmem_bytes = 0;
    double* staging = nullptr;
    size_t staging_elems = 0;
    void* scratch = nullptr;            // tensor-core GEMM hi/lo operand copies
    size_t scratch_bytes = 0;
    // INT8 weights feeding a tensor-core MATMUL, kept K-major ([N][Kp]) and refreshed by
    // every upload of the weight node
    struct Pack { uint32_t node; size_t off, K, N, Kp; };
    std::vector<Pack> packs;
    int8_t* packed = nullptr;
    size_t packed_bytes = 0;
    // FP32 weights (INPUT nodes) feeding tensor-core MATMULs, kept as TF32 hi/lo copies
    // ([Gb][K][pad4(N)] per step, lo after hi) and refreshed by every upload of the node;
    // conv weights (conv != 0) are kept as [Co][Kh][Kw][Ci] hi/lo copies the same way
    struct WSplit { uint32_t node; size_t hi_off, lo_off, K, N, Np; int conv = 0, co = 0, ci = 0, kh = 0, kw = 0; };
    std::vector<WSplit> wsplits;
    float* wsplit = nullptr;
    size_t wsplit_floats = 0;
    std::vector<float*> attn_lo;        // lo copies of the tensor-core attention steps
    std::vector<CUtensorMap> amaps_host;  // raw-A tensor maps of every step, uploaded to amaps at bind
    CUtensorMap* amaps = nullptr;
    std::vector<uint8_t> nhwc;          // node id -> 1: a conv output stored NHWC (only convs read it)
    float* lo_buf = nullptr;            // tf32_lo copies of NHWC-kept conv outputs
    size_t lo_floats = 0;
    float* gap_buf = nullptr;           // per-tile channel sums of convs feeding a global pool
    size_t gap_floats = 0;
    std::vector<LcuTcGemmPlan> tc_plans;
    std::vector<size_t> off;            // node id -> byte offset in dmem (NPOS: no storage)
    std::vector<Step> steps;
    cudaGraphExec_t exec = nullptr;
    int graph_launches = 0;
    int last_launches = 0;
};

static lancius_error fail(lancius_error e) { lancius_set_error(e); return e; }
static lancius_error cuda_fail(cudaError_t e) { return lcu_check_cuda(e); }

static void release_binding(lcu_ctx* c) {
    if (c->exec) { cudaGraphExecDestroy(c->exec); c->exec = nullptr; }
    if (c->dmem) { cudaFree(c->dmem); c->dmem = nullptr; }
    if (c->staging) { cudaFree(c->staging); c->staging = nullptr; }
    if (c->scratch) { cudaFree(c->scratch); c->scratch = nullptr; }
    if (c->packed) { cudaFree(c->packed); c->packed = nullptr; }
    c->packs.clear(); c->packed_bytes = 0;
    if (c->wsplit) { cudaFree(c->wsplit); c->wsplit = nullptr; }
    c->wsplits.clear(); c->wsplit_floats = 0;
    if (c->amaps) { cudaFree(c->amaps); c->amaps = nullptr; }
    for (float* p : c->attn_lo) cudaFree(p);
    c->attn_lo.clear();
    c->amaps_host.clear();
    c->dmem_bytes = 0; c->staging_elems = 0; c->scratch_bytes = 0;
    c->tc_plans.clear();
    c->nhwc.clear();
    if (c->lo_buf) { cudaFree(c->lo_buf); c->lo_buf = nullptr; }
    c->lo_floats = 0;
    if (c->gap_buf) { cudaFree(c->gap_buf); c->gap_buf = nullptr; }
    c->gap_floats = 0;
    c->off.clear(); c->steps.clear();
    c->g = nullptr; c->s = nullptr;
}

extern "C" {

lcu_ctx* lcu_create(int device) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n) {
        cudaGetLastError();
        lancius_set_error(LANCIUS_ERROR_INTERNAL);
        return nullptr;
    }
    if (cudaSetDevice(device) != cudaSuccess) { lancius_set_error(LANCIUS_ERROR_INTERNAL); return nullptr; }
    lcu_ctx* c = new (std::nothrow) lcu_ctx();
    if (!c) { lancius_set_error(LANCIUS_ERROR_OOM); return nullptr; }
    c->device = device;
    if (cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking) != cudaSuccess) {
        delete c;
        lancius_set_error(LANCIUS_ERROR_INTERNAL);
        return nullptr;
    }
    return c;
}

void lcu_destroy(lcu_ctx* c) {
    if (!c) return;
    cudaSetDevice(c->device);
    cudaStreamSynchronize(c->stream);
    release_binding(c);
    cudaStreamDestroy(c->stream);
    delete c;
}

lancius_error lcu_set_mode(lcu_ctx* c, lcu_mode mode) {
    if (!c) return fail(LANCIUS_ERROR_NULL_PTR);
    if (mode != LCU_MODE_FP32_EXACT && mode != LCU_MODE_TF32 && mode != LCU_MODE_BF16) return fail(LANCIUS_ERROR_UNSUPPORTED_DTYPE);
    if (c->mode != (int)mode && c->exec) { cudaGraphExecDestroy(c->exec); c->exec = nullptr; }
    c->mode = mode;
    return LANCIUS_ERROR_OK;
}

lancius_error lcu_set_graph_replay(lcu_ctx* c, int enable) {
    if (!c) return fail(LANCIUS_ERROR_NULL_PTR);
    c->replay = enable ? 1 : 0;
    if (!c->replay && c->exec) { cudaGraphExecDestroy(c->exec); c->exec = nullptr; }
    return LANCIUS_ERROR_OK;
}

lancius_error lcu_set_fusion(lcu_ctx* c, int enable) {
    if (!c) return fail(LANCIUS_ERROR_NULL_PTR);
    c->fusion = enable ? 1 : 0;
    return LANCIUS_ERROR_OK;
}

void* lcu_stream(lcu_ctx* c) { return c ? (void*)c->stream : nullptr; }

// Points a binding at another schedule object with the same waves over the same nodes
// (a caller that rebuilds its schedule per run); the launch list is kept.
void lcu_ctx_retarget_schedule(lcu_ctx* c, lancius_schedule* s) {
    if (c && c->dmem) c->s = s;
}

// Waits for `stream`, then reads the tensor-core kernels' watchdog words of the current
// device (set when a bounded mbarrier wait gave up): any set word is cleared and reported
// as LANCIUS_ERROR_INTERNAL. The words are per device, shared by every stream on it.
lancius_error lcu_check_stream(void* stream) {
    cudaStream_t st = lcu_as_stream(stream);
    int* words[4] = {lcu_gemm_watchdog_addr(), lcu_attention_watchdog_addr(), lcu_conv_watchdog_addr(),
                     lcu_int8_watchdog_addr()};
    int vals[4] = {0, 0, 0, 0};
    for (int i = 0; i < 4; i++)
        if (words[i]) {
            cudaError_t ce = cudaMemcpyAsync(&vals[i], words[i], sizeof(int), cudaMemcpyDeviceToHost, st);
            if (ce != cudaSuccess) return cuda_fail(ce);
        }
    cudaError_t ce = cudaStreamSynchronize(st);
    if (ce != cudaSuccess) return cuda_fail(ce);
    bool tripped = false;
    for (int i = 0; i < 4; i++)
        if (vals[i] && words[i]) {
            tripped = true;
            cudaMemsetAsync(words[i], 0, sizeof(int), st);
        }
    if (tripped) {
        cudaStreamSynchronize(st);
        return fail(LANCIUS_ERROR_INTERNAL);
    }
    return LANCIUS_ERROR_OK;
}

// Waits for the context's stream and reports watchdog trips (lcu_check_stream).
lancius_error lcu_synchronize(lcu_ctx* c) {
    if (!c) return fail(LANCIUS_ERROR_NULL_PTR);
    cudaSetDevice(c->device);
    return lcu_check_stream(c->stream);
}

int lcu_last_launch_count(lcu_ctx* c) { return c ? c->last_launches : 0; }

float* lcu_node_device_ptr(lcu_ctx* c, const lancius_node* n) {
    if (!c || !n || !c->dmem || n->id >= c->off.size() || c->off[n->id] == NPOS) return nullptr;
    return reinterpret_cast<float*>(c->dmem + c->off[n->id]);
}

}  // extern "C"

// ---------------------------------------------------------------------------
// binding

namespace {

struct Builder {
    lcu_ctx* c;
    lancius_graph* g;
    lancius_schedule* s;
    std::vector<uint32_t> wave_of;                 // node id -> wave
    std::vector<std::vector<const lancius_node*>> users;
    std::vector<Chain> chain;                      // indexed by MATMUL id
    std::vector<uint8_t> is_chain_root;
    std::vector<uint32_t> alias;                   // LCU_ALIAS_* or root id
    std::vector<char> tables;                      // host image of all launch tables
    std::vector<std::pair<size_t, size_t>> table_fix;  // (pos in tables, node offset) patched to device pointers

    const lancius_node* sole_user(const lancius_node* n) const {
        return users[n->id].size() == 1 ? users[n->id][0] : nullptr;
    }
    bool earlier(const lancius_node* a, const lancius_node* b) const { return wave_of[a->id] < wave_of[b->id]; }

    // MATMUL -> [ADD bias] -> [RELU|GELU] -> [ADD residual]
    void find_chains() {
        for (uint32_t i = 0; i < g->node_count; i++) {
            const lancius_node* m = g->nodes[i];
            if (m->op != LANCIUS_OP_MATMUL || m->ndim != 2) continue;
            if (m->inputs[1]->dtype == LANCIUS_DTYPE_INT8 && m->inputs[1]->runtime_data_int8) continue;   // INT8 path
            size_t M = m->shape[0], N = m->shape[1];
            Chain ch;
            const lancius_node* tail = m;
            const lancius_node* u = sole_user(tail);
            if (u && u->op == LANCIUS_OP_ADD && u->input_count == 2 && u->ndim == 2) {
                const lancius_node* other = u->inputs[0] == tail ? u->inputs[1] : u->inputs[0];
                if (u->inputs[0] != u->inputs[1] && other->op == LANCIUS_OP_BROADCAST && other->ndim == 2 &&
                    other->shape[0] == M && other->shape[1] == N && other->input_count == 1 &&
                    lancius_node_elements(other->inputs[0]) == N && earlier(other->inputs[0], m) &&
                    !other->inputs[0]->runtime_data_int8) {
                    ch.bias_src = other->inputs[0];
                    if (users[other->id].size() == 1) alias[other->id] = LCU_ALIAS_ELIDED;
                    alias[u->id] = m->id;
                    tail = u;
                    u = sole_user(tail);
                }
            }
            // small classifier heads: MATMUL -> ADD(bias) -> SOFTMAX over N <= 32 columns, the
            // whole row in one CUDA-core tile
            if (u && u->op == LANCIUS_OP_SOFTMAX && u->ndim == 2 && u->shape[0] == M && u->shape[1] == N &&
                lcu_gemm_softmax_fold_ok(M, N, m->inputs[0]->shape[m->inputs[0]->ndim - 1])) {
                ch.epi = LCU_EPI_SOFTMAX_ROW;
                alias[u->id] = m->id;
                chain[m->id] = ch;
                is_chain_root[m->id] = 1;
                continue;
            }
            if (u && (u->op == LANCIUS_OP_RELU || u->op == LANCIUS_OP_GELU)) {
                ch.epi = u->op == LANCIUS_OP_RELU ? LCU_EPI_RELU : LCU_EPI_GELU;
                alias[u->id] = m->id;
                tail = u;
                u = sole_user(tail);
            }
            if (u && u->op == LANCIUS_OP_ADD && u->input_count == 2 && u->ndim == 2 && u->inputs[0] != u->inputs[1]) {
                const lancius_node* other = u->inputs[0] == tail ? u->inputs[1] : u->inputs[0];
                if (lancius_node_elements(other) == M * N && earlier(other, m) && other->op != LANCIUS_OP_NOP) {
                    ch.resid = other;
                    alias[u->id] = m->id;
                    tail = u;
                }
            }
            chain[m->id] = ch;
            is_chain_root[m->id] = 1;
        }
    }

    void alias_views() {
        for (uint32_t i = 0; i < g->node_count; i++) {
            const lancius_node* n = g->nodes[i];
            if ((n->op == LANCIUS_OP_RESHAPE || n->op == LANCIUS_OP_FLATTEN) && n->input_count == 1 &&
                lancius_node_elements(n) <= lancius_node_elements(n->inputs[0]))
                alias[n->id] = n->inputs[0]->id;
        }
    }

    template <class T>
    size_t add_table(const std::vector<T>& v) {
        size_t pos = align_up(tables.size(), 64);
        tables.resize(pos + sizeof(T) * v.size());
        memcpy(tables.data() + pos, v.data(), sizeof(T) * v.size());
        return pos;
    }
};

// device pointer placeholder: node byte offset + 1 (0 stays NULL) -- patched at upload
inline const float* ptr_token(size_t off) { return reinterpret_cast<const float*>(off + 1); }

}  // namespace

static lancius_error build_steps(Builder& b, std::vector<size_t>& off, bool fused) {
    lcu_ctx* c = b.c;
    auto O = [&](const lancius_node* n) { return off[n->id]; };
    for (uint32_t w = 0; w < b.s->wave_count; w++) {
        // group key -> list of node indices in this wave
        std::map<std::string, std::vector<const lancius_node*>> groups;
        std::vector<std::string> order;
        for (uint32_t i = 0; i < b.s->waves[w].node_count; i++) {
            const lancius_node* n = b.s->waves[w].nodes[i];
            char key[256];
            key[0] = 0;
            switch (n->op) {
                case LANCIUS_OP_INPUT: case LANCIUS_OP_CONST: case LANCIUS_OP_NOP:
                    continue;
                default: break;
            }
            if (fused && b.alias[n->id] != LCU_ALIAS_NONE) continue;   // folded into a chain / view / elided
            for (uint32_t j = 0; j < n->input_count; j++) {
                const lancius_node* in = n->inputs[j];
                if (!in || off[in->id] == NPOS) return fail(LANCIUS_ERROR_NULL_PTR);
                const bool int8_weight_ok = j == 1 && (n->op == LANCIUS_OP_MATMUL || n->op == LANCIUS_OP_CONV2D ||
                                                       n->op == LANCIUS_OP_CONV2D_RELU_FUSED);
                if ((in->runtime_data_int8 || in->dtype == LANCIUS_DTYPE_INT8) && !int8_weight_ok)
                    return fail(LANCIUS_ERROR_UNSUPPORTED_DTYPE);
            }
            size_t E = lancius_node_elements(n);
            switch (n->op) {
                case LANCIUS_OP_MATMUL: {
                    const lancius_node *a = n->inputs[0], *bb = n->inputs[1];
                    size_t M = n->shape[0], N = n->shape[1], K = a->shape[a->ndim - 1];
                    if (lancius_node_elements(a) < M * K || lancius_node_elements(bb) < K * N) return fail(LANCIUS_ERROR_SHAPE_MISMATCH);
                    Chain ch = b.chain[n->id];
                    snprintf(key, sizeof key, "G:%zu:%zu:%zu:%d:%d:%d", M, N, K, ch.epi, ch.bias_src != nullptr, ch.resid != nullptr);
                } break;
                case LANCIUS_OP_ADD: case LANCIUS_OP_SUB: case LANCIUS_OP_MUL:
                    if (lancius_node_elements(n->inputs[0]) < E || lancius_node_elements(n->inputs[1]) < E)
                        return fail(LANCIUS_ERROR_SHAPE_MISMATCH);   // the reference reads past the end here
                    snprintf(key, sizeof key, "E:%d:%zu", (int)n->op, E);
                    break;
                case LANCIUS_OP_RELU: case LANCIUS_OP_GELU: case LANCIUS_OP_TANH:
                case LANCIUS_OP_RESHAPE: case LANCIUS_OP_FLATTEN:
                    if (lancius_node_elements(n->inputs[0]) < E) return fail(LANCIUS_ERROR_SHAPE_MISMATCH);
                    snprintf(key, sizeof key, "E:%d:%zu", (int)n->op, E);
                    break;
                case LANCIUS_OP_LAYERNORM:
                    if (n->ndim < 2 || lancius_node_elements(n->inputs[1]) < n->shape[1] ||
                        lancius_node_elements(n->inputs[2]) < n->shape[1] || lancius_node_elements(n->inputs[0]) < E)
                        return fail(LANCIUS_ERROR_SHAPE_MISMATCH);
                    snprintf(key, sizeof key, "L:%zu:%zu", n->shape[0], n->shape[1]);
                    break;
                case LANCIUS_OP_ATTENTION:
                    if (n->ndim != 3) return fail(LANCIUS_ERROR_SHAPE_MISMATCH);
                    for (int j = 0; j < 3; j++)
                        if (lancius_node_elements(n->inputs[j]) < E) return fail(LANCIUS_ERROR_SHAPE_MISMATCH);
                    if (n->shape[2] != 64 && n->shape[2] != 128) return fail(LANCIUS_ERROR_UNSUPPORTED_OP);
                    snprintf(key, sizeof key, "A:%zu:%zu:%zu:%d", n->shape[0], n->shape[1], n->shape[2], n->attr_val != 1.0);
                    break;
                case LANCIUS_OP_SOFTMAX: case LANCIUS_OP_SUM_AXIS1: case LANCIUS_OP_BROADCAST:
                case LANCIUS_OP_CONV2D: case LANCIUS_OP_CONV2D_RELU_FUSED: case LANCIUS_OP_MAXPOOL2D:
                case LANCIUS_OP_SUM: case LANCIUS_OP_SUM_AXIS0: case LANCIUS_OP_TRANSPOSE: case LANCIUS_OP_RELU_BWD:
                case LANCIUS_OP_SOFTMAX_BWD: case LANCIUS_OP_CROSS_ENTROPY: case LANCIUS_OP_CROSS_ENTROPY_BWD:
                case LANCIUS_OP_RMSNORM: case LANCIUS_OP_SWIGLU: case LANCIUS_OP_GQA: case LANCIUS_OP_MAXPOOL2D_BWD:
                case LANCIUS_OP_CONV2D_BWD: case LANCIUS_OP_CONV2D_BWD_W:
                    snprintf(key, sizeof key, "U:%u", n->id);      // one launch per node
                    break;
                default:
                    fprintf(stderr, "[LANCIUS CUDA] op %d (node %u) has no device kernel\n", (int)n->op, n->id);
                    return fail(LANCIUS_ERROR_UNSUPPORTED_OP);
            }
            std::string k(key);
            if (!groups.count(k)) order.push_back(k);
            groups[k].push_back(n);
        }
        for (const std::string& k : order) {
            const std::vector<const lancius_node*>& ns = groups[k];
            const lancius_node* n = ns[0];
            Step st;
            st.count = (int)ns.size();
            switch (n->op) {
                case LANCIUS_OP_MATMUL: {
                    st.kind = S_GEMM;
                    st.M = n->shape[0]; st.N = n->shape[1]; st.K = n->inputs[0]->shape[n->inputs[0]->ndim - 1];
                    st.epi = b.chain[n->id].epi;
                    st.tc = lcu_use_tensor_cores(st.M, st.N, st.K) &&
                            !(n->inputs[1]->dtype == LANCIUS_DTYPE_INT8 && n->inputs[1]->runtime_data_int8);
                    // distinct operands: same-shaped products of a wave often share A (Q/K/V of one
                    // LayerNorm output) or B (the weight shared by all batch elements)
                    std::vector<int> aidx(ns.size()), bidx(ns.size()), adup(ns.size(), 0), bdup(ns.size(), 0);
                    {
                        std::map<const lancius_node*, int> am, bm;
                        for (size_t i = 0; i < ns.size(); i++) {
                            auto ia = am.find(ns[i]->inputs[0]);
                            if (ia == am.end()) { aidx[i] = (int)am.size(); am[ns[i]->inputs[0]] = aidx[i]; }
                            else { aidx[i] = ia->second; adup[i] = 1; }
                            auto ib = bm.find(ns[i]->inputs[1]);
                            if (ib == bm.end()) { bidx[i] = (int)bm.size(); bm[ns[i]->inputs[1]] = bidx[i]; }
                            else { bidx[i] = ib->second; bdup[i] = 1; }
                        }
                        st.ga = (int)am.size(); st.gb = (int)bm.size();
                    }
                    if (st.tc) {
                        size_t need = lcu_gemm_tc_scratch_bytes(st.M, st.N, st.K, st.count, st.ga, st.gb, 3);
                        if (need > c->scratch_bytes) c->scratch_bytes = need;
                        st.plan_idx = (int)c->tc_plans.size();
                        c->tc_plans.push_back(LcuTcGemmPlan());
                        // weights that only uploads write are split once per upload, not per run
                        bool all_inputs = true;
                        for (const lancius_node* x : ns)
                            all_inputs = all_inputs && x->inputs[1]->op == LANCIUS_OP_INPUT &&
                                         x->inputs[1]->dtype != LANCIUS_DTYPE_INT8;
                        if (all_inputs && !lcu_no_weight_cache()) {
                            const size_t Np = (st.N + 3) & ~size_t(3), mat = st.K * Np;
                            st.wsplit_off = c->wsplit_floats;
                            for (size_t i = 0; i < ns.size(); i++)
                                if (!bdup[i])
                                    c->wsplits.push_back({ns[i]->inputs[1]->id, st.wsplit_off + bidx[i] * mat,
                                                          st.wsplit_off + (st.gb + bidx[i]) * mat, st.K, st.N, Np});
                            c->wsplit_floats += align_up(2 * st.gb * mat, 64);
                        }
                    }
                    if (n->inputs[1]->dtype == LANCIUS_DTYPE_INT8 && n->inputs[1]->runtime_data_int8) {
                        // INT8 weights: dynamic per-tensor quantisation of A (scheduler.c:195-220)
                        st.kind = S_MISC; st.lop = LANCIUS_OP_MATMUL; st.count = 1;
                        st.out = O(n); st.in0 = O(n->inputs[0]); st.in1 = O(n->inputs[1]); st.dscale = n->inputs[1]->scale;
                        st.table_off = b.add_table(std::vector<float>(64, 0.f));     // one float of scratch (max |a|)
                        st.tc = 0;
                        if (size_t need = lcu_matmul_int8_scratch_bytes(st.M, st.K, st.N)) {
                            // tensor-core INT8: quantised A in the context scratch, weights pre-packed
                            if (need > c->scratch_bytes) c->scratch_bytes = need;
                            const size_t Kp = (st.K + 15) & ~size_t(15);
                            const uint32_t wid = n->inputs[1]->id;
                            for (const auto& pk : c->packs)
                                if (pk.node == wid) st.packed_off = pk.off;
                            if (st.packed_off == (size_t)-1) {
                                st.packed_off = c->packed_bytes;
                                c->packs.push_back({wid, c->packed_bytes, st.K, st.N, Kp});
                                c->packed_bytes += align_up(st.N * Kp, 256);
                            }
                        }
                        if (ns.size() > 1) return fail(LANCIUS_ERROR_UNSUPPORTED_OP);
                        break;
                    }
                    std::vector<LcuGemmGroup> t;
                    for (size_t i = 0; i < ns.size(); i++) {
                        const lancius_node* x = ns[i];
                        const Chain& ch = b.chain[x->id];
                        t.push_back(LcuGemmGroup{ptr_token(O(x->inputs[0])), ptr_token(O(x->inputs[1])),
                                                 (float*)ptr_token(O(x)),
                                                 ch.bias_src ? ptr_token(O(ch.bias_src)) : nullptr,
                                                 ch.resid ? ptr_token(O(ch.resid)) : nullptr,
                                                 aidx[i], bidx[i], adup[i], bdup[i]});
                    }
                    st.table_off = b.add_table(t);
                } break;
                case LANCIUS_OP_ATTENTION: {
                    st.kind = S_ATTN;
                    st.S = n->shape[0]; st.H = n->shape[1]; st.D = n->shape[2]; st.causal = n->attr_val != 1.0;
                    std::vector<LcuAttnGroup> t;
                    for (const lancius_node* x : ns)
                        t.push_back(LcuAttnGroup{ptr_token(O(x->inputs[0])), ptr_token(O(x->inputs[1])),
                                                 ptr_token(O(x->inputs[2])), (float*)ptr_token(O(x))});
                    st.table_off = b.add_table(t);
                } break;
                case LANCIUS_OP_LAYERNORM: {
                    st.kind = S_LN; st.rows = n->shape[0]; st.cols = n->shape[1]; st.eps = 1e-5f; st.vec = 1;
                    std::vector<LcuRowGroup> t;
                    for (const lancius_node* x : ns)
                        t.push_back(LcuRowGroup{(float*)ptr_token(O(x)), ptr_token(O(x->inputs[0])),
                                                ptr_token(O(x->inputs[1])), ptr_token(O(x->inputs[2]))});
                    st.table_off = b.add_table(t);
                } break;
                case LANCIUS_OP_ADD: case LANCIUS_OP_SUB: case LANCIUS_OP_MUL:
                case LANCIUS_OP_RELU: case LANCIUS_OP_GELU: case LANCIUS_OP_TANH:
                case LANCIUS_OP_RESHAPE: case LANCIUS_OP_FLATTEN: {
                    st.kind = S_ELT;
                    st.op = n->op == LANCIUS_OP_ADD ? 0 : n->op == LANCIUS_OP_SUB ? 1 : n->op == LANCIUS_OP_MUL ? 2
                          : n->op == LANCIUS_OP_RELU ? 3 : n->op == LANCIUS_OP_GELU ? 4 : n->op == LANCIUS_OP_TANH ? 5 : 6;
                    st.n = lancius_node_elements(n);
                    st.vec = st.n % 4 == 0;
                    std::vector<LcuEltGroup> t;
                    for (const lancius_node* x : ns)
                        t.push_back(LcuEltGroup{(float*)ptr_token(O(x)), ptr_token(O(x->inputs[0])),
                                                x->input_count > 1 ? ptr_token(O(x->inputs[1])) : nullptr});
                    st.table_off = b.add_table(t);
                } break;
                case LANCIUS_OP_SOFTMAX:
                    st.kind = S_SOFTMAX; st.rows = n->shape[0]; st.cols = n->shape[1];
                    st.out = O(n); st.in0 = O(n->inputs[0]);
                    break;
                case LANCIUS_OP_SUM_AXIS1: {
                    st.kind = S_SUMAX1; st.rows = n->inputs[0]->shape[0]; st.cols = n->inputs[0]->shape[1];
                    st.out = O(n); st.in0 = O(n->inputs[0]);
                    const lancius_node* src = n->inputs[0];   // through reshapes to the node that holds the data
                    while ((src->op == LANCIUS_OP_RESHAPE || src->op == LANCIUS_OP_FLATTEN) && src->input_count == 1 &&
                           lancius_node_elements(src) == lancius_node_elements(src->inputs[0]))
                        src = src->inputs[0];
                    st.in_id = src->id;
                } break;
                case LANCIUS_OP_BROADCAST: {
                    size_t ie = lancius_node_elements(n->inputs[0]);
                    if (ie != 1 && ie < n->shape[1]) return fail(LANCIUS_ERROR_SHAPE_MISMATCH);
                    st.kind = S_BCAST; st.in_elems = ie; st.out = O(n); st.in0 = O(n->inputs[0]);
                    // scalar: fill every element; row vector: the first shape[0] x shape[1] block (scheduler.c:271-277)
                    st.rows = ie == 1 ? lancius_node_elements(n) : n->shape[0];
                    st.cols = ie == 1 ? 1 : n->shape[1];
                } break;
                case LANCIUS_OP_CONV2D: case LANCIUS_OP_CONV2D_RELU_FUSED: {
                    const lancius_node *in = n->inputs[0], *wt = n->inputs[1];
                    st.kind = S_CONV; st.relu = n->op == LANCIUS_OP_CONV2D_RELU_FUSED;
                    st.node_id = n->id; st.in_id = n->inputs[0]->id;
                    st.cn = in->shape[0]; st.ci = in->shape[1]; st.h = in->shape[2]; st.w = in->shape[3];
                    st.co = wt->shape[0]; st.kh = wt->shape[2]; st.kw = wt->shape[3]; st.stride = n->stride; st.pad = n->pad;
                    if (in->ndim != 4 || wt->ndim != 4 || wt->shape[1] != st.ci || st.stride == 0) return fail(LANCIUS_ERROR_SHAPE_MISMATCH);
                    st.out = O(n); st.in0 = O(in); st.in1 = O(wt);
                    if (wt->dtype == LANCIUS_DTYPE_INT8 && wt->runtime_data_int8) {
                        // INT8 weights: dynamic quantisation of the input (vision_ops.c:16-57)
                        st.kind = S_MISC; st.lop = n->op; st.dscale = wt->scale;
                        st.table_off = b.add_table(std::vector<float>(64, 0.f));
                        size_t need = lcu_conv2d_int8_scratch_bytes(st.cn, st.ci, st.h, st.w, st.co, st.kh, st.kw, st.stride,
                                                                    st.pad);
                        if (need > c->scratch_bytes) c->scratch_bytes = need;
                        break;
                    }
                    size_t ho = (st.h + 2 * st.pad - st.kh) / st.stride + 1, wo = (st.w + 2 * st.pad - st.kw) / st.stride + 1;
                    st.M = st.co; st.N = st.cn * ho * wo; st.K = st.ci * st.kh * st.kw;
                    st.tc = st.cn && st.ci && lcu_use_tensor_cores(st.M, st.N, st.K) &&
                            !(lcu_conv_smallk_supported(st.ci, st.kh, st.kw, st.co) && !lcu_force_tc_conv());
                    if (st.tc) {
                        size_t need = lcu_gemm_tc_scratch_bytes(st.M, st.N, st.K, 1, 1, 1, 3);
                        const LcuConvShape cs{(int)st.cn, (int)st.ci, (int)st.h, (int)st.w, (int)st.co, (int)st.kh,
                                              (int)st.kw, (int)st.stride, (int)st.pad, (int)ho, (int)wo};
                        if (lcu_conv_nhwc_supported(cs) && lcu_conv_nhwc_scratch_bytes(cs, 3) > need)
                            need = lcu_conv_nhwc_scratch_bytes(cs, 3);
                        if (need > c->scratch_bytes) c->scratch_bytes = need;
                        st.plan_idx = (int)c->tc_plans.size();
                        c->tc_plans.push_back(LcuTcGemmPlan());
                        std::vector<LcuGemmGroup> t{LcuGemmGroup{ptr_token(O(wt)), ptr_token(O(in)), (float*)ptr_token(O(n)),
                                                                 nullptr, nullptr}};
                        st.table_off = b.add_table(t);
                        // weights that only uploads write are split once per upload, not per run
                        if (lcu_conv_nhwc_supported(cs) && wt->op == LANCIUS_OP_INPUT && !lcu_no_weight_cache()) {
                            const size_t we = st.co * st.K;
                            st.wsplit_off = c->wsplit_floats;
                            lcu_ctx::WSplit ws{wt->id, st.wsplit_off, st.wsplit_off + align_up(we, 64), st.K, st.co, st.co};
                            ws.conv = 1; ws.co = (int)st.co; ws.ci = (int)st.ci; ws.kh = (int)st.kh; ws.kw = (int)st.kw;
                            c->wsplits.push_back(ws);
                            c->wsplit_floats += 2 * align_up(we, 64);
                        }
                    }
                } break;
                case LANCIUS_OP_SUM: case LANCIUS_OP_SUM_AXIS0: case LANCIUS_OP_TRANSPOSE: case LANCIUS_OP_RELU_BWD:
                case LANCIUS_OP_SOFTMAX_BWD: case LANCIUS_OP_CROSS_ENTROPY: case LANCIUS_OP_CROSS_ENTROPY_BWD:
                case LANCIUS_OP_RMSNORM: case LANCIUS_OP_SWIGLU: case LANCIUS_OP_GQA: case LANCIUS_OP_MAXPOOL2D_BWD:
                case LANCIUS_OP_CONV2D_BWD: case LANCIUS_OP_CONV2D_BWD_W: {
                    const lancius_node* i0 = n->inputs[0];
                    const lancius_node* i1 = n->input_count > 1 ? n->inputs[1] : nullptr;
                    const lancius_node* i2 = n->input_count > 2 ? n->inputs[2] : nullptr;
                    st.kind = S_MISC; st.lop = n->op; st.out = O(n); st.in0 = O(i0);
                    st.in1 = i1 ? O(i1) : 0; st.in2 = i2 ? O(i2) : 0;
                    st.n = lancius_node_elements(n);
                    size_t E0 = lancius_node_elements(i0), E1 = i1 ? lancius_node_elements(i1) : 0;
                    bool okshape = true;
                    switch (n->op) {
                        case LANCIUS_OP_SUM: st.n = E0; break;
                        case LANCIUS_OP_SUM_AXIS0: case LANCIUS_OP_TRANSPOSE:
                            okshape = i0->ndim == 2; st.rows = i0->shape[0]; st.cols = i0->shape[1]; break;
                        case LANCIUS_OP_RELU_BWD: case LANCIUS_OP_SWIGLU: okshape = E0 >= st.n && E1 >= st.n; break;
                        case LANCIUS_OP_SOFTMAX_BWD: case LANCIUS_OP_CROSS_ENTROPY_BWD:
                            okshape = n->ndim == 2 && E0 >= st.n && E1 >= st.n; st.rows = n->shape[0]; st.cols = n->shape[1]; break;
                        case LANCIUS_OP_CROSS_ENTROPY:
                            okshape = i0->ndim == 2; st.rows = i0->shape[0]; st.cols = i0->shape[1]; break;
                        case LANCIUS_OP_RMSNORM:
                            okshape = n->ndim >= 2 && E1 >= n->shape[1]; st.rows = n->shape[0]; st.cols = n->shape[1]; break;
                        case LANCIUS_OP_GQA:
                            okshape = n->ndim == 3 && n->kernel_w && n->kernel_h % n->kernel_w == 0 &&
                                      (n->shape[2] == 64 || n->shape[2] == 128) && n->shape[1] == n->kernel_h;
                            st.S = n->shape[0]; st.H = n->kernel_h; st.co = n->kernel_w; st.D = n->shape[2]; break;
                        case LANCIUS_OP_MAXPOOL2D_BWD:
                            okshape = i1 && i1->ndim == 4; if (!okshape) break;
                            st.cn = i1->shape[0]; st.ci = i1->shape[1]; st.h = i1->shape[2]; st.w = i1->shape[3];
                            st.kh = n->kernel_h; st.stride = n->stride; break;
                        case LANCIUS_OP_CONV2D_BWD:     // (grad, fwd_in, fwd_w)
                            okshape = i1 && i2 && i1->ndim == 4 && i2->ndim == 4 && i0->ndim == 4; if (!okshape) break;
                            st.cn = i1->shape[0]; st.ci = i1->shape[1]; st.h = i1->shape[2]; st.w = i1->shape[3];
                            st.co = i2->shape[0]; st.kh = i2->shape[2]; st.kw = i2->shape[3]; st.M = i0->shape[2]; st.N = i0->shape[3];
                            st.stride = n->stride; st.pad = n->pad; break;
                        case LANCIUS_OP_CONV2D_BWD_W:   // (grad, fwd_in)
                            okshape = i1 && i1->ndim == 4 && i0->ndim == 4; if (!okshape) break;
                            st.cn = i1->shape[0]; st.ci = i1->shape[1]; st.h = i1->shape[2]; st.w = i1->shape[3];
                            st.co = n->shape[0]; st.kh = n->shape[2]; st.kw = n->shape[3]; st.M = i0->shape[2]; st.N = i0->shape[3];
                            st.stride = n->stride; st.pad = n->pad; break;
                        default: break;
                    }
                    if (!okshape) return fail(LANCIUS_ERROR_SHAPE_MISMATCH);
                } break;
                case LANCIUS_OP_MAXPOOL2D: {
                    const lancius_node* in = n->inputs[0];
                    st.kind = S_MAXPOOL; st.cn = in->shape[0]; st.ci = in->shape[1]; st.h = in->shape[2]; st.w = in->shape[3];
                    st.kh = n->kernel_h; st.stride = n->stride; st.out = O(n); st.in0 = O(in);
                } break;
                default: return fail(LANCIUS_ERROR_UNSUPPORTED_OP);
            }
            st.node0 = n;
            c->steps.push_back(st);
        }
    }
    // MATMUL(+bias, act) immediately followed by a small MATMUL(+bias) -> SOFTMAX over its
    // output: one launch (k_mlp2) instead of two. The second product's weight and bias
    // must be INPUT nodes (resident before the first product runs). Opt-in (LCU_MLP_FUSE=1):
    // with L2 flushed between executions the two-launch form measured faster (20.5 us
    // against 22.4-35 us per MLP graph): the fused kernel's last CTA runs the second
    // product alone, on instructions and data that all come cold.
    const char* mlp_env = getenv("LCU_MLP_FUSE");
    const bool no_mlp_fuse = !(mlp_env && mlp_env[0] == '1');
    for (size_t i = 0; !no_mlp_fuse && i + 1 < c->steps.size(); i++) {
        Step &s1 = c->steps[i], &s2 = c->steps[i + 1];
        if (s1.kind != S_GEMM || s2.kind != S_GEMM || s1.tc || s2.tc || s1.count != 1 || s2.count != 1) continue;
        if (s2.epi != LCU_EPI_SOFTMAX_ROW || s1.epi == LCU_EPI_SOFTMAX_ROW || s2.K != s1.N || s2.M != s1.M) continue;
        const LcuGemmGroup* t1 = reinterpret_cast<const LcuGemmGroup*>(b.tables.data() + s1.table_off);
        const LcuGemmGroup* t2 = reinterpret_cast<const LcuGemmGroup*>(b.tables.data() + s2.table_off);
        if ((const void*)t2->a != (const void*)t1->c || t1->resid || t2->resid) continue;
        const lancius_node* m2 = s2.node0;
        const Chain& ch2 = b.chain[m2->id];
        if (m2->inputs[1]->op != LANCIUS_OP_INPUT || (ch2.bias_src && ch2.bias_src->op != LANCIUS_OP_INPUT)) continue;
        if (!lcu_mlp2_ok(s1.M, s1.N, s1.K, s2.N)) continue;
        s1.kind = S_MLP2;
        s1.table2_off = s2.table_off;
        s1.N2 = s2.N;
        s1.epi2 = s2.epi;
        s1.ticket_off = b.add_table(std::vector<unsigned>((s1.M + 15) / 16 + 1, 0u));
        c->steps.erase(c->steps.begin() + (long)(i + 1));
    }
    return LANCIUS_ERROR_OK;
}

static LcuConvShape conv_shape(const Step& s) {
    const size_t ho = (s.h + 2 * s.pad - s.kh) / s.stride + 1, wo = (s.w + 2 * s.pad - s.kw) / s.stride + 1;
    return LcuConvShape{(int)s.cn, (int)s.ci, (int)s.h, (int)s.w, (int)s.co, (int)s.kh, (int)s.kw, (int)s.stride,
                        (int)s.pad, (int)ho, (int)wo};
}

// A conv step that reads its input through the NHWC tensor-core path
static bool reads_nhwc_path(const Step& s) {
    return s.kind == S_CONV && s.tc && lcu_conv_nhwc_supported(conv_shape(s)) && !lcu_conv_force_im2col();
}

// A conv output read only by convs on the NHWC path is stored NHWC by its producer and read
// in place by them: no NCHW store and no NCHW -> NHWC pass in between. Downloads of such a
// node transpose back to NCHW. LCU_NO_NHWC_HANDOFF=1 turns this off.
static void plan_nhwc_handoff(lcu_ctx* c, const Builder& b) {
    const char* env = getenv("LCU_NO_NHWC_HANDOFF");
    if (env && env[0] == '1') return;
    c->nhwc.assign(b.g->next_id, 0);
    for (Step& p : c->steps) {
        if (p.kind != S_CONV) continue;
        const bool can_write = p.tc ? (reads_nhwc_path(p) && lcu_conv_nhwc_out_ok(conv_shape(p)))
                                    : lcu_conv_smallk_nhwc_ok(p.cn, p.ci, p.h, p.w, p.co, p.kh, p.kw, p.stride, p.pad) != 0;
        if (!can_write) continue;
        const std::vector<const lancius_node*>& users = b.users[p.node_id];
        if (users.empty()) continue;
        bool ok = true;
        for (const lancius_node* u : users) {
            bool found = false;
            for (const Step& q : c->steps)
                if (q.kind == S_CONV && q.node_id == u->id && q.in_id == p.node_id && reads_nhwc_path(q)) found = true;
            ok = ok && found && u->inputs[1] && u->inputs[1]->id != p.node_id;
        }
        if (!ok) continue;
        p.out_nhwc = 1;
        c->nhwc[p.node_id] = 1;
        // The producer also stores tf32_lo of its output, so the consumers load hi (the value
        // itself) and lo by TMA instead of splitting on chip (LCU_NO_NHWC_LO=1: split on chip)
        const char* lo_env = getenv("LCU_NO_NHWC_LO");
        const bool with_lo = !(lo_env && lo_env[0] == '1');
        if (with_lo) {
            const LcuConvShape cs = conv_shape(p);
            p.out_lo = c->lo_floats;
            c->lo_floats += align_up((size_t)cs.n * cs.co * cs.ho * cs.wo, 64);
        }
        for (Step& q : c->steps)
            if (q.kind == S_CONV && q.in_id == p.node_id) {
                q.in_nhwc = 1;
                if (with_lo) q.in_lo = p.out_lo;
            }
    }
}

// A global average pool over a tensor-core conv's NCHW output (SUM_AXIS1 over [N*Co][Ho*Wo],
// through reshapes) adds up per-tile channel sums that the conv's epilogue stores beside its
// output, instead of reading the output again. The output is still stored (any node can be
// downloaded). LCU_NO_GAP_FUSE=1 turns this off.
static void plan_gap_fusion(lcu_ctx* c) {
    const char* env = getenv("LCU_NO_GAP_FUSE");
    if (env && env[0] == '1') return;
    for (size_t i = 0; i < c->steps.size(); i++) {
        Step& q = c->steps[i];
        if (q.kind != S_SUMAX1) continue;
        for (size_t k = 0; k < i; k++) {
            Step& p = c->steps[k];
            if (p.kind != S_CONV || p.node_id != q.in_id || !reads_nhwc_path(p) || p.out_nhwc || p.gap_off != NPOS) continue;
            const LcuConvShape cs = conv_shape(p);
            const int tiles = lcu_conv_tiles_per_image(cs);
            if (tiles <= 0 || q.rows != (size_t)cs.n * cs.co || q.cols != (size_t)cs.ho * cs.wo) continue;
            p.gap_off = q.gap_off = c->gap_floats;
            p.gap_tiles = q.gap_tiles = tiles;
            q.gap_src = (int)k;
            c->gap_floats += align_up((size_t)cs.n * tiles * cs.co, 64);
        }
    }
}

extern "C" lancius_error lcu_bind_plan(lcu_ctx* c, lancius_schedule* s, lancius_graph* g, const lancius_memory_plan* plan) {
    if (!c || !s || !g) return fail(LANCIUS_ERROR_NULL_PTR);
    cudaSetDevice(c->device);
    cudaStreamSynchronize(c->stream);
    release_binding(c);

    Builder b;
    b.c = c; b.g = g; b.s = s;
    uint32_t ids = g->next_id;
    b.wave_of.assign(ids, 0);
    b.users.assign(ids, {});
    b.chain.assign(ids, Chain());
    b.is_chain_root.assign(ids, 0);
    b.alias.assign(ids, LCU_ALIAS_NONE);
    for (uint32_t w = 0; w < s->wave_count; w++)
        for (uint32_t i = 0; i < s->waves[w].node_count; i++) b.wave_of[s->waves[w].nodes[i]->id] = w;
    for (uint32_t i = 0; i < g->node_count; i++)
        for (uint32_t j = 0; j < g->nodes[i]->input_count; j++)
            if (g->nodes[i]->inputs[j]) b.users[g->nodes[i]->inputs[j]->id].push_back(g->nodes[i]);

    bool fused = plan == nullptr;
    lancius_memory_plan* own = nullptr;
    if (fused) {
        if (c->fusion) b.find_chains();
        b.alias_views();
        own = lcu_plan_aliased(s, g, 4, SLOT_ALIGN, b.alias.data());
        if (!own) return fail(LANCIUS_ERROR_OOM);
        plan = own;
    } else if (lancius_memory_plan_validate(plan, s, g, 4) != LANCIUS_ERROR_OK) {
        return fail(LANCIUS_ERROR_INVALID_MODEL);
    }

    // device layout: pool, then persistent INPUT/CONST slots
    std::vector<size_t> off(ids, NPOS);
    size_t cursor = align_up(plan->peak_memory, SLOT_ALIGN);
    size_t max_io = 0;
    for (uint32_t i = 0; i < g->node_count; i++) {
        const lancius_node* n = g->nodes[i];
        size_t E = lancius_node_elements(n);
        if (E > max_io) max_io = E;
        if (n->op == LANCIUS_OP_INPUT || n->op == LANCIUS_OP_CONST) {
            off[n->id] = cursor;
            cursor += align_up(E * 4 ? E * 4 : 4, SLOT_ALIGN);
        } else if (plan->is_pooled[n->id] == 1) {
            off[n->id] = plan->offsets[n->id];
        }
    }
    // aliases (views / chain members) resolve to their storage root
    for (int pass = 0; pass < 64; pass++) {
        bool changed = false;
        for (uint32_t i = 0; i < g->node_count; i++) {
            const lancius_node* n = g->nodes[i];
            uint32_t a = fused ? b.alias[n->id] : LCU_ALIAS_NONE;
            if (a != LCU_ALIAS_NONE && a != LCU_ALIAS_ELIDED && off[n->id] == NPOS && off[a] != NPOS) {
                off[n->id] = off[a]; changed = true;
            }
        }
        if (!changed) break;
    }
    lancius_error e = build_steps(b, off, fused);
    if (own) lancius_memory_plan_destroy(own);
    if (e != LANCIUS_ERROR_OK) { c->steps.clear(); return e; }
    if (fused) plan_nhwc_handoff(c, b);
    if (fused) plan_gap_fusion(c);

    size_t table_base = align_up(cursor, SLOT_ALIGN);
    size_t total = table_base + align_up(b.tables.size(), SLOT_ALIGN);
    cudaError_t ce = cudaMalloc(&c->dmem, total ? total : 256);
    if (ce != cudaSuccess) { cudaGetLastError(); c->steps.clear(); return fail(LANCIUS_ERROR_OOM); }
    c->dmem_bytes = total;
    // patch pointer tokens (offset + 1) into device addresses
    auto patch = [&](const float*& p) { if (p) p = reinterpret_cast<const float*>(c->dmem + ((size_t)p - 1)); };
    for (Step& st : c->steps) {
        char* base = b.tables.data() + st.table_off;
        if (st.kind == S_MLP2) {
            for (size_t toff : {st.table_off, st.table2_off}) {
                LcuGemmGroup* t = (LcuGemmGroup*)(b.tables.data() + toff);
                patch(t->a); patch(t->b); patch((const float*&)t->c); patch(t->bias); patch(t->resid);
            }
        }
        if (st.kind == S_GEMM || (st.kind == S_CONV && st.tc)) {
            LcuGemmGroup* t = (LcuGemmGroup*)base;
            for (int i = 0; i < st.count; i++) {
                patch(t[i].a); patch(t[i].b); patch((const float*&)t[i].c); patch(t[i].bias); patch(t[i].resid);
            }
            if (st.kind == S_GEMM && st.tc && !lcu_no_raw_a()) {
                // raw-A mode: the GEMM reads each distinct A in place and splits it on chip.
                // Needs K % 4 == 0, aligned A, and no C of the wave overlapping any A (the
                // groups' CTAs read A while others already store C).
                std::vector<CUtensorMap> maps(st.ga);
                bool ok = true;
                for (int i = 0; i < st.count && ok; i++) {
                    const char* a0 = (const char*)t[i].a;
                    const char* a1 = a0 + st.M * st.K * 4;
                    for (int j = 0; j < st.count && ok; j++) {
                        const char* c0 = (const char*)t[j].c;
                        ok = c0 + st.M * st.N * 4 <= a0 || a1 <= c0;
                    }
                    if (ok && !t[i].adup) ok = lcu_gemm_tc_make_raw_a_map(&maps[t[i].aidx], t[i].a, st.M, st.K);
                }
                if (ok) {
                    st.amap_idx = (int)c->amaps_host.size();
                    c->amaps_host.insert(c->amaps_host.end(), maps.begin(), maps.end());
                }
            }
        } else if (st.kind == S_ATTN) {
            LcuAttnGroup* t = (LcuAttnGroup*)base;
            for (int i = 0; i < st.count; i++) { patch(t[i].q); patch(t[i].k); patch(t[i].v); patch((const float*&)t[i].o); }
            if (lcu_attention_tc_supported(st.D)) {   // Q/K/V tensor maps of every node, read by TMA
                const size_t per_set = lcu_attention_tc_lo_floats(1, st.S, st.H);
                float* lo = nullptr;   // K/V lo copies only for the split-pass form
                if (lcu_attention_tc_needs_lo()) {
                    if (cudaMalloc(&lo, per_set * st.count * sizeof(float)) != cudaSuccess) {
                        cudaGetLastError();
                        release_binding(c);
                        return fail(LANCIUS_ERROR_OOM);
                    }
                    c->attn_lo.push_back(lo);
                }
                st.attn_lo = lo;
                std::vector<CUtensorMap> maps(LCU_ATTN_TC_MAPS * st.count);
                for (int i = 0; i < st.count; i++)
                    if (!lcu_attention_tc_make_maps(&maps[LCU_ATTN_TC_MAPS * i], t[i].q, t[i].k, t[i].v, t[i].o,
                                                    lo ? lo + per_set * i : nullptr, 1, st.S, st.H)) {
                        release_binding(c);
                        return fail(LANCIUS_ERROR_INTERNAL);
                    }
                st.amap_idx = (int)c->amaps_host.size();
                c->amaps_host.insert(c->amaps_host.end(), maps.begin(), maps.end());
            }
        } else if (st.kind == S_LN) {
            LcuRowGroup* t = (LcuRowGroup*)base;
            for (int i = 0; i < st.count; i++) { patch((const float*&)t[i].out); patch(t[i].in); patch(t[i].gamma); patch(t[i].beta); }
        } else if (st.kind == S_ELT) {
            LcuEltGroup* t = (LcuEltGroup*)base;
            for (int i = 0; i < st.count; i++) { patch((const float*&)t[i].out); patch(t[i].a); patch(t[i].b); }
        }
        st.table_off += table_base;
        if (st.kind == S_MLP2) {   // its second table and its tickets live in the table region too
            st.table2_off += table_base;
            st.ticket_off += table_base;
        }
    }
    if (!b.tables.empty()) {
        ce = cudaMemcpyAsync(c->dmem + table_base, b.tables.data(), b.tables.size(), cudaMemcpyHostToDevice, c->stream);
        if (ce != cudaSuccess) { release_binding(c); return cuda_fail(ce); }
    }
    if (c->scratch_bytes) {
        ce = cudaMalloc(&c->scratch, c->scratch_bytes);
        if (ce != cudaSuccess) { cudaGetLastError(); release_binding(c); return fail(LANCIUS_ERROR_OOM); }
    }
    if (c->packed_bytes) {
        ce = cudaMalloc(&c->packed, c->packed_bytes);
        if (ce != cudaSuccess) { cudaGetLastError(); release_binding(c); return fail(LANCIUS_ERROR_OOM); }
    }
    if (c->wsplit_floats) {
        ce = cudaMalloc(&c->wsplit, c->wsplit_floats * sizeof(float));
        if (ce != cudaSuccess) { cudaGetLastError(); release_binding(c); return fail(LANCIUS_ERROR_OOM); }
        // zero until the first upload, like the node slots of never-uploaded inputs
        ce = cudaMemsetAsync(c->wsplit, 0, c->wsplit_floats * sizeof(float), c->stream);
        if (ce != cudaSuccess) { release_binding(c); return cuda_fail(ce); }
    }
    if (c->gap_floats) {
        ce = cudaMalloc(&c->gap_buf, c->gap_floats * sizeof(float));
        if (ce != cudaSuccess) { cudaGetLastError(); release_binding(c); return fail(LANCIUS_ERROR_OOM); }
    }
    if (c->lo_floats) {
        ce = cudaMalloc(&c->lo_buf, c->lo_floats * sizeof(float));
        if (ce != cudaSuccess) { cudaGetLastError(); release_binding(c); return fail(LANCIUS_ERROR_OOM); }
    }
    if (!c->amaps_host.empty()) {
        const size_t bytes = c->amaps_host.size() * sizeof(CUtensorMap);
        ce = cudaMalloc(&c->amaps, bytes);
        if (ce != cudaSuccess) { cudaGetLastError(); release_binding(c); return fail(LANCIUS_ERROR_OOM); }
        ce = cudaMemcpyAsync(c->amaps, c->amaps_host.data(), bytes, cudaMemcpyHostToDevice, c->stream);
        if (ce != cudaSuccess) { release_binding(c); return cuda_fail(ce); }
    }
    ce = cudaMalloc(&c->staging, (max_io ? max_io : 1) * sizeof(double));
    if (ce != cudaSuccess) { cudaGetLastError(); release_binding(c); return fail(LANCIUS_ERROR_OOM); }
    c->staging_elems = max_io;
    c->off = off;
    c->g = g; c->s = s;
    // CONST nodes hold attr_val from bind time on (the reference fills them on first execution, :330-342)
    for (uint32_t i = 0; i < g->node_count; i++) {
        const lancius_node* n = g->nodes[i];
        if (n->op == LANCIUS_OP_CONST)
            if (lcu_fill((float*)(c->dmem + off[n->id]), (float)n->attr_val, lancius_node_elements(n), c->stream) != LANCIUS_ERROR_OK) {
                release_binding(c); return fail(LANCIUS_ERROR_INTERNAL);
            }
    }
    ce = cudaStreamSynchronize(c->stream);
    if (ce != cudaSuccess) { release_binding(c); return cuda_fail(ce); }
    return LANCIUS_ERROR_OK;
}

// ---------------------------------------------------------------------------
// transfers

static bool node_slot(lcu_ctx* c, const lancius_node* n, float** p, size_t* E) {
    if (!c || !n || !c->g || n->id >= c->off.size() || c->off[n->id] == NPOS) return false;
    *p = reinterpret_cast<float*>(c->dmem + c->off[n->id]);
    *E = lancius_node_elements(n);
    return true;
}

// re-split every TF32 hi/lo weight copy made from node `id` (device data at d), in stream order
static lancius_error refresh_weight_splits(lcu_ctx* c, uint32_t id, const float* d) {
    for (const auto& w : c->wsplits)
        if (w.node == id) {
            lancius_error e = w.conv ? lcu_conv_weight_split(d, c->wsplit + w.hi_off, c->wsplit + w.lo_off, w.co, w.ci,
                                                             w.kh, w.kw, c->stream)
                                     : lcu_tf32_split_rows(d, w.K, w.N, w.Np, c->wsplit + w.hi_off, c->wsplit + w.lo_off,
                                                           c->stream);
            if (e != LANCIUS_ERROR_OK) return e;
        }
    return LANCIUS_ERROR_OK;
}

extern "C" lancius_error lcu_upload(lcu_ctx* c, const lancius_node* n, const void* host, lancius_dtype dt) {
    float* d; size_t E;
    if (!host) return fail(LANCIUS_ERROR_NULL_PTR);
    if (!node_slot(c, n, &d, &E)) return fail(LANCIUS_ERROR_NULL_PTR);
    cudaSetDevice(c->device);
    if (dt == LANCIUS_DTYPE_FP32) {
        cudaError_t ce = cudaMemcpyAsync(d, host, E * 4, cudaMemcpyHostToDevice, c->stream);
        if (ce != cudaSuccess) return cuda_fail(ce);
        return refresh_weight_splits(c, n->id, d);
    }
    if (dt == LANCIUS_DTYPE_INT8) {     // INT8 weights are stored as bytes in the node's slot
        cudaError_t ce = cudaMemcpyAsync(d, host, E, cudaMemcpyHostToDevice, c->stream);
        if (ce != cudaSuccess) return cuda_fail(ce);
        for (const auto& pk : c->packs)     // and re-packed K-major for the tensor-core MATMULs
            if (pk.node == n->id) {
                lancius_error e = lcu_int8_pack_kmajor(c->packed + pk.off, reinterpret_cast<const int8_t*>(d), pk.K, pk.N,
                                                       pk.Kp, c->stream);
                if (e != LANCIUS_ERROR_OK) return e;
            }
        return LANCIUS_ERROR_OK;
    }
    if (dt != LANCIUS_DTYPE_FP64) return fail(LANCIUS_ERROR_UNSUPPORTED_DTYPE);
    if (E > c->staging_elems) return fail(LANCIUS_ERROR_SHAPE_MISMATCH);
    cudaError_t ce = cudaMemcpyAsync(c->staging, host, E * 8, cudaMemcpyHostToDevice, c->stream);
    if (ce != cudaSuccess) return cuda_fail(ce);
    lancius_error e = lcu_convert_f64_to_f32(d, c->staging, E, c->stream);
    if (e != LANCIUS_ERROR_OK) return e;
    return refresh_weight_splits(c, n->id, d);
}

extern "C" lancius_error lcu_refresh_weights(lcu_ctx* c) {
    if (!c || !c->g) return fail(LANCIUS_ERROR_NULL_PTR);
    cudaSetDevice(c->device);
    for (const auto& w : c->wsplits) {
        lancius_error e = refresh_weight_splits(c, w.node, reinterpret_cast<const float*>(c->dmem + c->off[w.node]));
        if (e != LANCIUS_ERROR_OK) return e;
    }
    return LANCIUS_ERROR_OK;
}

// FP32 device -> host copy queued on the context's stream; returns at once (the data is
// there after lcu_synchronize). With page-locked `host` the copy overlaps other streams'
// work, e.g. the next request's uploads on a second context.
// A node kept NHWC between two convs: transpose it to NCHW (FP32 or FP64) in the staging
// buffer, in stream order; returns the buffer to copy from, or null.
static const void* nchw_view(lcu_ctx* c, const lancius_node* n, const float* d, int f64) {
    if (n->id >= c->nhwc.size() || !c->nhwc[n->id]) return nullptr;
    if (lcu_nhwc_to_nchw(c->staging, d, (int)n->shape[0], (int)n->shape[1], (int)n->shape[2], (int)n->shape[3], f64,
                         c->stream) != LANCIUS_ERROR_OK)
        return nullptr;
    return c->staging;
}

extern "C" lancius_error lcu_download_async(lcu_ctx* c, const lancius_node* n, void* host) {
    float* d; size_t E;
    if (!host) return fail(LANCIUS_ERROR_NULL_PTR);
    if (!node_slot(c, n, &d, &E)) return fail(LANCIUS_ERROR_NULL_PTR);
    cudaSetDevice(c->device);
    if (const void* v = nchw_view(c, n, d, 0))
        return cuda_fail(cudaMemcpyAsync(host, v, E * 4, cudaMemcpyDeviceToHost, c->stream));
    return cuda_fail(cudaMemcpyAsync(host, d, E * 4, cudaMemcpyDeviceToHost, c->stream));
}

extern "C" lancius_error lcu_download(lcu_ctx* c, const lancius_node* n, void* host, lancius_dtype dt) {
    float* d; size_t E;
    if (!host) return fail(LANCIUS_ERROR_NULL_PTR);
    if (!node_slot(c, n, &d, &E)) return fail(LANCIUS_ERROR_NULL_PTR);
    cudaSetDevice(c->device);
    cudaError_t ce;
    const bool nhwc = n->id < c->nhwc.size() && c->nhwc[n->id];
    if (nhwc && E > c->staging_elems) return fail(LANCIUS_ERROR_SHAPE_MISMATCH);
    if (dt == LANCIUS_DTYPE_FP32) {
        const void* v = nhwc ? nchw_view(c, n, d, 0) : d;
        if (!v) return fail(LANCIUS_ERROR_INTERNAL);
        ce = cudaMemcpyAsync(host, v, E * 4, cudaMemcpyDeviceToHost, c->stream);
    } else if (dt == LANCIUS_DTYPE_FP64) {
        if (E > c->staging_elems) return fail(LANCIUS_ERROR_SHAPE_MISMATCH);
        if (nhwc) {
            if (!nchw_view(c, n, d, 1)) return fail(LANCIUS_ERROR_INTERNAL);
        } else {
            lancius_error e = lcu_convert_f32_to_f64(c->staging, d, E, c->stream);
            if (e != LANCIUS_ERROR_OK) return e;
        }
        ce = cudaMemcpyAsync(host, c->staging, E * 8, cudaMemcpyDeviceToHost, c->stream);
    } else {
        return fail(LANCIUS_ERROR_UNSUPPORTED_DTYPE);
    }
    if (ce != cudaSuccess) return cuda_fail(ce);
    return lcu_synchronize(c);    // also reports a tripped watchdog of the kernels that produced it
}

extern "C" lancius_error lcu_upload_bound_inputs(lcu_ctx* c) {
    if (!c || !c->g) return fail(LANCIUS_ERROR_NULL_PTR);
    for (uint32_t i = 0; i < c->g->node_count; i++) {
        const lancius_node* n = c->g->nodes[i];
        if (n->op == LANCIUS_OP_INPUT && n->dtype == LANCIUS_DTYPE_INT8 && n->runtime_data_int8) {
            lancius_error e = lcu_upload(c, n, n->runtime_data_int8, LANCIUS_DTYPE_INT8);
            if (e != LANCIUS_ERROR_OK) return e;
        } else if (n->op == LANCIUS_OP_INPUT && n->runtime_data) {
            lancius_error e = lcu_upload(c, n, n->runtime_data, LANCIUS_DTYPE_FP64);
            if (e != LANCIUS_ERROR_OK) return e;
        }
    }
    return LANCIUS_ERROR_OK;
}

extern "C" void* lcu_host_alloc(size_t bytes) {
    void* p = nullptr;
    if (cudaMallocHost(&p, bytes ? bytes : 1) != cudaSuccess) { cudaGetLastError(); lancius_set_error(LANCIUS_ERROR_OOM); return nullptr; }
    return p;
}
extern "C" void lcu_host_free(void* p) { if (p) cudaFreeHost(p); }

// ---------------------------------------------------------------------------
// execution

static lancius_error run_misc(const Step& s, char* base, void* scratch, const int8_t* packed, void* st) {
    auto F = [&](size_t off) { return reinterpret_cast<float*>(base + off); };
    switch (s.lop) {
        case LANCIUS_OP_MATMUL:
            return lcu_matmul_int8(F(s.out), F(s.in0), reinterpret_cast<const int8_t*>(base + s.in1), s.dscale, s.M, s.K, s.N,
                                   s.packed_off == (size_t)-1 ? nullptr : packed + s.packed_off, F(s.table_off), scratch, st);
        case LANCIUS_OP_CONV2D: case LANCIUS_OP_CONV2D_RELU_FUSED:
            return lcu_conv2d_int8(F(s.out), F(s.in0), reinterpret_cast<const int8_t*>(base + s.in1), s.dscale, s.cn, s.ci, s.h,
                                   s.w, s.co, s.kh, s.kw, s.stride, s.pad, s.lop == LANCIUS_OP_CONV2D_RELU_FUSED,
                                   F(s.table_off), scratch, st);
        case LANCIUS_OP_SUM: return lcu_sum(F(s.out), F(s.in0), s.n, st);
        case LANCIUS_OP_SUM_AXIS0: return lcu_sum_axis0(F(s.out), F(s.in0), s.rows, s.cols, st);
        case LANCIUS_OP_TRANSPOSE: return lcu_transpose(F(s.out), F(s.in0), s.rows, s.cols, st);
        case LANCIUS_OP_RELU_BWD: return lcu_relu_bwd(F(s.out), F(s.in0), F(s.in1), s.n, st);
        case LANCIUS_OP_SOFTMAX_BWD: return lcu_softmax_bwd(F(s.out), F(s.in0), F(s.in1), s.rows, s.cols, st);
        case LANCIUS_OP_CROSS_ENTROPY: return lcu_cross_entropy(F(s.out), F(s.in0), F(s.in1), s.rows, s.cols, st);
        case LANCIUS_OP_CROSS_ENTROPY_BWD:
            return lcu_cross_entropy_bwd(F(s.out), F(s.in0), F(s.in1), F(s.in2), s.rows, s.cols, st);
        case LANCIUS_OP_RMSNORM: return lcu_rmsnorm(F(s.out), F(s.in0), F(s.in1), s.rows, s.cols, 1e-5f, st);
        case LANCIUS_OP_SWIGLU: return lcu_swiglu(F(s.out), F(s.in0), F(s.in1), s.n, st);
        case LANCIUS_OP_GQA: return lcu_gqa(F(s.out), F(s.in0), F(s.in1), F(s.in2), s.S, s.H, s.co, s.D, st);
        case LANCIUS_OP_MAXPOOL2D_BWD:
            return lcu_maxpool2d_bwd(F(s.out), F(s.in0), F(s.in1), s.cn, s.ci, s.h, s.w, s.kh, s.stride, st);
        case LANCIUS_OP_CONV2D_BWD:
            return lcu_conv2d_bwd(F(s.out), F(s.in0), F(s.in2), s.cn, s.ci, s.h, s.w, s.co, s.M, s.N, s.kh, s.kw, s.stride, s.pad, st);
        case LANCIUS_OP_CONV2D_BWD_W:
            return lcu_conv2d_bwd_w(F(s.out), F(s.in0), F(s.in1), s.cn, s.ci, s.h, s.w, s.co, s.M, s.N, s.kh, s.kw, s.stride, s.pad, st);
        default:
            lancius_set_error(LANCIUS_ERROR_UNSUPPORTED_OP);
            return LANCIUS_ERROR_UNSUPPORTED_OP;
    }
}

static lancius_error run_steps(lcu_ctx* c) {
    char* base = c->dmem;
    void* st = c->stream;
    auto F = [&](size_t off) { return reinterpret_cast<float*>(base + off); };
    for (const Step& s : c->steps) {
        lancius_error e = LANCIUS_ERROR_OK;
        switch (s.kind) {
            case S_GEMM:
                if (s.tc) {
                    LcuTcGemmPlan& p = c->tc_plans[s.plan_idx];
                    int passes = lcu_gemm_passes(c->mode);
                    if (p.passes != passes || p.M != s.M) {
                        e = lcu_gemm_tc_prepare(&p, c->scratch, s.M, s.N, s.K, s.count, s.ga, s.gb, passes);
                        if (e != LANCIUS_ERROR_OK) break;
                        if (s.wsplit_off != NPOS && passes > 0) {
                            const size_t mat = s.K * ((s.N + 3) & ~size_t(3));
                            float* hi = c->wsplit + s.wsplit_off;
                            e = lcu_gemm_tc_use_presplit_b(&p, hi, hi + s.gb * mat);
                            if (e != LANCIUS_ERROR_OK) break;
                        }
                        if (s.amap_idx >= 0 && passes > 0 && (e = lcu_gemm_tc_use_raw_a(&p, c->amaps + s.amap_idx)) != LANCIUS_ERROR_OK) break;
                    }
                    e = lcu_gemm_tc_run(&p, (const LcuGemmGroup*)(base + s.table_off), s.epi, st);
                } else {
                    e = lcu_gemm_simt_grouped((const LcuGemmGroup*)(base + s.table_off), s.count, s.M, s.N, s.K, s.epi, st);
                }
                break;
            case S_MLP2:
                e = lcu_mlp2((const LcuGemmGroup*)(base + s.table_off), (const LcuGemmGroup*)(base + s.table2_off), s.M, s.N,
                             s.K, s.epi, s.N2, s.epi2, reinterpret_cast<unsigned*>(base + s.ticket_off), st);
                break;
            case S_ATTN:
                if (lcu_attention_tc_supported(s.D) && !lcu_force_simt())
                    e = lcu_attention_tc((const LcuAttnGroup*)(base + s.table_off), nullptr, nullptr, nullptr, nullptr,
                                         (size_t)s.count, s.S, s.H, s.causal, lcu_contraction_mode(c->mode),
                                         s.amap_idx >= 0 ? c->amaps + s.amap_idx : nullptr, s.attn_lo, st);
                else
                    e = lcu_attention_simt((const LcuAttnGroup*)(base + s.table_off), nullptr, nullptr, nullptr, nullptr,
                                           (size_t)s.count, s.S, s.H, s.D, s.causal, st);
                break;
            case S_LN:
                e = lcu_layernorm_grouped((const LcuRowGroup*)(base + s.table_off), s.count,
                                          LcuRowGroup{nullptr, nullptr, nullptr, nullptr}, s.rows, s.cols, s.eps, s.vec, st);
                break;
            case S_ELT:
                e = lcu_eltwise_grouped(s.op, (const LcuEltGroup*)(base + s.table_off), s.count, s.n, s.vec, st);
                break;
            case S_SOFTMAX: e = lcu_softmax(F(s.out), F(s.in0), s.rows, s.cols, st); break;
            case S_SUMAX1:
                if (s.gap_src >= 0 && c->steps[s.gap_src].gap_done)
                    e = lcu_conv_gap_sum(F(s.out), c->gap_buf + s.gap_off, (int)c->steps[s.gap_src].cn,
                                         (int)c->steps[s.gap_src].co, s.gap_tiles, st);
                else
                    e = lcu_sum_axis1(F(s.out), F(s.in0), s.rows, s.cols, st);
                break;
            case S_BCAST: e = lcu_broadcast(F(s.out), F(s.in0), s.in_elems, s.rows, s.cols, st); break;
            case S_CONV:
                s.gap_done = 0;
                if (s.tc) {
                    const size_t ho = (s.h + 2 * s.pad - s.kh) / s.stride + 1, wo = (s.w + 2 * s.pad - s.kw) / s.stride + 1;
                    const LcuConvShape cs{(int)s.cn, (int)s.ci, (int)s.h, (int)s.w, (int)s.co, (int)s.kh, (int)s.kw,
                                          (int)s.stride, (int)s.pad, (int)ho, (int)wo};
                    if (lcu_conv_nhwc_supported(cs) && !lcu_conv_force_im2col()) {
                        e = lcu_conv2d_tc_nhwc_ex(F(s.out), F(s.in0), F(s.in1), cs, s.relu, lcu_contraction_mode(c->mode), c->scratch, st,
                                                  s.in_nhwc, s.out_nhwc, s.in_lo != NPOS ? c->lo_buf + s.in_lo : nullptr,
                                                  s.out_lo != NPOS ? c->lo_buf + s.out_lo : nullptr,
                                                  s.wsplit_off != NPOS ? c->wsplit + s.wsplit_off : nullptr,
                                                  s.wsplit_off != NPOS ? c->wsplit + s.wsplit_off + align_up((size_t)s.co * s.K, 64)
                                                                       : nullptr,
                                                  s.gap_off != NPOS ? c->gap_buf + s.gap_off : nullptr, &s.gap_done);
                        break;
                    }
                    LcuTcGemmPlan& p = c->tc_plans[s.plan_idx];
                    int passes = lcu_gemm_passes(lcu_contraction_mode(c->mode));
                    if (p.passes != passes || p.M != s.M) {
                        e = lcu_gemm_tc_prepare(&p, c->scratch, s.M, s.N, s.K, 1, 1, 1, passes);
                        if (e != LANCIUS_ERROR_OK) break;
                        size_t ho = (s.h + 2 * s.pad - s.kh) / s.stride + 1, wo = (s.w + 2 * s.pad - s.kw) / s.stride + 1;
                        p.conv = LcuConvShape{(int)s.cn, (int)s.ci, (int)s.h, (int)s.w, (int)s.co, (int)s.kh, (int)s.kw,
                                              (int)s.stride, (int)s.pad, (int)ho, (int)wo};
                    }
                    e = lcu_gemm_tc_run(&p, (const LcuGemmGroup*)(base + s.table_off), s.relu ? LCU_EPI_RELU : LCU_EPI_NONE, st);
                    break;
                }
                if (s.out_nhwc)
                    e = lcu_conv2d_smallk_ex(F(s.out), F(s.in0), F(s.in1), s.cn, s.ci, s.h, s.w, s.co, s.kh, s.kw, s.stride,
                                             s.pad, s.relu, 1, st, s.out_lo != NPOS ? c->lo_buf + s.out_lo : nullptr);
                else
                    e = lcu_conv2d(F(s.out), F(s.in0), F(s.in1), s.cn, s.ci, s.h, s.w, s.co, s.kh, s.kw, s.stride, s.pad,
                                   s.relu, lcu_contraction_mode(c->mode), st);
                break;
            case S_MAXPOOL: e = lcu_maxpool2d(F(s.out), F(s.in0), s.cn, s.ci, s.h, s.w, s.kh, s.stride, st); break;
            case S_MISC: e = run_misc(s, base, c->scratch, c->packed, st); break;
        }
        if (e != LANCIUS_ERROR_OK) return e;
    }
    return LANCIUS_ERROR_OK;
}

extern "C" void lancius_schedule_execute_cuda(lancius_schedule* s, lcu_ctx* c) {
    if (!c || !s) { lancius_set_error(LANCIUS_ERROR_NULL_PTR); return; }
    if (s != c->s || !c->dmem) { lancius_set_error(LANCIUS_ERROR_INVALID_MODEL); return; }
    cudaSetDevice(c->device);
    lcu_reset_launch_count();
    if (!c->replay) {
        run_steps(c);
        c->last_launches = lcu_launch_count();
        return;
    }
    if (!c->exec) {
        cudaGraph_t graph = nullptr;
        cudaError_t ce = cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal);
        if (ce != cudaSuccess) { cuda_fail(ce); return; }
        lancius_error e = run_steps(c);
        ce = cudaStreamEndCapture(c->stream, &graph);
        if (e != LANCIUS_ERROR_OK || ce != cudaSuccess) {
            if (graph) cudaGraphDestroy(graph);
            if (ce != cudaSuccess) cuda_fail(ce);
            return;
        }
        ce = cudaGraphInstantiate(&c->exec, graph, 0);
        cudaGraphDestroy(graph);
        if (ce != cudaSuccess) { c->exec = nullptr; cuda_fail(ce); return; }
        c->graph_launches = lcu_launch_count();
    }
    cuda_fail(cudaGraphLaunch(c->exec, c->stream));
    c->last_launches = c->graph_launches;
}
