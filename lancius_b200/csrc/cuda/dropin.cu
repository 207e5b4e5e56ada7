// The reference's own executors, lancius_schedule_execute / _parallel / _static
// (bleeding/v11A1/src/runtime/lancius_scheduler.c:311-413,475-520), with their names,
// arguments and host memory contract kept and the math moved to the GPU, so a Lancius
// program (examples/run_edge.c, the stable FFI) links against this library unchanged.
//
// Per call:
//   1. every computed node gets host runtime_data exactly as the reference places it
//      (arena / attached pool for _execute and _parallel, a 32-byte aligned bump over
//      flat_buffer in wave order for _static); CONST nodes are filled on the host too;
//   2. the calling thread's implicit device context binds the schedule once (the
//      binding is reused while the waves hold the same nodes with the same shapes,
//      so callers that rebuild the schedule per run do not re-plan the device);
//   3. bound INPUT data (FP64, or INT8 weights) is uploaded, the schedule runs on the
//      device (replayed from a CUDA graph after the first run), and the outputs are
//      copied back as FP64 into their runtime_data.
#include "lcu_internal.h"
#include "lancius/lancius_arena.h"
#include "lancius/lancius_threadpool.h"

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <unordered_set>
#include <vector>

namespace {

struct NodeKey {                    // what a binding depends on, per node in wave order
    const lancius_node* n;
    int op;
    size_t shape[4];
    uint8_t ndim;
    uint32_t kh, kw, stride, pad;
    double attr;
    int dtype;
    const void* in[3];
    bool operator==(const NodeKey& o) const { return std::memcmp(this, &o, sizeof(NodeKey)) == 0; }
};

NodeKey key_of(const lancius_node* n) {
    NodeKey k;
    std::memset(&k, 0, sizeof(k));  // padding bytes take part in the comparison
    k.n = n; k.op = n->op; k.ndim = n->ndim;
    for (int i = 0; i < 4; i++) k.shape[i] = n->shape[i];
    k.kh = n->kernel_h; k.kw = n->kernel_w; k.stride = n->stride; k.pad = n->pad;
    k.attr = n->attr_val; k.dtype = n->dtype;
    for (uint32_t i = 0; i < n->input_count && i < 3; i++) k.in[i] = n->inputs[i];
    return k;
}

struct Implicit {
    lcu_ctx* ctx = nullptr;
    int all = -1;                      // binding made for "download every node"
    std::vector<NodeKey> key;
    std::vector<lancius_node*> nodes;  // the proxy graph's node table (sorted by id)
    lancius_graph proxy{};
    std::vector<lancius_node*> outs;   // nodes copied back after each run
};
thread_local Implicit tl;
thread_local int tl_force_all = 0;

bool download_all() {
    const char* v = std::getenv("LCU_DROPIN_DOWNLOAD_ALL");
    return tl_force_all || (v && v[0] == '1');
}

int device_index() {
    const char* v = std::getenv("LANCIUS_CUDA_DEVICE");
    return v ? std::atoi(v) : 0;
}

bool computed(const lancius_node* n) {
    return n->op != LANCIUS_OP_INPUT && n->op != LANCIUS_OP_CONST && n->op != LANCIUS_OP_NOP;
}

// Binds (or re-uses the binding of) the schedule on this thread's device context.
lancius_error bind(lancius_schedule* s, bool all) {
    std::vector<NodeKey> key;
    for (uint32_t w = 0; w < s->wave_count; w++)
        for (uint32_t i = 0; i < s->waves[w].node_count; i++) key.push_back(key_of(s->waves[w].nodes[i]));
    if (!tl.ctx) {
        tl.ctx = lcu_create(device_index());
        if (!tl.ctx) return lancius_get_error();
        lcu_set_graph_replay(tl.ctx, 1);
        const char* m = std::getenv("LANCIUS_CUDA_MODE");   // "tf32" / "bf16": the fast modes
        if (m && !std::strcmp(m, "tf32")) lcu_set_mode(tl.ctx, LCU_MODE_TF32);
        if (m && !std::strcmp(m, "bf16")) lcu_set_mode(tl.ctx, LCU_MODE_BF16);
    }
    if (tl.all == (int)all && key == tl.key) {
        lcu_ctx_retarget_schedule(tl.ctx, s);
        return LANCIUS_ERROR_OK;
    }
    // The schedule holds every node of its graph (INPUTs in the first wave); the proxy
    // graph gives the device binding the node table it walks, indexed by id.
    tl.nodes.clear();
    uint32_t next_id = 0;
    std::unordered_set<const lancius_node*> members;
    for (auto& k : key) {
        tl.nodes.push_back(const_cast<lancius_node*>(k.n));
        members.insert(k.n);
        next_id = std::max(next_id, k.n->id + 1);
    }
    for (auto& k : key)
        for (uint32_t j = 0; j < k.n->input_count; j++)
            if (k.n->inputs[j] && !members.count(k.n->inputs[j])) {
                lancius_set_error(LANCIUS_ERROR_INVALID_MODEL);   // an input outside the schedule
                return LANCIUS_ERROR_INVALID_MODEL;
            }
    std::sort(tl.nodes.begin(), tl.nodes.end(), [](const lancius_node* a, const lancius_node* b) { return a->id < b->id; });
    tl.proxy = lancius_graph{};
    tl.proxy.nodes = tl.nodes.data();
    tl.proxy.node_count = tl.proxy.node_cap = (uint32_t)tl.nodes.size();
    tl.proxy.next_id = next_id;
    std::vector<uint8_t> read(next_id, 0);
    for (auto* n : tl.nodes)
        for (uint32_t j = 0; j < n->input_count; j++)
            if (n->inputs[j]) read[n->inputs[j]->id] = 1;
    tl.outs.clear();
    for (auto* n : tl.nodes)
        if (computed(n) && (all || !read[n->id])) tl.outs.push_back(n);
    tl.key.clear();
    tl.all = -1;
    lcu_set_fusion(tl.ctx, all ? 0 : 1);
    lancius_error e = lcu_bind_plan(tl.ctx, s, &tl.proxy, nullptr);
    if (e != LANCIUS_ERROR_OK) return e;
    tl.key = std::move(key);
    tl.all = all ? 1 : 0;
    return LANCIUS_ERROR_OK;
}

void fill_const(lancius_node* n) {
    const size_t e = lancius_node_elements(n);
    for (size_t k = 0; k < e; k++) n->runtime_data[k] = n->attr_val;
}

// Host placement of the arena executors (scheduler.c:329-357): a node without
// runtime_data gets the attached pool's slot when the plan pools it, else arena memory.
bool place_arena(lancius_schedule* s, lancius_arena* scratch) {
    for (uint32_t w = 0; w < s->wave_count; w++)
        for (uint32_t i = 0; i < s->waves[w].node_count; i++) {
            lancius_node* n = s->waves[w].nodes[i];
            lancius_runtime_sync_from_legacy(n);
            if (n->op == LANCIUS_OP_INPUT || n->op == LANCIUS_OP_NOP || n->runtime_data) continue;
            const bool pooled = s->plan && s->plan->is_pooled[n->id] && s->static_pool;
            n->runtime_data = pooled ? reinterpret_cast<double*>(static_cast<uint8_t*>(s->static_pool) + s->plan->offsets[n->id])
                                     : static_cast<double*>(lancius_arena_alloc(scratch, lancius_node_bytes(n), 32));
            lancius_node_set_owner(n, pooled ? LANCIUS_MEMORY_POOL : LANCIUS_MEMORY_ARENA);
            if (!n->runtime_data) { lancius_set_error(LANCIUS_ERROR_OOM); return false; }
            if (n->op == LANCIUS_OP_CONST) fill_const(n);
        }
    return true;
}

// Host placement of the static executor (scheduler.c:481-506): every computed node, in
// wave order, at the next 32-byte boundary of flat_buffer; no reuse.
void place_static(lancius_schedule* s, void* flat) {
    size_t off = 0;
    for (uint32_t w = 0; w < s->wave_count; w++)
        for (uint32_t i = 0; i < s->waves[w].node_count; i++) {
            lancius_node* n = s->waves[w].nodes[i];
            if (n->op == LANCIUS_OP_INPUT || n->op == LANCIUS_OP_CONST) continue;
            off = (off + 31) & ~size_t(31);
            n->runtime_data = reinterpret_cast<double*>(static_cast<char*>(flat) + off);
            if (n->rt) {
                n->rt->buffer = n->runtime_data;
                n->rt->offset = off;
            }
            lancius_node_set_owner(n, LANCIUS_MEMORY_POOL);
            off += lancius_node_bytes(n);
        }
}

void run_on_device(lancius_schedule* s) {
    const bool all = download_all();
    if (bind(s, all) != LANCIUS_ERROR_OK) return;
    if (lcu_upload_bound_inputs(tl.ctx) != LANCIUS_ERROR_OK) return;
    lancius_clear_error();
    lancius_schedule_execute_cuda(s, tl.ctx);
    if (lancius_get_error() != LANCIUS_ERROR_OK) return;
    for (auto* n : tl.outs)
        if (n->runtime_data && lcu_download(tl.ctx, n, n->runtime_data, LANCIUS_DTYPE_FP64) != LANCIUS_ERROR_OK) return;
    lcu_synchronize(tl.ctx);
}

}  // namespace

extern "C" void lancius_schedule_execute(lancius_schedule* s, lancius_arena* scratch) {
    if (!s) return;
    if (!place_arena(s, scratch)) return;
    run_on_device(s);
}

extern "C" void lancius_schedule_execute_parallel(lancius_schedule* s, lancius_arena* scratch, lancius_pool* pool) {
    if (!s || !pool) return;
    if (!place_arena(s, scratch)) return;
    run_on_device(s);
}

extern "C" void lancius_schedule_execute_static(lancius_schedule* s, void* flat_buffer) {
    if (!s || !flat_buffer) return;
    place_static(s, flat_buffer);
    run_on_device(s);
}

// The stable FFI lets a caller read any tensor after a run (lancius_read_output), so its
// runs copy back every computed node (stable_api.c sets this around its execute call).
extern "C" void lcu_dropin_force_all(int on) { tl_force_all = on ? 1 : 0; }

extern "C" void lancius_dropin_release(void) {
    if (tl.ctx) lcu_destroy(tl.ctx);
    tl.ctx = nullptr;
    tl.key.clear();
    tl.nodes.clear();
    tl.outs.clear();
    tl.all = -1;
}
