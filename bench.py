"""Benchmark for the Lancius B200 backend (one JSON line on rank 0).

Default workload: FP32 causal multi-head attention, batch 8
x seq 512 x 8 heads x head_dim 64 per GPU, built through the Lancius graph API and
run by lancius_schedule_execute_cuda. Metric: attention GB/s (algorithmic bytes =
Q,K,V read + O written once, FP32 = 16*B*S*H*D per graph). Weak scaling: every
rank runs its own batch of 8; there is no data-path collective.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
                  [--config attention|mlp|conv|encoder|encoder_b256|gemm4096|decode|...]
"""
import argparse
import ctypes as C
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

L2_FLUSH_BYTES = 256 << 20     # > 126 MB L2: written between timed steps
L2_NOTE = "flushed between timed steps (256 MiB write, then read back: no dirty lines left)"


def flush_l2(buf):
    """Evict L2 between timed steps: write a buffer twice its size, then read it back, so
    the lines left behind are clean and the next step pays no write-back of this buffer."""
    buf.fill_(1.0)
    buf.sum()


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return {"hbm_gbs": p["hbm_gbs"], "bf16_tflops": p["bf16_tflops"], "src": "measured"}
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "src": "fallback"}


# per-config workload description -------------------------------------------------
def build(cfg, graph, rank, world=1):
    from lancius_b200 import configs
    if cfg == "attention":
        return configs.attention(graph, batch=8, seq=512, heads=8, head_dim=64, seed=1 + 1000 * rank)
    if cfg == "mlp":
        return configs.mlp(graph, batch=64, seed=0 + 1000 * rank)
    if cfg == "conv":
        return configs.conv_stack(graph, batch=32, hw=224, seed=2 + 1000 * rank)
    if cfg == "encoder":
        return configs.encoder(graph, batch=16, seq=512, layers=12, seed=3, first=16 * rank)
    if cfg == "encoder_b256":      # batch 256 sharded over the ranks
        from lancius_b200.shard import shard_range
        lo, hi = shard_range(256, rank, world)
        return configs.encoder(graph, batch=hi - lo, seq=512, layers=12, seed=3, first=lo)
    if cfg.startswith("gemm"):
        return configs.gemm(graph, int(cfg[4:]), seed=4 + 1000 * rank)
    raise SystemExit(f"unknown config {cfg}")


METRIC = {
    "attention": ("attention GB/s", "GB/s", "attention_b8_s512_h8_d64_causal_fp32"),
    "mlp": ("graph inferences/sec", "graphs/s", "mlp_784_256_10_b64_fp32"),
    "conv": ("conv stack TFLOP/s", "TFLOP/s", "conv_stack_b32_224_fp32"),
    "encoder": ("encoder TFLOP/s", "TFLOP/s", "encoder_bert_base_l12_b16_s512_fp32"),
    "encoder_b256": ("encoder TFLOP/s", "TFLOP/s", "encoder_bert_base_l12_b256_s512_fp32_batch_sharded"),
}


PER_GPU_BATCH = {"attention": 8, "mlp": 64, "conv": 32, "encoder": 16}


def config_of(cfg, workload):
    """The workload keys both arms print (identical dicts, so the two lines compare)."""
    return {"workload": workload, "per_gpu_batch": PER_GPU_BATCH.get(cfg)}


def attention_traffic():
    """DRAM bytes (read + write) of one k_attn_tc launch, from the committed ncu summary --
    only while the kernel source is the one that capture measured (its sha256 prefix is
    recorded there); None otherwise."""
    import hashlib
    try:
        src = open(os.path.join(ROOT, "lancius_b200", "csrc", "cuda", "attention_tc.cu"), "rb").read()
        txt = open(os.path.join(ROOT, "profiles", "attention_tcgen05_b8_s512_h8_d64.md")).read()
    except OSError:
        return None, None
    h = hashlib.sha256(src).hexdigest()[:16]
    import re
    m = re.search(r"source sha256 \(first 16\): `([0-9a-f]{16})`.*?dram bytes per launch: `(\d+)`", txt, re.S)
    if not m or m.group(1) != h:
        return None, h
    return int(m.group(2)), h


def metric_of(cfg, built, seconds_per_graph):
    if cfg in ("attention",):
        return built.bytes / seconds_per_graph / 1e9
    if cfg == "mlp":
        return 1.0 / seconds_per_graph
    return built.flops / seconds_per_graph / 1e12   # conv, encoder, gemm: TFLOP/s


def metric_names(cfg):
    if cfg == "decode":
        return ("decode attention GB/s", "GB/s", "kv_cache_decode_b{batch}_s{seq}_h{heads}_d{head_dim}_fp32".format(**DECODE))
    if cfg in METRIC:
        return METRIC[cfg]
    return ("GEMM TFLOP/s", "TFLOP/s", f"{cfg}_square_fp32")


# clocks sampled during the timed region --------------------------------------------
class Clocks:
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-i", str(self.gpu), "-lms", "200"], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for nm, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# CPU baseline: the reference's own code (oracle/_ref) on this host's cores -----------
def _all_host_threads():
    """torchrun sets OMP_NUM_THREADS=1 for multi-rank jobs; the reference CPU path must
    use every host core, so raise the OpenMP team size explicitly."""
    try:
        gomp = C.CDLL("libgomp.so.1")
        gomp.omp_set_num_threads(os.cpu_count())
    except OSError:
        pass
    return os.cpu_count()


def _ref_sample(cfg):
    """One bounded sample of `cfg` for the reference's own CPU executor: (graph builder,
    factor from the sample's time to one full unit of the metric, description)."""
    from lancius_b200 import configs
    if cfg == "attention":
        return (lambda g: configs.attention(g, batch=8, seq=512, heads=8, head_dim=64, seed=1)), 1.0, \
            "the full batch-8 graph (S512 H8 D64 causal)"
    if cfg == "mlp":
        return (lambda g: configs.mlp(g, batch=64, seed=0)), 1.0, "the full batch-64 graph"
    if cfg == "conv":
        return (lambda g: configs.conv_stack(g, batch=1, hw=224, seed=2)), 32.0, \
            "1 of 32 images through the conv stack, scaled x32"
    if cfg in ("encoder", "encoder_b256"):
        nb = 16 if cfg == "encoder" else 256
        # the reference's ATTENTION is always causal; it still visits every key (masking by
        # -1e9), so its cost equals the unmasked attention of this config
        return (lambda g: configs.encoder(g, batch=1, seq=512, layers=1, seed=3, causal=True)), 12.0 * nb, \
            f"1 layer of 1 sequence (S512, d768; causal ATTENTION node, same cost), scaled x12 layers x{nb} sequences"
    if cfg.startswith("gemm"):
        n = int(cfg[4:])
        ns = min(n, 1024)
        return (lambda g: configs.gemm(g, ns, seed=4)), (n / ns) ** 3, \
            f"a {ns}^3 product, scaled by (N/{ns})^3 to {n}^3 (the reference MATMUL is one thread, i-k-j)"
    return None


def _ref_run_seconds(ref, build, min_s=3.0, max_reps=None):
    """Seconds per run of the sample graph through lancius_schedule_execute (arena mode),
    and the sample's Built record (its algorithmic FLOPs and bytes)."""
    import oracle
    from lancius_b200 import Graph
    g = Graph(ref)
    b = build(g)
    b.bind_host()
    t0 = time.perf_counter()
    reps = 0
    while True:
        oracle.run_reference_graph(ref, g, b.outputs[:1], arena_bytes=512 << 20)
        reps += 1
        if time.perf_counter() - t0 > min_s or (max_reps and reps >= max_reps):
            break
    return (time.perf_counter() - t0) / reps, reps, b


def _sample_value(cfg, b, sec):
    """The metric's throughput measured on the sample (the scaling factor cancels)."""
    if cfg == "mlp":
        return 1.0 / sec
    if cfg == "attention":
        return b.bytes / sec / 1e9
    return b.flops / sec / 1e12


def cpu_baseline(cfg, steps=None):
    """Times the reference's arena-mode executor on a bounded sample of the workload.
    Returns (value in the metric's unit, description dict)."""
    import oracle
    if not oracle.reference_available():
        return None
    smp = _ref_sample(cfg)
    if smp is None:
        return None
    ref = oracle.reference()
    cores = _all_host_threads()
    build, factor, what = smp
    sec, reps, b = _ref_run_seconds(ref, build, max_reps=steps)
    return _sample_value(cfg, b, sec), {
        "kind": "reference", "cores": cores,
        "sample": f"{reps} runs of {what} through lancius_schedule_execute; OpenMP threads = {cores}"}


# the B200 arm -----------------------------------------------------------------------
def run_b200(args, rank, world, local_rank):
    import torch
    import lancius_b200 as L

    torch.cuda.set_device(local_rank)
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=torch.device("cuda", local_rank))

    mode = {"tf32": L.MODE_TF32, "bf16": L.MODE_BF16}.get(args.mode, L.MODE_FP32_EXACT)
    dev = L.Device(local_rank, mode)
    g = L.Graph()
    built = build(args.config, g, rank, world)
    sched = g.schedule()
    dev.set_graph_replay(True)
    dev.bind(sched)
    for node, arr in built.inputs:
        dev.upload(node, arr)

    ext = torch.cuda.ExternalStream(dev.stream)
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device="cuda")

    def step_device(ev0, ev1):
        with torch.cuda.stream(ext):
            flush_l2(flush)                 # evict L2 between timed steps
            ev0.record(ext)
        dev.execute(sched)
        with torch.cuda.stream(ext):
            ev1.record(ext)

    for _ in range(args.warmup):
        step_device(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
    torch.cuda.synchronize()

    clocks = Clocks(local_rank)
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    clocks.start()
    for e0, e1 in evs:
        step_device(e0, e1)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    clk = clocks.stop()
    dev_ms = [e0.elapsed_time(e1) for e0, e1 in evs]
    launches_per_step = dev.last_launch_count
    total_ms = sum(dev_ms)

    # e2e through the public API with pinned host buffers: every step uploads its inputs
    # (H2D), executes and downloads its outputs (D2H). Requests alternate between two
    # contexts (each with its own stream and copy of the graph), so one request's D2H and
    # the next one's H2D overlap on the full-duplex link, as a server pipelines requests.
    g2 = L.Graph()
    built2 = build(args.config, g2, rank, world)
    sched2 = g2.schedule()
    dev2 = L.Device(local_rank, mode)
    dev2.set_graph_replay(True)
    dev2.bind(sched2)
    for node, arr in built2.inputs:
        dev2.upload(node, arr)
    in_bytes = sum(arr.size * 4 for _, arr in built.inputs if _is_activation(args.config, _))
    out_bytes = sum(o.size * 4 for o in built.outputs)
    lanes = []
    for d, b, sc in ((dev, built, sched), (dev2, built2, sched2)):
        hin = []
        for node, arr in b.inputs:
            if not _is_activation(args.config, node):
                continue
            p = d.lib.lcu_host_alloc(arr.size * 4)
            np.ctypeslib.as_array(C.cast(p, C.POINTER(C.c_float)), shape=(arr.size,))[:] = arr.ravel()
            hin.append((node, p))
        hout = [(o, d.lib.lcu_host_alloc(o.size * 4)) for o in b.outputs]
        lanes.append((d, sc, hin, hout))

    def request(lane):
        d, sc, hin, hout = lane
        for node, p in hin:
            d.upload_ptr(node, p, 2)
        d.execute(sc)
        for node, p in hout:
            rc = d.lib.lcu_download_async(d.ptr, node.ptr, p)
            assert rc == 0, rc

    for i in range(max(2, args.warmup)):
        request(lanes[i % 2])
    dev.synchronize(); dev2.synchronize()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    ext2 = torch.cuda.ExternalStream(dev2.stream)
    e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
    e0.record(ext)
    ext2.wait_event(e0)                      # the second lane starts no earlier than the first
    for i in range(args.steps):
        if i >= 2:
            lanes[i % 2][0].synchronize()    # that lane's previous request has delivered its outputs
        request(lanes[i % 2])
    e1.record(ext)
    e2.record(ext2)
    torch.cuda.synchronize()
    e2e_ms = max(e0.elapsed_time(e1), e0.elapsed_time(e2))
    if dist:
        dist.barrier()
    for d, _, hin, hout in lanes:
        for _, p in hin + hout:
            d.lib.lcu_host_free(p)
    dev2.close()

    dropin_ms = dropin_e2e_ms(args, rank, world, local_rank, dist)
    if dist:
        t = torch.tensor([total_ms, e2e_ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms, e2e_ms = t.tolist()
    built.meta["dropin_ms"] = dropin_ms
    return built, total_ms, e2e_ms, dev_ms, launches_per_step, clk, in_bytes, out_bytes, dist


def dropin_e2e_ms(args, rank, world, local_rank, dist):
    """Milliseconds for args.steps requests through the reference's own entry point as an
    unchanged Lancius program calls it: lancius_schedule_execute_static on a graph whose
    INPUT nodes hold FP64 host arrays (pageable memory). Each call uploads every bound
    input (weights included), runs the schedule on the GPU and copies the outputs back to
    their FP64 host buffers; it returns when they are there. Max over ranks."""
    import torch
    import lancius_b200 as L
    os.environ["LANCIUS_CUDA_DEVICE"] = str(local_rank)
    os.environ["LANCIUS_CUDA_MODE"] = args.mode
    lib = L.load()
    lib.lancius_schedule_execute_static.argtypes = [C.c_void_p, C.c_void_p]
    lib.lancius_schedule_execute_static.restype = None
    lib.lancius_dropin_release.argtypes = []
    g = L.Graph()
    b = build(args.config, g, rank, world)
    b.bind_host()
    sched = g.schedule()
    flat = np.zeros(sum(n.size * 8 + 32 for n in g.nodes()) // 8 + 1)
    fp = flat.ctypes.data_as(C.c_void_p)
    for _ in range(max(2, args.warmup)):
        lib.lancius_schedule_execute_static(sched.ptr, fp)
    if lib.lancius_get_error() != 0:
        raise RuntimeError(f"lancius_schedule_execute_static: error {lib.lancius_get_error()}")
    if dist:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        lib.lancius_schedule_execute_static(sched.ptr, fp)
    ms = (time.perf_counter() - t0) * 1e3
    lib.lancius_dropin_release()
    if dist:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = t.item()
    return ms


def run_colsplit(args, rank, world, local_rank, n):
    """GEMM n^3 split by columns over the ranks: lcu_gemm_colsplit = local 3xTF32 GEMM on
    the rank's slab + NCCL all-gather + repack. Total work fixed (strong scaling)."""
    import torch
    import torch.distributed as dist
    import lancius_b200 as L
    from lancius_b200 import data
    torch.cuda.set_device(local_rank)
    dist.init_process_group("nccl", device_id=torch.device("cuda", local_rank))
    lib = L.load()
    uid = C.create_string_buffer(128)
    if rank == 0:
        assert lib.lcu_comm_unique_id(uid, 128) == 0
    t = torch.tensor(list(uid.raw), dtype=torch.uint8, device="cuda")
    dist.broadcast(t, 0)
    comm = lib.lcu_comm_create(world, rank, C.c_char_p(bytes(t.cpu().tolist())), local_rank)
    assert comm, "lcu_comm_create failed"
    ns = n // world
    a_h = data.uniform(data.sub_seed(4, 1), (n, n), -1, 1).astype(np.float32)
    b_full = data.uniform(data.sub_seed(4, 2), (n, n), -1, 1).astype(np.float32)
    b_h = np.ascontiguousarray(b_full[:, rank * ns:(rank + 1) * ns])
    del b_full
    a = torch.from_numpy(a_h).cuda()
    b = torch.from_numpy(b_h).cuda()
    c = torch.empty((n, n), device="cuda")
    stream = torch.cuda.current_stream()
    sp = C.c_void_p(stream.cuda_stream)
    flush = torch.empty(L2_FLUSH_BYTES // 4, device="cuda")

    # default: the fused kernel (epilogue stores into every rank's C over NVLink);
    # LCU_COLSPLIT_NCCL=1 selects GEMM + ncclAllGather + repack
    nccl_path = os.environ.get("LCU_COLSPLIT_NCCL") == "1"
    fn = lib.lcu_gemm_colsplit if nccl_path else lib.lcu_gemm_colsplit_fused

    def step():
        rc = fn(comm, C.c_void_p(c.data_ptr()), C.c_void_p(a.data_ptr()), C.c_void_p(b.data_ptr()), n, n, n, 0, sp)
        assert rc == 0, rc
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    dist.barrier()
    evs = []
    clocks = Clocks(local_rank)
    clocks.start()
    for _ in range(args.steps):
        flush_l2(flush)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(); step(); e1.record()
        evs.append((e0, e1))
    torch.cuda.synchronize()
    dist.barrier()
    clk = clocks.stop()
    total_ms = sum(e0.elapsed_time(e1) for e0, e1 in evs)
    # e2e: pinned host A and slab in, full C out, every step
    a_pin, b_pin, c_pin = (torch.empty(x.shape, dtype=torch.float32).pin_memory() for x in (a_h, b_h, a_h))
    a_pin.copy_(torch.from_numpy(a_h)); b_pin.copy_(torch.from_numpy(b_h))
    dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        a.copy_(a_pin, non_blocking=True); b.copy_(b_pin, non_blocking=True)
        step()
        c_pin.copy_(c, non_blocking=True)
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1)
    tt = torch.tensor([total_ms, e2e_ms], device="cuda")
    dist.all_reduce(tt, op=dist.ReduceOp.MAX)
    total_ms, e2e_ms = tt.tolist()
    lib.lcu_comm_destroy(comm)
    if rank == 0:
        flops = 2.0 * n ** 3
        pk = peaks()
        val = flops / (total_ms / 1e3 / args.steps) / 1e12
        line = {
            "metric": "GEMM TFLOP/s", "value": round(val, 3), "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(total_ms / args.steps, 4), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded U[-1,1), splitmix64)",
            "config": config_of(f"gemm{n}", metric_names(f"gemm{n}")[2]), "mode": "fp32_exact",
            "exchange": "ncclAllGather + repack" if nccl_path else "fused: epilogue stores to peer C over NVLink",
            "l2": L2_NOTE, "parallelism": f"column-split x{world}",
            "roofline": {"bound": "tensor", "achieved": round(val / world, 2), "peak": pk["bf16_tflops"],
                         "unit": "TFLOP/s per GPU", "frac": round(val / world / pk["bf16_tflops"], 4), "traffic": None,
                         "peak_src": pk["src"] + " bf16 (3xTF32 issues 3 TF32 MMAs per product)"},
            "cpu_baseline": None,
            "e2e": {"value": round(flops / (e2e_ms / 1e3 / args.steps) / 1e12, 3), "unit": "TFLOP/s",
                    "h2d_bytes_per_step": int(a_h.nbytes + b_h.nbytes), "d2h_bytes_per_step": int(4 * n * n)},
            # per step: A and B hi/lo splits, the GEMM, the split-K reduce when K > 8192, and
            # the repack on the NCCL path
            "gpu_launches": (3 + (1 if n > 8192 else 0) + (1 if nccl_path else 0)) * args.steps, "clocks": clk,
        }
        print(json.dumps(line))
    dist.destroy_process_group()


DECODE = dict(batch=32, seq=8192, heads=8, head_dim=128)


def _decode_ref_seconds(ref, q, kc, vc, limit_s=8.0):
    """Seconds per batch of the reference kernel_attention_kv_cache (FP64, one call per
    sequence, sequences spread over all host threads); bounded sample of sequences."""
    from concurrent.futures import ThreadPoolExecutor
    B, S, H, D = kc.shape
    dp = lambda a: a.ctypes.data_as(C.POINTER(C.c_double))
    outs = [np.empty(H * D) for _ in range(B)]
    cores = os.cpu_count()

    def one(b):
        ref.kernel_attention_kv_cache(dp(outs[b]), dp(q[b]), dp(kc[b]), dp(vc[b]), C.c_size_t(S), C.c_size_t(H),
                                      C.c_size_t(D))
    done, t0 = 0, time.perf_counter()
    with ThreadPoolExecutor(cores) as ex:
        while True:
            list(ex.map(one, range(B)))
            done += 1
            if time.perf_counter() - t0 > limit_s:
                break
    return (time.perf_counter() - t0) / done, cores


def run_decode(args, rank, world, local_rank):
    """KV-cache decode attention (kernel_attention_kv_cache) per GPU: a batch of
    sequences, one new query token each, against resident FP32 caches. Weak scaling."""
    import torch
    import lancius_b200 as L
    from lancius_b200 import data
    torch.cuda.set_device(local_rank)
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=torch.device("cuda", local_rank))
    lib = L.load()
    B, S, H, D = DECODE["batch"], DECODE["seq"], DECODE["heads"], DECODE["head_dim"]
    g = torch.Generator(device="cuda").manual_seed(7 + rank)
    kc = torch.randn((B, S, H, D), device="cuda", generator=g)
    vc = torch.randn((B, S, H, D), device="cuda", generator=g)
    q_h = data.normal(8 + rank, (B, H * D)).astype(np.float32)
    q = torch.from_numpy(q_h).cuda()
    out = torch.empty((B, H * D), device="cuda")
    stream = torch.cuda.current_stream()
    sp = C.c_void_p(stream.cuda_stream)
    ptr = lambda t: C.c_void_p(t.data_ptr())
    flush = torch.empty(L2_FLUSH_BYTES // 4, device="cuda")

    def step():
        rc = lib.lcu_attention_kv_cache_batched(ptr(out), ptr(q), ptr(kc), ptr(vc), B, S, H, D, sp)
        assert rc == 0, rc
    for _ in range(args.warmup):
        flush_l2(flush); step()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    clocks = Clocks(local_rank)
    clocks.start()
    evs = []
    for _ in range(args.steps):
        flush_l2(flush)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(); step(); e1.record()
        evs.append((e0, e1))
    torch.cuda.synchronize()
    clk = clocks.stop()
    dev_ms = [e0.elapsed_time(e1) for e0, e1 in evs]
    total_ms = sum(dev_ms)
    # e2e: the caches stay resident (they are the decoder's state); each step copies the
    # new query tokens in from pinned memory and the attention output back
    q_pin = torch.from_numpy(q_h).pin_memory()
    o_pin = torch.empty((B, H * D)).pin_memory()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        q.copy_(q_pin, non_blocking=True)
        step()
        o_pin.copy_(out, non_blocking=True)
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1)
    if dist:
        t = torch.tensor([total_ms, e2e_ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms, e2e_ms = t.tolist()
    bytes_ = 4.0 * (2 * B * S * H * D + 2 * B * H * D)
    if rank == 0:
        sec = total_ms / 1e3 / args.steps
        val = bytes_ / sec / 1e9 * world
        pk = peaks()
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            import oracle
            if oracle.reference_available():
                ref = oracle.reference()
                nb = 4   # bounded sample: 4 sequences at the full cache length
                kd, vd = (t[:nb].double().cpu().numpy() for t in (kc, vc))
                qd = q_h[:nb].astype(np.float64)
                rsec, cores = _decode_ref_seconds(ref, qd, kd, vd)
                cpu = {"value": round(4.0 * (2 * nb * S * H * D + 2 * nb * H * D) / rsec / 1e9, 4), "unit": "GB/s",
                       "cores": cores, "kind": "reference",
                       "sample": f"{nb} of {B} sequences (S{S} H{H} D{D}) through kernel_attention_kv_cache, "
                                 "one call per sequence on a thread pool; FP32-equivalent bytes"}
        line = {
            "metric": "decode attention GB/s", "value": round(val, 3), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(total_ms / args.steps, 5),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (N(0,1) caches, seeded)",
            "config": {"workload": f"kv_cache_decode_b{B}_s{S}_h{H}_d{D}_fp32", "per_gpu_batch": B},
            "mode": "fp32", "l2": L2_NOTE + "; caches 2.1 GB > L2",
            "parallelism": f"batch-sharded x{world}",
            "roofline": {"bound": "hbm", "achieved": round(bytes_ / sec / 1e9, 1), "peak": pk["hbm_gbs"],
                         "unit": "GB/s", "frac": round(bytes_ / sec / 1e9 / pk["hbm_gbs"], 4), "traffic": None,
                         "kernel": "k_decode_vec (split-KV) + k_decode_merge", "peak_src": pk["src"] + " hbm_gbs"},
            "cpu_baseline": cpu,
            "e2e": {"value": round(bytes_ / (e2e_ms / 1e3 / args.steps) / 1e9 * world, 3), "unit": "GB/s",
                    "h2d_bytes_per_step": int(q_h.nbytes), "d2h_bytes_per_step": int(4 * B * H * D)},
            "gpu_launches": 2 * args.steps, "clocks": clk,
            "step_ms_min_max": [round(min(dev_ms), 5), round(max(dev_ms), 5)],
        }
        print(json.dumps(line))
    if dist:
        dist.destroy_process_group()


def run_int8_gemm(args, rank, world, local_rank, n):
    """MATMUL with INT8 weights (the reference's mixed-precision path) at n x n x n through
    the executor: per step max|A| + quantise A + transpose B + tcgen05 kind::i8 GEMM."""
    import torch
    import lancius_b200 as L
    from lancius_b200 import data
    torch.cuda.set_device(local_rank)
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=torch.device("cuda", local_rank))
    dev = L.Device(local_rank)
    g = L.Graph()
    a = g.input(n, n)
    b = g.input(n, n)
    out = g.matmul(a, b)
    a_h = data.uniform(data.sub_seed(4 + rank, 1), (n, n), -1.0, 1.0).astype(np.float32)
    wq = np.round(data.uniform(data.sub_seed(4, 2), (n, n), -127, 127)).astype(np.int8)
    g.bind(a, a_h.astype(np.float64))
    g.bind_int8(b, wq, 0.01)
    sched = g.schedule()
    dev.set_graph_replay(True)
    dev.bind(sched)
    dev.upload_bound_inputs()
    ext = torch.cuda.ExternalStream(dev.stream)
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device="cuda")

    def step(e0=None, e1=None):
        with torch.cuda.stream(ext):
            flush_l2(flush)
            if e0: e0.record(ext)
        dev.execute(sched)
        if e1:
            with torch.cuda.stream(ext):
                e1.record(ext)
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    clocks = Clocks(local_rank)
    clocks.start()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    for e0, e1 in evs:
        step(e0, e1)
    torch.cuda.synchronize()
    clk = clocks.stop()
    dev_ms = [e0.elapsed_time(e1) for e0, e1 in evs]
    total_ms = sum(dev_ms)
    launches = dev.last_launch_count
    # e2e: A in from pinned memory, C out, weights resident
    pa = dev.lib.lcu_host_alloc(n * n * 4)
    pc = dev.lib.lcu_host_alloc(n * n * 4)
    np.ctypeslib.as_array(C.cast(pa, C.POINTER(C.c_float)), shape=(n * n,))[:] = a_h.ravel()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(ext)
    for _ in range(args.steps):
        dev.upload_ptr(a, pa, 2)
        dev.execute(sched)
        dev.download_ptr(out, pc, 2)
    e1.record(ext)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1)
    dev.lib.lcu_host_free(pa); dev.lib.lcu_host_free(pc)
    if dist:
        t = torch.tensor([total_ms, e2e_ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms, e2e_ms = t.tolist()
    if rank == 0:
        ops = 2.0 * n ** 3
        sec = total_ms / 1e3 / args.steps
        val = ops / sec / 1e12 * world
        pk = peaks()
        line = {
            "metric": "INT8 GEMM TOPS", "value": round(val, 2), "unit": "TOPS", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(total_ms / args.steps, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "s8 x s8 -> s32",
            "data": "synthetic (A ~ U[-1,1), int8 weights ~ U[-127,127], seeded)",
            "config": {"workload": f"int8_weight_matmul{n}", "mode": "dynamic per-tensor INT8 (reference semantics)",
                       "l2": L2_NOTE, "parallelism": f"replicas x{world}"},
            "roofline": {"bound": "tensor", "achieved": round(ops / sec / 1e12, 2), "peak": pk["bf16_tflops"] * 2,
                         "unit": "TOPS", "frac": round(ops / sec / 1e12 / (pk["bf16_tflops"] * 2), 4), "traffic": None,
                         "peak_src": pk["src"] + " bf16 x 2 (INT8 dense rate is twice BF16)"},
            "cpu_baseline": None,
            "e2e": {"value": round(ops / (e2e_ms / 1e3 / args.steps) / 1e12 * world, 2), "unit": "TOPS",
                    "h2d_bytes_per_step": 4 * n * n, "d2h_bytes_per_step": 4 * n * n},
            "gpu_launches": launches * args.steps, "clocks": clk,
            "step_ms_min_max": [round(min(dev_ms), 4), round(max(dev_ms), 4)],
        }
        print(json.dumps(line))
    if dist:
        dist.destroy_process_group()


def _is_activation(cfg, node):
    # per-step inputs (weights stay resident): attention Q/K/V, conv/mlp/encoder X, gemm A and B
    return True if cfg in ("attention",) or cfg.startswith("gemm") else node.id == 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--config", default="attention")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--mode", default="fp32_exact", choices=["fp32_exact", "tf32", "bf16"],
                    help="contraction precision: 3xTF32 (FP32-exact, default), one TF32 pass, or BF16 GEMMs "
                         "(conv and attention then run one TF32 pass)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local_rank = int(os.environ.get("LOCAL_RANK", 0))
    metric, unit, workload = metric_names(args.config)

    if args.impl == "reference":
        if rank != 0:
            return
        res = reference_arm(args, metric, unit, workload)
        print(json.dumps(res))
        return

    if args.config.startswith("gemm") and world > 1:
        run_colsplit(args, rank, world, local_rank, int(args.config[4:]))
        return
    if args.config == "decode":
        run_decode(args, rank, world, local_rank)
        return
    if args.config.startswith("int8gemm"):
        run_int8_gemm(args, rank, world, local_rank, int(args.config[8:]))
        return
    built, total_ms, e2e_ms, dev_ms, launches, clk, in_b, out_b, dist = run_b200(args, rank, world, local_rank)
    if rank != 0:
        if dist:
            dist.destroy_process_group()
        return
    sec_per_graph = total_ms / 1e3 / args.steps
    value = metric_of(args.config, built, sec_per_graph) * world
    e2e_val = metric_of(args.config, built, e2e_ms / 1e3 / args.steps) * world
    pk = peaks()
    roof = None
    passes = 1 if args.mode == "tf32" else 3
    if args.mode == "bf16":   # BF16 GEMMs against the BF16 peak; attention runs one TF32 pass
        passes = 1 if args.config == "attention" else 0.5
    if args.config == "attention":
        achieved = built.bytes / (sec_per_graph) / 1e9
        # traffic: dram__bytes_read.sum + dram__bytes_write.sum of one k_attn_tc launch, from
        # the ncu capture of this exact kernel source (None when the source changed since)
        traffic, src_hash = attention_traffic()
        roof = {"bound": "hbm", "achieved": round(achieved, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
                "frac": round(achieved / pk["hbm_gbs"], 4), "traffic": traffic,
                "traffic_src": f"ncu capture of k_attn_tc, source sha256 {src_hash}",
                "kernel": "attention (one grouped launch over the 8 ATTENTION nodes)",
                "peak_src": pk["src"] + " hbm_gbs (burst copy)",
                # the kernel is compute-bound: its algorithmic FLOPs (QK^T and PV over the
                # causal triangle) against the 3xTF32 ceiling = TF32 dense (bf16 / 2) / 3
                "tensor_view": {"achieved_tflops": round(built.flops / sec_per_graph / 1e12, 2),
                                "mode_ceiling_tflops": round(pk["bf16_tflops"] / 2 / passes, 1),
                                "frac_of_mode_ceiling": round(built.flops / sec_per_graph / 1e12 / (pk["bf16_tflops"] / 2 / passes), 4)}}
    else:
        achieved = built.flops / sec_per_graph / 1e12
        roof = {"bound": "tensor", "achieved": round(achieved, 2), "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                "frac": round(achieved / pk["bf16_tflops"], 4), "traffic": None, "peak_src": pk["src"] + " bf16",
                # FP32-exact = 3 TF32 MMAs per product, TF32 mode = 1; TF32 dense rate = bf16 / 2
                "tf32_peak": round(pk["bf16_tflops"] / 2, 1), "frac_of_tf32_peak": round(achieved / (pk["bf16_tflops"] / 2), 4),
                "mode_ceiling": round(pk["bf16_tflops"] / 2 / passes, 1),
                "frac_of_mode_ceiling": round(achieved / (pk["bf16_tflops"] / 2 / passes), 4)}
    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        try:
            r = cpu_baseline(args.config)
            if r:
                cpu = dict(value=round(r[0], 4), unit=unit, **r[1])
        except Exception as ex:  # the baseline is reported, never required
            cpu = {"error": str(ex)[:200]}
    line = {
        "metric": metric, "value": round(value, 3), "unit": unit, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(total_ms / args.steps, 5), "higher_is_better": True,
        "scaling": "strong" if args.config == "encoder_b256" else "weak", "vs_baseline": None,
        "dtype": {"tf32": "tf32", "bf16": "bf16 (GEMM operands), f32 accumulate"}.get(args.mode, "f32"),
        "data": "synthetic (seeded N(0,1), splitmix64)",
        "config": config_of(args.config, workload),
        "mode": args.mode, "l2": L2_NOTE,
        "parallelism": f"batch-sharded x{world}",
        "roofline": roof,
        "cpu_baseline": cpu,
        "e2e": {"value": round(e2e_val, 3), "unit": unit, "h2d_bytes_per_step": in_b, "d2h_bytes_per_step": out_b},
        # the same workload through lancius_schedule_execute_static, FP64 pageable host buffers
        # (inputs, weights included, uploaded and outputs copied back on every call)
        "e2e_dropin": {"value": round(metric_of(args.config, built, built.meta["dropin_ms"] / 1e3 / args.steps) * world, 3),
                       "unit": unit, "entry": "lancius_schedule_execute_static", "host_dtype": "f64",
                       "h2d_bytes_per_step": 2 * sum(arr.size * 4 for _, arr in built.inputs),
                       "d2h_bytes_per_step": 2 * out_b},
        "gpu_launches": launches * args.steps,
        "clocks": clk,
        "step_ms_min_max": [round(min(dev_ms), 5), round(max(dev_ms), 5)],
    }
    print(json.dumps(line))
    if dist:
        dist.destroy_process_group()


def reference_arm(args, metric, unit, workload):
    import oracle
    from lancius_b200 import Graph, configs
    if not oracle.reference_available():
        return {"impl": "reference", "unavailable": "oracle/_ref/liblancius_ref.so was not built"}
    if args.config == "decode":
        return reference_arm_decode(args, metric, unit, workload)
    if args.config != "attention":
        return reference_arm_sampled(args, metric, unit, workload)
    ref = oracle.reference()
    _all_host_threads()
    g = Graph(ref)
    b = configs.attention(g, batch=8, seq=512, heads=8, head_dim=64, seed=1)
    b.bind_host()
    sched = ref.lancius_ir_schedule(g.ptr)
    arena = ref.lancius_arena_create(256 << 20)
    times = []
    # the executor recomputes every node on every call; buffers from the first call are reused
    for i in range(args.warmup + args.steps):
        t0 = time.perf_counter()
        ref.lancius_schedule_execute(sched, arena)
        t1 = time.perf_counter()
        if i >= args.warmup:
            times.append(t1 - t0)
    ref.lancius_arena_destroy(arena)
    ref.lancius_schedule_destroy(sched)
    sec = sum(times) / len(times)
    val = b.bytes / sec / 1e9
    cores = os.cpu_count()
    return {"impl": "reference", "metric": metric, "value": round(val, 4), "unit": unit, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(sec * 1e3, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64",
            "data": "synthetic (seeded N(0,1), splitmix64)",
            "config": config_of(args.config, workload), "executor": "lancius_schedule_execute (arena mode)",
            "cpu_baseline": {"value": round(val, 4), "unit": unit, "kind": "reference", "cores": cores,
                             "sample": "the full batch-8 graph per step on the host CPU, reference C sources "
                                       "compiled by oracle/Makefile; OpenMP threads = all host cores"},
            "e2e": {"value": round(val, 4), "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def reference_arm_sampled(args, metric, unit, workload):
    """The reference's own executor on the host cores for the non-attention configs: each
    step runs one bounded sample of the workload (see _ref_sample)."""
    import oracle
    smp = _ref_sample(args.config)
    if smp is None:
        return {"impl": "reference", "unavailable": f"no reference sample defined for {args.config}"}
    ref = oracle.reference()
    cores = _all_host_threads()
    build, factor, what = smp
    secs = []
    b = None
    for i in range(args.warmup + args.steps):
        sec, _, b = _ref_run_seconds(ref, build, min_s=0.0, max_reps=1)
        if i >= args.warmup:
            secs.append(sec)
    sec = sum(secs) / len(secs)
    val = _sample_value(args.config, b, sec)
    return {"impl": "reference", "metric": metric, "value": round(val, 6), "unit": unit, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(sec * factor * 1e3, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64",
            "data": "synthetic (seeded, splitmix64)",
            "config": config_of(args.config, workload), "executor": "lancius_schedule_execute (arena mode)",
            "cpu_baseline": {"value": round(val, 6), "unit": unit, "kind": "reference", "cores": cores,
                             "sample": f"each step: {what}; OpenMP threads = all host cores"},
            "e2e": {"value": round(val, 6), "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def reference_arm_decode(args, metric, unit, workload):
    """kernel_attention_kv_cache (the reference's own FP64 C kernel) on the host cores,
    each step a bounded sample of 4 of the batch's sequences scaled to the batch."""
    import oracle
    ref = oracle.reference()
    B, S, H, D = DECODE["batch"], DECODE["seq"], DECODE["heads"], DECODE["head_dim"]
    nb = 4
    rng = np.random.default_rng(7)
    kc, vc = rng.standard_normal((nb, S, H, D)), rng.standard_normal((nb, S, H, D))
    q = rng.standard_normal((nb, H * D))
    times = []
    for i in range(args.warmup + args.steps):
        sec, cores = _decode_ref_seconds(ref, q, kc, vc, limit_s=0.0)
        if i >= args.warmup:
            times.append(sec * B / nb)
    sec = sum(times) / len(times)
    val = 4.0 * (2 * B * S * H * D + 2 * B * H * D) / sec / 1e9
    metric = "decode attention GB/s"
    return {"impl": "reference", "metric": metric, "value": round(val, 4), "unit": "GB/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(sec * 1e3, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64",
            "data": "synthetic (N(0,1) caches, seeded)",
            "config": {"workload": workload, "per_gpu_batch": B}, "executor": "kernel_attention_kv_cache per sequence",
            "cpu_baseline": {"value": round(val, 4), "unit": "GB/s", "kind": "reference", "cores": cores,
                             "sample": f"{nb} of {B} sequences per step, scaled x{B // nb}; one call per sequence "
                                       "on a thread pool of all host cores; FP32-equivalent bytes"},
            "e2e": {"value": round(val, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


if __name__ == "__main__":
    main()
