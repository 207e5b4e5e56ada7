"""The C ABI library loads without a GPU and exports every function include/ declares."""
import glob
import os
import re
import subprocess

import lancius_b200 as L

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
DECL = re.compile(r"^\s*(?!static|typedef|return|#|\*|/)[A-Za-z_][\w\s\*]*?\b([a-z_][a-z0-9_]*)\s*\([^;{]*\)\s*;", re.M)


def declared():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "**", "*.h"), recursive=True):
        src = open(h).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        src = re.sub(r"//[^\n]*", "", src)
        src = re.sub(r"#define[^\n]*(\\\n[^\n]*)*", "", src)
        for m in DECL.finditer(src):
            names.add(m.group(1))
    return names


def test_library_loads_and_exports_all_declared_symbols():
    lib = L.load()
    names = declared()
    assert {"lcu_create", "lancius_schedule_execute_cuda", "lcu_matmul", "lancius_matmul",
            "lancius_build_memory_plan", "lcu_matmul_noalloc", "lancius_schedule_execute",
            "lancius_schedule_execute_parallel", "lancius_schedule_execute_static", "lancius_compile_and_run",
            "lancius_read_output", "lancius_pool_create", "lcu_check_stream", "lcu_noalloc_prepare"} <= names
    out = subprocess.run(["nm", "-D", "--defined-only", L.LIB_PATH], capture_output=True, text=True).stdout
    exported = {ln.split()[-1] for ln in out.splitlines() if " T " in ln}
    missing = sorted(n for n in names if n not in exported)
    assert not missing, f"declared but not exported: {missing}"
    for n in names:
        getattr(lib, n)   # resolvable through ctypes too


def test_build_info_names_kernels():
    info = L.load().lcu_build_info().decode()
    assert "gemm_tcgen05_3xtf32" in info and "attention_tcgen05_3xtf32" in info


def test_errors_without_device():
    """Without a GPU, context creation fails cleanly with LANCIUS_ERROR_INTERNAL (no abort)."""
    import torch
    if torch.cuda.is_available():
        return
    lib = L.load()
    assert not lib.lcu_create(0)
    assert lib.lancius_get_error() == -10


def test_pool_runs_every_task():
    """lancius_pool (reference lancius_threadpool.h): submitted tasks all run before wait returns."""
    import ctypes as C
    lib = L.load()
    lib.lancius_pool_create.restype = C.c_void_p
    lib.lancius_pool_create.argtypes = [C.c_int]
    TASK = C.CFUNCTYPE(None, C.c_void_p)
    lib.lancius_pool_submit.argtypes = [C.c_void_p, TASK, C.c_void_p]
    lib.lancius_pool_wait.argtypes = [C.c_void_p]
    lib.lancius_pool_destroy.argtypes = [C.c_void_p]
    hits = (C.c_int * 300)()

    @TASK
    def task(arg):
        hits[arg - 1] += 1

    pool = lib.lancius_pool_create(4)
    assert pool
    for rnd in range(2):
        for i in range(300):
            lib.lancius_pool_submit(pool, task, i + 1)
        lib.lancius_pool_wait(pool)
        assert list(hits) == [rnd + 1] * 300
    lib.lancius_pool_destroy(pool)


def test_dropin_program_links_against_library():
    """A C program using the reference's executor and stable-FFI names links against
    liblancius_b200.so alone (run on the GPU by test_gpu_dropin.py)."""
    L.load()
    d = os.path.join(ROOT, "tests", "dropin")
    subprocess.run(["make", "-C", d], check=True, capture_output=True)
    r = subprocess.run([os.path.join(d, "dropin_main")], capture_output=True, text=True)
    assert r.returncode == 1 and "usage" in r.stderr
