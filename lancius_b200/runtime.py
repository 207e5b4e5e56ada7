"""Device context: binds a scheduled Lancius graph to one B200 and runs it.

Thin wrapper over the lcu_* C ABI (include/lancius_cuda.h); every call raises
LanciusError on a non-zero status.
"""
import ctypes as C

import numpy as np

from . import _abi
from ._lib import load
from .graph import LanciusError

MODE_FP32_EXACT, MODE_TF32, MODE_BF16 = 0, 1, 2
EPI_NONE, EPI_RELU, EPI_GELU = 0, 1, 2


def _ok(rc, what):
    if rc != 0:
        raise LanciusError(rc, what)


class Device:
    def __init__(self, device=0, mode=MODE_FP32_EXACT):
        self.lib = load()
        self.ptr = self.lib.lcu_create(device)
        if not self.ptr:
            raise LanciusError(self.lib.lancius_get_error(), f"lcu_create({device})")
        self.set_mode(mode)
        self.sched = None

    def set_mode(self, mode):
        _ok(self.lib.lcu_set_mode(self.ptr, mode), "lcu_set_mode")

    def set_graph_replay(self, on):
        _ok(self.lib.lcu_set_graph_replay(self.ptr, 1 if on else 0), "lcu_set_graph_replay")

    def set_fusion(self, on):
        _ok(self.lib.lcu_set_fusion(self.ptr, 1 if on else 0), "lcu_set_fusion")

    @property
    def stream(self):
        return self.lib.lcu_stream(self.ptr)

    def bind(self, schedule, plan=None):
        _ok(self.lib.lcu_bind_plan(self.ptr, schedule.ptr, schedule.graph.ptr, plan), "lcu_bind_plan")
        self.sched = schedule

    def upload(self, node, array):
        a = np.ascontiguousarray(array)
        if a.dtype == np.float32:
            dt = _abi.DTYPE_FP32
        else:
            a = np.ascontiguousarray(a, dtype=np.float64)
            dt = _abi.DTYPE_FP64
        if a.size != node.size:
            raise ValueError(f"upload {node}: {a.size} values for {node.size} elements")
        _ok(self.lib.lcu_upload(self.ptr, node.ptr, a.ctypes.data_as(C.c_void_p), dt), "lcu_upload")
        # the copy is asynchronous on the context stream: keep the source alive until it lands
        self.synchronize()

    def upload_ptr(self, node, host_ptr, dtype):
        _ok(self.lib.lcu_upload(self.ptr, node.ptr, host_ptr, dtype), "lcu_upload")

    def upload_bound_inputs(self):
        _ok(self.lib.lcu_upload_bound_inputs(self.ptr), "lcu_upload_bound_inputs")
        self.synchronize()

    def download(self, node, dtype=np.float64):
        out = np.empty(node.shape, dtype=dtype)
        dt = _abi.DTYPE_FP32 if dtype == np.float32 else _abi.DTYPE_FP64
        _ok(self.lib.lcu_download(self.ptr, node.ptr, out.ctypes.data_as(C.c_void_p), dt), "lcu_download")
        return out

    def download_ptr(self, node, host_ptr, dtype):
        _ok(self.lib.lcu_download(self.ptr, node.ptr, host_ptr, dtype), "lcu_download")

    def device_ptr(self, node):
        return self.lib.lcu_node_device_ptr(self.ptr, node.ptr)

    def refresh_weights(self):
        """Remakes the TF32 hi/lo weight copies after writes through device_ptr()."""
        _ok(self.lib.lcu_refresh_weights(self.ptr), "lcu_refresh_weights")

    def execute(self, schedule=None):
        s = schedule or self.sched
        self.lib.lancius_clear_error()
        self.lib.lancius_schedule_execute_cuda(s.ptr, self.ptr)
        err = self.lib.lancius_get_error()
        if err != 0:
            raise LanciusError(err, "lancius_schedule_execute_cuda")

    def synchronize(self):
        _ok(self.lib.lcu_synchronize(self.ptr), "lcu_synchronize")

    @property
    def last_launch_count(self):
        return self.lib.lcu_last_launch_count(self.ptr)

    def close(self):
        if self.ptr:
            self.lib.lcu_destroy(self.ptr)
            self.ptr = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
