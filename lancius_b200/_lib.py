"""Loads the in-tree liblancius_b200.so (the C11 host runtime + sm_100a kernels).

There is no fallback: if the library is missing the import fails with the
build command to run.
"""
import ctypes as C
import os

from ._abi import B200_FUNCS, IR_FUNCS, declare

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liblancius_b200.so")

_lib = None


def load():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is not built: run `make -C {HERE}` "
                              "(or __graft_entry__.build())")
        lib = C.CDLL(LIB_PATH, mode=os.RTLD_LOCAL)
        declare(lib, IR_FUNCS)
        declare(lib, B200_FUNCS)
        _lib = lib
    return _lib
