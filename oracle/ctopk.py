"""ctypes loader of the C restatement of torch's CPU top-k order (``oracle/topk_select.c``).
Test infrastructure only."""
from __future__ import annotations

import ctypes
import os
import subprocess

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "_build", "libmoe_oracle.so")
_lib = None


def build() -> str:
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB


def _load():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB):
            build()
        lib = ctypes.CDLL(LIB)
        lib.oracle_topk_rows.restype = None
        lib.oracle_topk_rows.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                         ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
        _lib = lib
    return _lib


def topk_torch_cpu_order(values: torch.Tensor, k: int):
    """``(vals, ids)`` of ``torch.topk(values, k)`` computed by the C restatement."""
    v = values.detach().float().contiguous().cpu()
    t, n = v.shape
    ids = torch.empty(t, k, dtype=torch.int64)
    out = torch.empty(t, k, dtype=torch.float32)
    scratch = ctypes.create_string_buffer(8 * n)
    _load().oracle_topk_rows(v.data_ptr(), n, t, n, k, ids.data_ptr(), out.data_ptr(), ctypes.addressof(scratch))
    return out, ids
