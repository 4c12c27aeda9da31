"""ctypes binding of ``libmuserve_moe.so`` (the C ABI of ``include/muserve_moe.h``).

The library is the only compute path: when it is missing, or no sm_100 GPU is visible,
every op raises instead of falling back to anything else.
"""
from __future__ import annotations

import ctypes
import os
import threading

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libmuserve_moe.so")

MSV_OK, MSV_ERR_INVALID, MSV_ERR_UNSUPPORTED, MSV_ERR_CUDA, MSV_ERR_TIMEOUT = 0, -1, -2, -3, -4
MSV_F32, MSV_BF16, MSV_I32, MSV_I64, MSV_E4M3 = 0, 1, 2, 3, 4
COMBINE_V2, COMBINE_DISPATCH, COMBINE_BATCHED = 0, 1, 2
FWD_ROUTING_GIVEN = 1

P = ctypes.c_void_p
I = ctypes.c_int
I64 = ctypes.c_int64
SZ = ctypes.c_size_t


class MoeShape(ctypes.Structure):
    _fields_ = [("tokens", I), ("hidden", I), ("num_experts", I), ("top_k", I), ("inter", I),
                ("shared_inter", I), ("placement", I), ("tp", I), ("rank", I), ("add_shared", I),
                ("combine_mode", I), ("weights_dtype", I)]


class MoeWeights(ctypes.Structure):
    _fields_ = [("gate_w", P), ("up_w", P), ("gu_expert_rows", I64), ("gate_s", P), ("up_s", P),
                ("gu_scale_expert_stride", I64), ("down_w", P), ("down_s", P),
                ("sh_gate_w", P), ("sh_up_w", P), ("sh_down_w", P), ("sh_gate_s", P), ("sh_up_s", P),
                ("sh_down_s", P), ("sh_gate_logit_w", P)]


MAX_TP = 8


class TpComm(ctypes.Structure):
    _fields_ = [("world", I), ("rank", I), ("max_tokens", I), ("hidden", I), ("shared", P * MAX_TP), ("epoch", P)]


_SIGS = {
    "msv_last_error": (ctypes.c_char_p, []),
    "msv_version": (I, []),
    "msv_launch_count": (ctypes.c_ulonglong, []),
    "msv_check_device_error": (I, [P]),
    "msv_route_topk": (I, [P, I64, I, I, I, I, P, I, P, I, P]),
    "msv_topk_select": (I, [P, I64, I, I, I, P, I, P, P]),
    "msv_router_workspace_size": (SZ, [I, I, I]),
    "msv_router_from_hidden": (I, [P, P, I, I, I, I, I, I, P, I, P, I, P, P, SZ, P]),
    "msv_router_from_hidden_bias": (I, [P, P, I, I, I, I, I, I, P, P, I, P, I, P, P, SZ, P]),
    "msv_add_rms_norm_gemma": (I, [P, P, P, I, I, ctypes.c_float, P, P]),
    "msv_moe_permute": (I, [P, I, I, I, I, I, I, I, I, P, P, P, P, P, P]),
    "msv_fp8_quant_128": (I, [P, I64, I, I, P, P, I64, P, I64, I64, P]),
    "msv_ragged_gemm_workspace_size": (SZ, [I, I]),
    "msv_ragged_moe_gemm_fp8": (I, [P, P, I, I, P, P, I, I, P, P, P, SZ, P]),
    "msv_ragged_moe_gemm_fp8_noalloc": (I, [P, P, I, I, P, P, I, I, P, P, P]),
    "msv_gemm_fp8_workspace_size": (SZ, [I, I]),
    "msv_gemm_fp8_nt_groupwise": (I, [P, P, I, I, P, P, I, P, P, SZ, P]),
    "msv_moe_forward_workspace_size": (SZ, [ctypes.POINTER(MoeShape)]),
    "msv_moe_forward": (I, [ctypes.POINTER(MoeShape), ctypes.POINTER(MoeWeights), P, P, P, P, P, I, P, SZ, P]),
    "msv_moe_forward_profiled": (I, [ctypes.POINTER(MoeShape), ctypes.POINTER(MoeWeights), P, P, P, P, P, I, P, SZ,
                                     P, P]),
    "msv_ipc_handle_bytes": (SZ, []),
    "msv_ipc_export": (I, [P, P, ctypes.POINTER(ctypes.c_uint64)]),
    "msv_ipc_import": (I, [P, ctypes.c_uint64, ctypes.POINTER(P)]),
    "msv_ipc_close": (I, [P]),
    "msv_tp_shared_bytes": (SZ, [I, I]),
    "msv_tp_epoch_bytes": (SZ, []),
    "msv_moe_forward_tp": (I, [ctypes.POINTER(MoeShape), ctypes.POINTER(MoeWeights), P, P, P, P, P, I, P, SZ,
                               ctypes.POINTER(TpComm), P]),
    "msv_moe_forward_tp_profiled": (I, [ctypes.POINTER(MoeShape), ctypes.POINTER(MoeWeights), P, P, P, P, P, I, P,
                                        SZ, ctypes.POINTER(TpComm), P, P]),
}

_lock = threading.Lock()
_lib = None


def load(require_gpu: bool = True):
    """Load the library (once).  Raises when it is missing or, with ``require_gpu``, when no
    CUDA device is visible: there is no CPU fallback."""
    global _lib
    if require_gpu and not torch.cuda.is_available():
        raise RuntimeError("muserve_b200 needs an sm_100 CUDA device; none is visible")
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise RuntimeError(f"{LIB_PATH} is missing: run `python -m muserve_b200.build`")
                lib = ctypes.CDLL(LIB_PATH)
                for name, (res, args) in _SIGS.items():
                    fn = getattr(lib, name)
                    fn.restype = res
                    fn.argtypes = args
                _lib = lib
    return _lib


def check(rc: int, what: str = "") -> None:
    if rc != MSV_OK:
        msg = load(require_gpu=False).msv_last_error().decode()
        if rc == MSV_ERR_INVALID:
            raise AssertionError(f"{what}: {msg}")
        raise RuntimeError(f"{what}: status {rc}: {msg}")


def stream_ptr(stream: torch.cuda.Stream | None = None) -> int:
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


_ws_cache: dict = {}


def workspace(nbytes: int, device: torch.device) -> torch.Tensor:
    """A device byte buffer of at least ``nbytes``, reused across calls on the same device and
    stream (the kernels that use it are stream-ordered)."""
    key = (device, torch.cuda.current_stream(device).cuda_stream)
    buf = _ws_cache.get(key)
    if buf is None or buf.numel() < nbytes:
        buf = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=device)
        _ws_cache[key] = buf
    return buf


def header_symbols(header: str) -> list[str]:
    """Names of the functions declared in ``include/muserve_moe.h``."""
    import re
    src = open(header).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(msv_[a-z0-9_]+)\s*\(", src)))
