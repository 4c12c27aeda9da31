"""Typed torch wrappers over the C ABI (``include/muserve_moe.h``).

Tensors must already be on the current CUDA device; work is enqueued on the current torch
stream.  These are the building blocks of the reference-shaped modules in
``muserve_b200.kernels``, ``muserve_b200.mate`` and ``muserve_b200.model``.
"""
from __future__ import annotations

import torch

from . import _lib
from ._lib import check, ptr, stream_ptr

FP8 = torch.float8_e4m3fn

_DT = {torch.float32: _lib.MSV_F32, torch.bfloat16: _lib.MSV_BF16, torch.int32: _lib.MSV_I32,
       torch.int64: _lib.MSV_I64}


def _cuda(t: torch.Tensor, name: str):
    assert t.is_cuda, f"{name} must be a CUDA tensor"


def route_topk(logits: torch.Tensor, k: int, renormalize: bool = True,
               w_dtype: torch.dtype = torch.bfloat16, ids_dtype: torch.dtype = torch.int64):
    """softmax -> top-k (torch CPU order) -> renormalise -> cast (``qwen35_layer_v2.py:569-572``)."""
    lib = _lib.load()
    _cuda(logits, "logits")
    assert logits.dtype == torch.float32 and logits.dim() == 2 and logits.stride(1) == 1
    t, e = logits.shape
    w = torch.empty(t, k, dtype=w_dtype, device=logits.device)
    ids = torch.empty(t, k, dtype=ids_dtype, device=logits.device)
    check(lib.msv_route_topk(ptr(logits), logits.stride(0), t, e, k, int(renormalize), ptr(w), _DT[w_dtype],
                             ptr(ids), _DT[ids_dtype], stream_ptr()), "msv_route_topk")
    return w, ids


def router_from_hidden(hidden: torch.Tensor, gate_weight: torch.Tensor, k: int, renormalize: bool = True,
                       round_logits_bf16: bool = True, w_dtype: torch.dtype = torch.bfloat16,
                       ids_dtype: torch.dtype = torch.int32, return_logits: bool = False,
                       logit_bias: torch.Tensor | None = None):
    """Router from the hidden states on the tensor cores: ``hidden @ gate_weight.T`` (bf16 in, fp32
    accumulation), optionally rounded to bf16 (``qwen35_layer_v2.py:567-568``), then softmax,
    top-k and renormalisation as :func:`route_topk` (``:569-572``).  With
    ``round_logits_bf16=False`` and fp32 weights it is ``moe_dispatch.moe_gate``
    (``kernels/moe_dispatch.py:8-24``).  ``logit_bias`` ([E] fp32, not in the reference) is added
    to the logits before the softmax: the expert-popularity prior of the 60-layer stack
    benchmark.  Returns ``(topk_w, topk_ids[, logits])``; ``logits`` exclude the bias."""
    lib = _lib.load()
    _cuda(hidden, "hidden")
    _cuda(gate_weight, "gate_weight")
    assert hidden.dtype == torch.bfloat16 and gate_weight.dtype == torch.bfloat16
    hidden, gate_weight = hidden.contiguous(), gate_weight.contiguous()
    t, h = hidden.shape
    e, h2 = gate_weight.shape
    assert h == h2
    w = torch.empty(t, k, dtype=w_dtype, device=hidden.device)
    ids = torch.empty(t, k, dtype=ids_dtype, device=hidden.device)
    logits = torch.empty(t, e, dtype=torch.float32, device=hidden.device) if return_logits else None
    nbytes = lib.msv_router_workspace_size(t, h, e)
    if nbytes == 0:
        check(_lib.MSV_ERR_INVALID, "msv_router_workspace_size")
    ws = _lib.workspace(nbytes, hidden.device)
    if logit_bias is None:
        check(lib.msv_router_from_hidden(ptr(hidden), ptr(gate_weight), t, h, e, k, int(renormalize),
                                         int(round_logits_bf16), ptr(w), _DT[w_dtype], ptr(ids), _DT[ids_dtype],
                                         ptr(logits), ptr(ws), ws.numel(), stream_ptr()), "msv_router_from_hidden")
    else:
        _cuda(logit_bias, "logit_bias")
        assert logit_bias.dtype == torch.float32 and logit_bias.shape == (e,) and logit_bias.is_contiguous()
        check(lib.msv_router_from_hidden_bias(ptr(hidden), ptr(gate_weight), t, h, e, k, int(renormalize),
                                              int(round_logits_bf16), ptr(logit_bias), ptr(w), _DT[w_dtype], ptr(ids),
                                              _DT[ids_dtype], ptr(logits), ptr(ws), ws.numel(), stream_ptr()),
              "msv_router_from_hidden_bias")
    return (w, ids, logits) if return_logits else (w, ids)


def add_rms_norm_gemma(h: torch.Tensor, weight: torch.Tensor | None, add: torch.Tensor | None = None,
                       eps: float = 1e-6, out: torch.Tensor | None = None, norm: bool = True):
    """``rms_norm_gemma`` of ``qwen35_layer_v2.py:59-62`` as the decoder layer calls it
    (``:713-715``), with the residual add before it fused in: when ``add`` is given, ``h`` is
    first updated in place to ``bf16(h + add)``.  Returns the normalised ``[T, H]`` bf16 tensor
    (``out`` when given), or ``h`` when ``norm`` is False (add only)."""
    lib = _lib.load()
    _cuda(h, "h")
    assert h.dtype == torch.bfloat16 and h.dim() == 2 and h.is_contiguous()
    t, hd = h.shape
    if add is not None:
        _cuda(add, "add")
        assert add.dtype == torch.bfloat16 and add.shape == h.shape and add.is_contiguous()
    if norm:
        _cuda(weight, "weight")
        assert weight.dtype == torch.bfloat16 and weight.shape == (hd,) and weight.is_contiguous()
        if out is None:
            out = torch.empty_like(h)
    else:
        assert add is not None, "add-only needs add"
        out = None
    check(lib.msv_add_rms_norm_gemma(ptr(h), ptr(add), ptr(weight) if norm else None, t, hd, float(eps), ptr(out),
                                     stream_ptr()), "msv_add_rms_norm_gemma")
    return out if norm else h


def topk_select(values: torch.Tensor, k: int, ids_dtype: torch.dtype = torch.int64):
    """``torch.topk(values, k)`` with torch's CPU tie order, on the GPU."""
    lib = _lib.load()
    _cuda(values, "values")
    assert values.dtype == torch.float32 and values.dim() == 2 and values.stride(1) == 1
    t, e = values.shape
    ids = torch.empty(t, k, dtype=ids_dtype, device=values.device)
    vals = torch.empty(t, k, dtype=torch.float32, device=values.device)
    check(lib.msv_topk_select(ptr(values), values.stride(0), t, e, k, ptr(ids), _DT[ids_dtype], ptr(vals),
                              stream_ptr()), "msv_topk_select")
    return vals, ids


def permute(topk_ids: torch.Tensor, num_experts: int, tp: int = 1, rank: int = 0, alignment: int = 128):
    """Dispatch bookkeeping of ``qwen35_layer_v2.py:574-605`` (placement ``e % tp == rank``).

    Returns ``(sort_order, inverse_order, sorted_expert_ids, expert_counts, num_local)`` with
    the first ``num_local`` entries of the orders valid (``num_local`` stays on the device)."""
    lib = _lib.load()
    _cuda(topk_ids, "topk_ids")
    assert topk_ids.dim() == 2 and topk_ids.is_contiguous() and topk_ids.dtype in (torch.int32, torch.int64)
    t, k = topk_ids.shape
    dev = topk_ids.device
    p = t * k
    placement = 1 if tp > 1 else 0
    e_local = (num_experts + tp - 1) // tp if placement else num_experts
    mpad = -(-p // alignment) * alignment if alignment > 0 else p
    so = torch.empty(p, dtype=torch.int64, device=dev)
    io = torch.empty(p, dtype=torch.int64, device=dev)
    se = torch.empty(max(mpad, 1), dtype=torch.int32, device=dev)
    cnt = torch.empty(e_local, dtype=torch.int32, device=dev)
    nl = torch.empty(1, dtype=torch.int32, device=dev)
    check(lib.msv_moe_permute(ptr(topk_ids), _DT[topk_ids.dtype], t, k, num_experts, placement, tp, rank,
                              alignment, ptr(so), ptr(io), ptr(se), ptr(cnt), ptr(nl), stream_ptr()),
          "msv_moe_permute")
    return so, io, se, cnt, nl


def fp8_quant_128(x: torch.Tensor, row_index: torch.Tensor | None = None, scale_kb_major: bool = False):
    """``_fast_fp8_quantize`` (``qwen35_layer_v2.py:71-86``) of a bf16 ``[M,K]`` matrix, rows
    optionally gathered through ``row_index``.  Returns ``(q [M,K] e4m3, s [M,K/128] f32)``
    (``s`` as a ``[K/128, M]`` kb-major buffer transposed view when ``scale_kb_major``)."""
    lib = _lib.load()
    _cuda(x, "x")
    assert x.dtype == torch.bfloat16 and x.dim() == 2 and x.stride(1) == 1
    kdim = x.shape[1]
    assert kdim % 128 == 0, f"K={kdim} not divisible by block_size=128"
    m = row_index.numel() if row_index is not None else x.shape[0]
    q = torch.empty(m, kdim, dtype=FP8, device=x.device)
    if scale_kb_major:
        sbuf = torch.empty(kdim // 128, m, dtype=torch.float32, device=x.device)
        s, s_row, s_kb = sbuf.t(), 1, m
    else:
        s = torch.empty(m, kdim // 128, dtype=torch.float32, device=x.device)
        s_row, s_kb = kdim // 128, 1
    if row_index is not None:
        assert row_index.dtype == torch.int32 and row_index.is_contiguous()
    check(lib.msv_fp8_quant_128(ptr(x), x.stride(0), m, kdim, ptr(row_index), ptr(q), kdim, ptr(s), s_row, s_kb,
                                stream_ptr()), "msv_fp8_quant_128")
    return q, s


def ragged_gemm(a: torch.Tensor, a_scale: torch.Tensor, w: torch.Tensor, w_scale: torch.Tensor,
                m_indices: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
    """Row-grouped block-scaled FP8 GEMM (``mate.gemm.ragged_m_moe_gemm_8bit``)."""
    lib = _lib.load()
    m, kdim = a.shape
    e, n, kw = w.shape
    assert a.dtype == FP8 and w.dtype == FP8 and kw == kdim
    assert a.is_contiguous() and w.is_contiguous() and a_scale.is_contiguous() and w_scale.is_contiguous()
    assert a_scale.dtype == torch.float32 and w_scale.dtype == torch.float32
    assert a_scale.shape == (m, kdim // 128) and w_scale.shape == (e, n // 128, kdim // 128)
    assert m_indices.dtype == torch.int32 and m_indices.numel() == m and m_indices.is_contiguous()
    assert out.dtype == torch.bfloat16 and out.shape == (m, n) and out.is_contiguous()
    ws_n = lib.msv_ragged_gemm_workspace_size(m, n)
    ws = _lib.workspace(ws_n, a.device)
    check(lib.msv_ragged_moe_gemm_fp8(ptr(a), ptr(a_scale), m, kdim, ptr(w), ptr(w_scale), e, n, ptr(m_indices),
                                      ptr(out), ptr(ws), ws.numel(), stream_ptr()), "msv_ragged_moe_gemm_fp8")
    return out


def gemm_nt(a: torch.Tensor, a_scale: torch.Tensor, b: torch.Tensor, b_scale: torch.Tensor,
            out: torch.Tensor | None = None) -> torch.Tensor:
    """Dense block-scaled FP8 GEMM ``a [M,K] x b [N,K]^T -> bf16 [M,N]``."""
    lib = _lib.load()
    m, kdim = a.shape
    n, kb = b.shape
    assert kb == kdim, "K dimension mismatch"
    assert a.dtype == FP8 and b.dtype == FP8 and a.is_contiguous() and b.is_contiguous()
    assert a_scale.dtype == torch.float32 and b_scale.dtype == torch.float32
    assert a_scale.shape == (m, kdim // 128) and b_scale.shape == (n // 128, kdim // 128)
    a_scale, b_scale = a_scale.contiguous(), b_scale.contiguous()
    if out is None:
        out = torch.empty(m, n, dtype=torch.bfloat16, device=a.device)
    ws_n = lib.msv_gemm_fp8_workspace_size(m, n)
    ws = _lib.workspace(ws_n, a.device)
    check(lib.msv_gemm_fp8_nt_groupwise(ptr(a), ptr(a_scale), m, kdim, ptr(b), ptr(b_scale), n, ptr(out), ptr(ws),
                                        ws.numel(), stream_ptr()), "msv_gemm_fp8_nt_groupwise")
    return out


# ── whole layer ──────────────────────────────────────────────────────────────────────────

def weights_struct(weights: dict) -> tuple[_lib.MoeWeights, dict]:
    """``MoeWeights`` view of a reference-layout weights dict (``loader.py:212-264``).

    Accepts the fused ``moe.experts.gate_up_proj.*`` tensors (``qwen35_layer_v2.py:543-558``)
    or separate ``gate_proj``/``up_proj`` stacks; never copies or mutates the dict."""
    w = _lib.MoeWeights()
    info = {}
    if "moe.experts.gate_up_proj.weight" in weights:
        gu = weights["moe.experts.gate_up_proj.weight"]
        gs = weights["moe.experts.gate_up_proj.weight_scale_inv"]
        e, two_i, h = gu.shape
        inter = two_i // 2
        assert gu.is_contiguous() and gs.is_contiguous() and gs.dtype == torch.float32
        w.gate_w, w.up_w = gu.data_ptr(), gu.data_ptr() + inter * h
        w.gu_expert_rows = two_i
        w.gate_s = gs.data_ptr()
        w.up_s = gs.data_ptr() + (inter // 128) * (h // 128) * 4
        w.gu_scale_expert_stride = (two_i // 128) * (h // 128)
    else:
        g = weights["moe.experts.gate_proj.weight"]
        u = weights["moe.experts.up_proj.weight"]
        gs = weights["moe.experts.gate_proj.weight_scale_inv"]
        us = weights["moe.experts.up_proj.weight_scale_inv"]
        e, inter, h = g.shape
        for t in (g, u, gs, us):
            assert t.is_contiguous()
        assert gs.dtype == torch.float32 and us.dtype == torch.float32
        w.gate_w, w.up_w, w.gu_expert_rows = g.data_ptr(), u.data_ptr(), inter
        w.gate_s, w.up_s = gs.data_ptr(), us.data_ptr()
        w.gu_scale_expert_stride = (inter // 128) * (h // 128)
    d = weights["moe.experts.down_proj.weight"]
    ds = weights["moe.experts.down_proj.weight_scale_inv"]
    assert d.is_contiguous() and ds.is_contiguous() and d.shape == (e, h, inter)
    w.down_w, w.down_s = d.data_ptr(), ds.data_ptr()
    info.update(local_experts=e, inter=inter, hidden=h, shared_inter=0)
    if "moe.shared_expert.gate_proj.weight" in weights:
        sg = weights["moe.shared_expert.gate_proj.weight"]
        su = weights["moe.shared_expert.up_proj.weight"]
        sd = weights["moe.shared_expert.down_proj.weight"]
        for t in (sg, su, sd):
            assert t.dtype == FP8 and t.is_contiguous(), "shared expert must be FP8 with block scales"
        w.sh_gate_w, w.sh_up_w, w.sh_down_w = sg.data_ptr(), su.data_ptr(), sd.data_ptr()
        w.sh_gate_s = weights["moe.shared_expert.gate_proj.weight_scale_inv"].contiguous().data_ptr()
        w.sh_up_s = weights["moe.shared_expert.up_proj.weight_scale_inv"].contiguous().data_ptr()
        w.sh_down_s = weights["moe.shared_expert.down_proj.weight_scale_inv"].contiguous().data_ptr()
        info["shared_inter"] = sg.shape[0]
        if "moe.shared_expert_gate.weight" in weights:
            sgw = weights["moe.shared_expert_gate.weight"]
            assert sgw.dtype == torch.bfloat16 and sgw.is_contiguous()
            w.sh_gate_logit_w = sgw.data_ptr()
    return w, info


def moe_layer(hidden: torch.Tensor, weights: dict, top_k: int, num_experts: int,
              router_logits: torch.Tensor | None = None, topk_w: torch.Tensor | None = None,
              topk_ids: torch.Tensor | None = None, placement: int = 0, tp: int = 1, rank: int = 0,
              add_shared: bool = True, combine_mode: int = _lib.COMBINE_V2,
              weights_dtype: torch.dtype = torch.bfloat16, out: torch.Tensor | None = None,
              return_routing: bool = False, comm=None):
    """One MoE layer (``qwen35_layer_v2.py:561-675`` after the router GEMM) in six kernels:
    router, dispatch bookkeeping, gather+quantise, gate_up GEMM (SwiGLU + requant epilogue),
    down GEMM, weighted combine (+ shared expert).  Either ``router_logits`` or
    ``topk_w``/``topk_ids`` (given routing) must be passed.  With ``comm`` (a
    :class:`muserve_b200.distributed.TpComm`) the combine is fused with the sum over the TP
    group (``:657-662`` with ``distributed.py:62-64``) and ``out`` is the all-reduced result."""
    lib = _lib.load()
    assert hidden.dtype == torch.bfloat16 and hidden.dim() == 2 and hidden.is_contiguous()
    t, h = hidden.shape
    ws_struct, info = weights_struct(weights)
    assert info["hidden"] == h
    shape = _lib.MoeShape(tokens=t, hidden=h, num_experts=num_experts, top_k=top_k, inter=info["inter"],
                          shared_inter=info["shared_inter"], placement=placement, tp=tp, rank=rank,
                          add_shared=int(add_shared), combine_mode=combine_mode, weights_dtype=_DT[weights_dtype])
    flags = 0
    if router_logits is None:
        assert topk_w is not None and topk_ids is not None, "need router logits or the routing"
        assert topk_ids.dtype == torch.int32 and topk_w.dtype == weights_dtype
        topk_ids, topk_w = topk_ids.contiguous(), topk_w.contiguous()
        flags |= _lib.FWD_ROUTING_GIVEN
    else:
        assert router_logits.dtype == torch.float32 and router_logits.shape == (t, num_experts)
        router_logits = router_logits.contiguous()
        topk_w = torch.empty(t, top_k, dtype=weights_dtype, device=hidden.device)
        topk_ids = torch.empty(t, top_k, dtype=torch.int32, device=hidden.device)
    if out is None:
        out = torch.empty(t, h, dtype=torch.bfloat16, device=hidden.device)
    nbytes = lib.msv_moe_forward_workspace_size(ctypes_ref(shape))
    if nbytes == 0:
        check(_lib.MSV_ERR_INVALID, "msv_moe_forward_workspace_size")
    ws = _lib.workspace(nbytes, hidden.device)
    if comm is None:
        check(lib.msv_moe_forward(ctypes_ref(shape), ctypes_ref(ws_struct), ptr(hidden), ptr(router_logits),
                                  ptr(topk_w), ptr(topk_ids), ptr(out), flags, ptr(ws), ws.numel(), stream_ptr()),
              "msv_moe_forward")
    else:
        check(lib.msv_moe_forward_tp(ctypes_ref(shape), ctypes_ref(ws_struct), ptr(hidden), ptr(router_logits),
                                     ptr(topk_w), ptr(topk_ids), ptr(out), flags, ptr(ws), ws.numel(),
                                     ctypes_ref(comm.struct), stream_ptr()), "msv_moe_forward_tp")
    if return_routing:
        return out, topk_w, topk_ids
    return out


def ctypes_ref(obj):
    import ctypes
    return ctypes.byref(obj)


def launch_count() -> int:
    """Kernels this library has launched in this process (a graph replay does not count)."""
    return int(_lib.load().msv_launch_count())


def check_device_error() -> None:
    """Raise if a bounded device-side wait timed out since the last check (syncs the stream)."""
    lib = _lib.load()
    check(lib.msv_check_device_error(stream_ptr()), "device")
