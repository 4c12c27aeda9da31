"""MoE half of the reference's active layer (``muserve/model/qwen35_layer_v2.py``) on sm_100a.

``moe_forward(hidden, weights)`` keeps the reference's signature and weights-dict contract
(``:561``, ``loader.py:212-264``).  The router (``:567-572``) runs as the library's router GEMM
on the tensor cores (bf16 x bf16 -> fp32, rounded to bf16 as ``bf16_linear(...).float()``) plus
softmax / top-k; shapes that GEMM does not take (H % 64, E % 16) use ``F.linear`` and the
library's top-k.  Everything after it runs in the library's layer kernels (dispatch,
gather+quantise, gate_up GEMM with SwiGLU+requant epilogue, down GEMM, combine + shared
expert).  With tensor parallelism the per-rank partial ``[T,H]`` is all-reduced once
(the V1 / BASELINE placement, ``qwen35_layer.py:565-571``) instead of V2's ``[T*k,H]``
buffer (``:652-657``); results differ from V2 only by bf16 rounding of partial sums.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from .. import config, moe
from ..distributed import all_reduce, fused_allreduce_comm, get_tp_rank, get_tp_size


def rms_norm_gemma(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """Gemma-style RMS norm, the weight stored as an offset from 1.0 (``:59-62``), on the GPU
    kernel: ``bf16(x * rsqrt(mean(x^2) + eps) * bf16(1 + weight))``."""
    shape = x.shape
    out = moe.add_rms_norm_gemma(x.reshape(-1, shape[-1]).contiguous(), weight.contiguous(), eps=eps)
    return out.reshape(shape)


def _fast_fp8_quantize(x: torch.Tensor, block_size: int = 128):
    """Per-token per-128-channel e4m3 quantisation (``:71-86``): ``(x_fp8 [M,K], x_scale [M,K/128])``."""
    assert block_size == 128, "only 128-channel blocks"
    orig = x.shape
    x2 = x.reshape(-1, orig[-1])
    assert x2.shape[1] % block_size == 0, f"K={x2.shape[1]} not divisible by block_size={block_size}"
    q, s = moe.fp8_quant_128(x2.contiguous())
    return q, s


def fp8_linear(x: torch.Tensor, w_fp8: torch.Tensor, w_scale: torch.Tensor) -> torch.Tensor:
    """``x [..., K] @ w [N, K]^T`` with dynamic per-128 activation quantisation (``:89-107``)."""
    orig = x.shape
    xq, xs = _fast_fp8_quantize(x.reshape(-1, orig[-1]))
    out = moe.gemm_nt(xq, xs, w_fp8, w_scale)
    return out.reshape(*orig[:-1], w_fp8.shape[0])


def bf16_linear(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """``F.linear`` in bf16 (``:110-112``)."""
    return F.linear(x, w)


def linear_maybe_fp8(x: torch.Tensor, weights: dict, prefix: str) -> torch.Tensor:
    w = weights[f"{prefix}.weight"]
    s = weights.get(f"{prefix}.weight_scale_inv")
    return fp8_linear(x, w, s) if s is not None else bf16_linear(x, w)


def _layout(weights: dict, num_experts: int, tp: int) -> str:
    lay = weights.get("moe.layout")
    if lay is not None:
        return lay
    if tp == 1:
        return "inter"
    w = weights.get("moe.experts.gate_proj.weight", weights.get("moe.experts.gate_up_proj.weight"))
    return "expert" if w.shape[0] * tp == num_experts else "inter"


def moe_forward(hidden: torch.Tensor, weights: dict, *, top_k: int | None = None,
                return_routing: bool = False, logit_bias: torch.Tensor | None = None) -> torch.Tensor:
    """MoE forward. hidden: [total, HIDDEN] bf16 -> output: [total, HIDDEN] bf16 (``:561-675``).
    ``logit_bias`` ([E] fp32, not in the reference) is added to the router logits: the expert
    popularity prior of the 60-layer stack benchmark."""
    k = top_k if top_k is not None else config.NUM_EXPERTS_PER_TOK
    gate_w = weights["moe.gate.weight"]
    num_experts = gate_w.shape[0]
    tp, rank = get_tp_size(), get_tp_rank()
    hidden = hidden.contiguous()
    lay = _layout(weights, num_experts, tp)
    placement = 1 if (tp > 1 and lay == "expert") else 0
    if hidden.shape[1] % 64 == 0 and num_experts % 16 == 0 and 16 <= num_experts <= 1024:
        topk_w, topk_ids = moe.router_from_hidden(hidden, gate_w, k, logit_bias=logit_bias)  # :567-572
        route = dict(topk_w=topk_w, topk_ids=topk_ids)
    else:
        logits = bf16_linear(hidden, gate_w).float()                                 # :568
        route = dict(router_logits=logits if logit_bias is None else logits + logit_bias)
    # with the group's fused buffers the combine sums over the TP group itself (peer memory)
    comm = fused_allreduce_comm(hidden.shape[0], hidden.shape[1]) if tp > 1 else None
    res = moe.moe_layer(hidden, weights, top_k=k, num_experts=num_experts, placement=placement, tp=tp,
                        rank=rank, add_shared=(placement == 0 or rank == 0), return_routing=return_routing,
                        comm=comm, **route)
    out = res[0] if return_routing else res
    if tp > 1 and comm is None:
        all_reduce(out)
    return res if return_routing else out
