"""Kernel-layer MoE routing and expert compute (``muserve/kernels/moe_dispatch.py``).

``moe_experts_fp8`` keeps the reference's signature, but quantises activations with the V2
dynamic per-token-per-128-channel scales (``qwen35_layer_v2.py:71-86``) instead of the
reference's direct e4m3 cast with unit scales (``moe_dispatch.py:50-58``, ``:66-72``), which
clips activations above 448 and flushes small ones; the weighted accumulation keeps the
reference's order and rounding (experts ascending, ``out = bf16(out + d * w_fp32)``).
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from .. import _lib, config, moe


def moe_gate(hidden: torch.Tensor, gate_weight: torch.Tensor, top_k: int | None = None):
    """Routing scores and top-k (``moe_dispatch.py:8-24``): fp32 logits, softmax, top-k,
    renormalise.  Returns ``(topk_ids [T,k] int32, topk_weights [T,k] fp32)``."""
    k = top_k if top_k is not None else config.NUM_EXPERTS_PER_TOK
    t, h = hidden.shape
    e = gate_weight.shape[0]
    if (hidden.dtype == torch.bfloat16 and gate_weight.dtype == torch.bfloat16 and h % 64 == 0 and e % 16 == 0
            and 16 <= e <= 1024):
        # bf16 products are exact in fp32, so the tensor-core GEMM with fp32 accumulation and no
        # final rounding computes the reference's fp32 linear up to the order of the fp32 sum
        w, ids = moe.router_from_hidden(hidden, gate_weight, k, round_logits_bf16=False, w_dtype=torch.float32)
        return ids, w
    logits = F.linear(hidden.float(), gate_weight.float())
    w, ids = moe.route_topk(logits.contiguous(), k, renormalize=True, w_dtype=torch.float32, ids_dtype=torch.int32)
    return ids, w


def moe_experts_fp8(hidden: torch.Tensor, topk_ids: torch.Tensor, topk_weights: torch.Tensor,
                    gate_up_weight: torch.Tensor, gate_up_scale: torch.Tensor,
                    down_weight: torch.Tensor, down_scale: torch.Tensor) -> torch.Tensor:
    """Expert computation with FP8 GEMMs (``moe_dispatch.py:27-79``): ``[T,H]`` bf16."""
    assert hidden.dtype == torch.bfloat16
    e = gate_up_weight.shape[0]
    weights = {"moe.experts.gate_up_proj.weight": gate_up_weight.contiguous(),
               "moe.experts.gate_up_proj.weight_scale_inv": gate_up_scale.float().contiguous(),
               "moe.experts.down_proj.weight": down_weight.contiguous(),
               "moe.experts.down_proj.weight_scale_inv": down_scale.float().contiguous()}
    return moe.moe_layer(hidden.contiguous(), weights, top_k=topk_ids.shape[1], num_experts=e,
                         topk_w=topk_weights.float().contiguous(), topk_ids=topk_ids.to(torch.int32).contiguous(),
                         combine_mode=_lib.COMBINE_DISPATCH, weights_dtype=torch.float32)
