"""Batched MoE forward (``muserve/kernels/batched_moe.py:19-115``) on the fused sm_100a path.

Routing as the reference (bf16 router GEMM, fp32 softmax/top-k, bf16 weights), the GEMM on the
library's tensor-core router kernel (``F.linear`` only for shapes it does not take); the weighted
accumulation keeps its order and rounding (local experts ascending,
``out = bf16(out + bf16(d * w))``); the shared expert is added
(on rank 0) in the same combine.  Accepts
the per-expert keys it reads (``moe.expert_{e}.*``) or the stacked ``moe.experts.*``.
"""
from __future__ import annotations

import torch

from .. import _lib, config, moe
from ..distributed import all_reduce, fused_allreduce_comm, get_tp_rank, get_tp_size
from ..loader import stack_per_expert


def batched_moe_forward(hidden: torch.Tensor, weights: dict, *, top_k: int | None = None) -> torch.Tensor:
    k = top_k if top_k is not None else config.NUM_EXPERTS_PER_TOK
    if "moe.experts.gate_proj.weight" not in weights and "moe.experts.gate_up_proj.weight" not in weights:
        n = sum(1 for key in weights if key.endswith(".gate_proj.weight") and key.startswith("moe.expert_"))
        stack_per_expert(weights, n)
    gate_w = weights["moe.gate.weight"]
    num_experts = gate_w.shape[0]
    tp, rank = get_tp_size(), get_tp_rank()
    hidden = hidden.contiguous()
    if hidden.shape[1] % 64 == 0 and num_experts % 16 == 0 and 16 <= num_experts <= 1024:
        # batched_moe.py:28-32: bf16_linear(hidden, gate_w).float() -> softmax -> top-k -> bf16
        topk_w, topk_ids = moe.router_from_hidden(hidden, gate_w, k)
        route = dict(topk_w=topk_w, topk_ids=topk_ids)
    else:
        route = dict(router_logits=torch.nn.functional.linear(hidden, gate_w).float())
    # the shared expert joins the same launch; it is added once (rank 0) before the all-reduce,
    # which differs from the reference's post-all-reduce add only by bf16 rounding at TP > 1
    # with the group's fused buffers (distributed.init_fused_allreduce) the combine kernel sums
    # over the TP group itself; otherwise NCCL's all-reduce follows
    comm = fused_allreduce_comm(hidden.shape[0], hidden.shape[1]) if tp > 1 else None
    out = moe.moe_layer(hidden, weights, top_k=k, num_experts=num_experts, placement=1 if tp > 1 else 0, tp=tp,
                        rank=rank, add_shared=(rank == 0), combine_mode=_lib.COMBINE_BATCHED, comm=comm, **route)
    if comm is None:
        all_reduce(out)
    return out
