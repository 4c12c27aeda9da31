"""Tensor-parallel layout of one MoE layer's weights dict (``muserve/loader.py``).

Two layouts, both keyed like the reference's dict (``loader.py:212-264``):

* ``"inter"`` (intermediate sharding): rank r keeps rows ``[r*I/tp, (r+1)*I/tp)`` of every
  expert's gate and up projections (column-parallel, ``_col_shard`` semantics along the
  output dim, ``loader.py:52-55``) and the same columns of down (row-parallel,
  ``_row_shard``, ``loader.py:58-61``), scales sliced by the same 128-blocks; the shared
  expert is sharded the same way; router and shared-expert gate are replicated.  Each rank
  produces a partial [T,H] and one all-reduce sums them.
* ``"expert"`` (the reference's own placement): rank r keeps whole experts
  ``e % tp == r`` stacked as local expert ``e // tp`` (``loader.py:230-264``); router and
  shared expert replicated (``loader.py:212-228``).

The layout is recorded in the dict under ``"moe.layout"`` (a str, not a tensor).
"""
from __future__ import annotations

import torch

BLOCK = 128


def _col_shard(t: torch.Tensor, rank: int, tp: int, dim: int) -> torch.Tensor:
    n = t.shape[dim] // tp
    return t.narrow(dim, rank * n, n).contiguous()


def shard_moe_weights(weights: dict, tp: int, rank: int, layout: str = "inter") -> dict:
    """This rank's view of a full (TP=1) MoE weights dict."""
    assert layout in ("inter", "expert")
    out = {}
    if layout == "expert":
        for key, t in weights.items():
            if key.startswith("moe.experts."):
                out[key] = t[rank::tp].contiguous()
            else:
                out[key] = t
        out["moe.layout"] = "expert"
        return out
    for key, t in weights.items():
        if not torch.is_tensor(t):
            continue
        if key in ("moe.gate.weight", "moe.shared_expert_gate.weight"):
            out[key] = t
            continue
        is_scale = key.endswith("weight_scale_inv")
        if key.startswith("moe.experts.gate_up_proj"):
            raise ValueError("shard before fusing gate and up")
        if key.startswith(("moe.experts.gate_proj", "moe.experts.up_proj")):
            n = t.shape[1]
            assert n % tp == 0 and (is_scale or (n // tp) % BLOCK == 0), "I/tp must be whole 128-blocks"
            out[key] = _col_shard(t, rank, tp, 1)
        elif key.startswith("moe.experts.down_proj"):
            out[key] = _col_shard(t, rank, tp, 2)
        elif key.startswith(("moe.shared_expert.gate_proj", "moe.shared_expert.up_proj")):
            out[key] = _col_shard(t, rank, tp, 0)
        elif key.startswith("moe.shared_expert.down_proj"):
            out[key] = _col_shard(t, rank, tp, 1)
        else:
            out[key] = t
    out["moe.layout"] = "inter"
    return out


def fuse_gate_up(weights: dict) -> dict:
    """``cat([gate, up], dim=1)`` of the routed experts' weights and scales, as the reference
    does lazily (``qwen35_layer_v2.py:543-558``).  Returns a new dict."""
    out = {k: v for k, v in weights.items()
           if not k.startswith(("moe.experts.gate_proj", "moe.experts.up_proj"))}
    out["moe.experts.gate_up_proj.weight"] = torch.cat(
        [weights["moe.experts.gate_proj.weight"], weights["moe.experts.up_proj.weight"]], dim=1)
    out["moe.experts.gate_up_proj.weight_scale_inv"] = torch.cat(
        [weights["moe.experts.gate_proj.weight_scale_inv"], weights["moe.experts.up_proj.weight_scale_inv"]], dim=1)
    return out


def stack_per_expert(weights: dict, num_local: int) -> dict:
    """Stack per-expert ``moe.expert_{e}.{proj}.weight[_scale_inv]`` keys into
    ``moe.experts.{proj}.*`` ``[E_local, N, K]`` tensors (``loader.py:246-264``), in place."""
    for proj in ("gate_proj", "up_proj", "down_proj"):
        for suf in ("weight", "weight_scale_inv"):
            keys = [f"moe.expert_{e}.{proj}.{suf}" for e in range(num_local)]
            if all(k in weights for k in keys):
                weights[f"moe.experts.{proj}.{suf}"] = torch.stack([weights.pop(k) for k in keys]).contiguous()
    return weights
