"""MoE weights of one layer read straight from a Hugging Face FP8 checkpoint
(``muserve/loader.py:87-264``, the ``mlp.*`` part of ``load_layer_weights``).

Checkpoint layout (``model.safetensors.index.json`` + shards), per layer ``L`` under
``model.language_model.layers.L.`` (``loader.py:98``):

* ``mlp.gate.weight`` [E, H] bf16 (router)
* ``mlp.experts.{e}.{gate,up,down}_proj.weight`` e4m3 [I, H] / [I, H] / [H, I] and
  ``...weight_scale_inv`` [N/128, K/128] (bf16 or f32 in the file; fp32 here, as the
  reference's ``maybe()`` converts every ``scale_inv``, ``loader.py:120-125``)
* ``mlp.shared_expert.{gate,up,down}_proj.weight[_scale_inv]`` and
  ``mlp.shared_expert_gate.weight`` [1, H] bf16

The result is the reference's weights dict (``moe.gate.weight``, ``moe.experts.*`` stacked
``[E_local, N, K]``, ``moe.shared_expert.*``, ``moe.shared_expert_gate.weight``), already in the
layout this package's GEMMs read:

* routed gate and up are written straight into one ``moe.experts.gate_up_proj.*`` tensor
  ``[E_local, 2I, H]`` (the reference concatenates them lazily on first use,
  ``qwen35_layer_v2.py:543-558``), so no second copy is ever made;
* every stacked tensor is allocated once on ``device`` and filled expert by expert, so peak
  host memory is one expert, not the layer;
* ``layout="expert"``: experts ``e % tp == rank`` become local expert ``e // tp``
  (``loader.py:230-264``); router and shared expert are replicated (``:212-228``).
  ``layout="inter"``: every expert, with rows ``[r I/tp, (r+1) I/tp)`` of gate and up and the
  same columns of down (and the shared expert sliced alike); only those rows are read from
  the file.  The dict records the layout under ``"moe.layout"``.
"""
from __future__ import annotations

import json
import os
from collections import defaultdict

import torch

BLOCK = 128
PROJS = ("gate_proj", "up_proj", "down_proj")


def load_index(model_path: str) -> dict:
    """``{tensor name: shard file}`` from ``model.safetensors.index.json`` (``loader.py:30-34``)."""
    with open(os.path.join(model_path, "model.safetensors.index.json")) as f:
        return json.load(f)["weight_map"]


def layer_prefix(layer_idx: int) -> str:
    return f"model.language_model.layers.{layer_idx}."


class _Reader:
    """Opens each shard file once and reads whole tensors or row/column slices of them."""

    def __init__(self, model_path: str, index: dict):
        from safetensors import safe_open
        self._open = safe_open
        self.path = model_path
        self.index = index
        self.files = {}

    def _file(self, name: str):
        if name not in self.index:
            raise KeyError(f"checkpoint has no tensor {name!r}")
        shard = self.index[name]
        if shard not in self.files:
            self.files[shard] = self._open(os.path.join(self.path, shard), framework="pt", device="cpu")
        return self.files[shard]

    def has(self, name: str) -> bool:
        return name in self.index

    def shape(self, name: str) -> list:
        return list(self._file(name).get_slice(name).get_shape())

    def get(self, name: str, rows: slice | None = None, cols: slice | None = None) -> torch.Tensor:
        f = self._file(name)
        if rows is None and cols is None:
            return f.get_tensor(name)
        sl = f.get_slice(name)
        rows = rows if rows is not None else slice(None)
        cols = cols if cols is not None else slice(None)
        return sl[rows, cols]


def _scale(t: torch.Tensor) -> torch.Tensor:
    return t.float()


def load_moe_layer(model_path: str, layer_idx: int, tp: int = 1, rank: int = 0, layout: str = "expert",
                   device="cpu", weight_index: dict | None = None, fuse_gate_up: bool = True) -> dict:
    """One layer's MoE weights dict for TP rank ``rank`` of ``tp`` (see the module docstring)."""
    if layout not in ("expert", "inter"):
        raise ValueError(f"layout must be 'expert' or 'inter', not {layout!r}")
    if not (0 <= rank < tp):
        raise ValueError(f"rank {rank} outside tp {tp}")
    index = weight_index if weight_index is not None else load_index(model_path)
    rd = _Reader(model_path, index)
    p = layer_prefix(layer_idx)
    device = torch.device(device)
    out: dict = {}

    gate = p + "mlp.gate.weight"
    out["moe.gate.weight"] = rd.get(gate).to(device)
    num_experts, hidden = out["moe.gate.weight"].shape

    # routed experts present in the checkpoint
    present = defaultdict(set)
    ep = p + "mlp.experts."
    for name in index:
        if name.startswith(ep):
            e, rest = name[len(ep):].split(".", 1)
            present[int(e)].add(rest)
    if sorted(present) != list(range(num_experts)):
        raise KeyError(f"layer {layer_idx}: experts in the checkpoint are not 0..{num_experts - 1}")
    inter = rd.shape(ep + "0.gate_proj.weight")[0]
    if inter % BLOCK or hidden % BLOCK:
        raise ValueError(f"inter {inter} and hidden {hidden} must be multiples of {BLOCK}")

    if layout == "expert":
        if num_experts % tp:
            raise ValueError(f"{num_experts} experts do not split over tp {tp}")
        experts = list(range(rank, num_experts, tp))
        i_loc, r0 = inter, 0
    else:
        if inter % (tp * BLOCK):
            raise ValueError(f"inter {inter} / tp {tp} must be whole {BLOCK}-blocks")
        experts = list(range(num_experts))
        i_loc, r0 = inter // tp, rank * (inter // tp)
    rows = slice(r0, r0 + i_loc)
    srows = slice(r0 // BLOCK, (r0 + i_loc) // BLOCK)
    kb_h, kb_i = hidden // BLOCK, i_loc // BLOCK
    n_loc = len(experts)

    def empty(shape, like: torch.Tensor):
        return torch.empty(shape, dtype=like.dtype, device=device)

    stacks: dict = {}
    for j, e in enumerate(experts):
        base = f"{ep}{e}."
        g = rd.get(base + "gate_proj.weight", rows=rows)
        u = rd.get(base + "up_proj.weight", rows=rows)
        gs = _scale(rd.get(base + "gate_proj.weight_scale_inv", rows=srows))
        us = _scale(rd.get(base + "up_proj.weight_scale_inv", rows=srows))
        d = rd.get(base + "down_proj.weight", cols=rows)
        ds = _scale(rd.get(base + "down_proj.weight_scale_inv", cols=srows))
        if g.shape != (i_loc, hidden) or d.shape != (hidden, i_loc) or gs.shape != (kb_i, kb_h) or ds.shape != (kb_h, kb_i):
            raise ValueError(f"expert {e}: unexpected shapes {tuple(g.shape)} {tuple(d.shape)} {tuple(gs.shape)} {tuple(ds.shape)}")
        if j == 0:
            if fuse_gate_up:
                stacks["moe.experts.gate_up_proj.weight"] = empty((n_loc, 2 * i_loc, hidden), g)
                stacks["moe.experts.gate_up_proj.weight_scale_inv"] = empty((n_loc, 2 * kb_i, kb_h), gs)
            else:
                stacks["moe.experts.gate_proj.weight"] = empty((n_loc, i_loc, hidden), g)
                stacks["moe.experts.up_proj.weight"] = empty((n_loc, i_loc, hidden), u)
                stacks["moe.experts.gate_proj.weight_scale_inv"] = empty((n_loc, kb_i, kb_h), gs)
                stacks["moe.experts.up_proj.weight_scale_inv"] = empty((n_loc, kb_i, kb_h), us)
            stacks["moe.experts.down_proj.weight"] = empty((n_loc, hidden, i_loc), d)
            stacks["moe.experts.down_proj.weight_scale_inv"] = empty((n_loc, kb_h, kb_i), ds)
        if fuse_gate_up:
            stacks["moe.experts.gate_up_proj.weight"][j, :i_loc].copy_(g)
            stacks["moe.experts.gate_up_proj.weight"][j, i_loc:].copy_(u)
            stacks["moe.experts.gate_up_proj.weight_scale_inv"][j, :kb_i].copy_(gs)
            stacks["moe.experts.gate_up_proj.weight_scale_inv"][j, kb_i:].copy_(us)
        else:
            stacks["moe.experts.gate_proj.weight"][j].copy_(g)
            stacks["moe.experts.up_proj.weight"][j].copy_(u)
            stacks["moe.experts.gate_proj.weight_scale_inv"][j].copy_(gs)
            stacks["moe.experts.up_proj.weight_scale_inv"][j].copy_(us)
        stacks["moe.experts.down_proj.weight"][j].copy_(d)
        stacks["moe.experts.down_proj.weight_scale_inv"][j].copy_(ds)
    out.update(stacks)

    # shared expert (replicated in the expert layout, sliced like the routed experts otherwise)
    sp = p + "mlp.shared_expert."
    if rd.has(sp + "gate_proj.weight"):
        s_inter = rd.shape(sp + "gate_proj.weight")[0]
        if layout == "inter":
            if s_inter % (tp * BLOCK):
                raise ValueError(f"shared inter {s_inter} / tp {tp} must be whole {BLOCK}-blocks")
            n = s_inter // tp
            srow, sblk = slice(rank * n, (rank + 1) * n), slice(rank * n // BLOCK, (rank + 1) * n // BLOCK)
        else:
            srow = sblk = None
        for proj in ("gate_proj", "up_proj"):
            out[f"moe.shared_expert.{proj}.weight"] = rd.get(sp + f"{proj}.weight", rows=srow).to(device)
            out[f"moe.shared_expert.{proj}.weight_scale_inv"] = _scale(
                rd.get(sp + f"{proj}.weight_scale_inv", rows=sblk)).to(device)
        out["moe.shared_expert.down_proj.weight"] = rd.get(sp + "down_proj.weight", cols=srow).to(device)
        out["moe.shared_expert.down_proj.weight_scale_inv"] = _scale(
            rd.get(sp + "down_proj.weight_scale_inv", cols=sblk)).to(device)
    if rd.has(p + "mlp.shared_expert_gate.weight"):
        out["moe.shared_expert_gate.weight"] = rd.get(p + "mlp.shared_expert_gate.weight").to(device)
    for k in list(out):
        if torch.is_tensor(out[k]) and not out[k].is_contiguous():
            out[k] = out[k].contiguous()
    out["moe.layout"] = layout
    return out
