"""Seeded synthetic MoE layers on the GPU (there is no checkpoint here).

Same recipe as the CPU oracle's ``make_layer_weights``: every weight is drawn fp32
``N(0, 0.02)`` and quantised per 128x128 block (``s = amax/448`` stored as
``*_weight_scale_inv``, ``w = clamp(W/s) -> e4m3``); router gate and shared-expert gate are
bf16 ``N(0, 0.02)``.  Draws come from a CUDA generator, so values differ from the CPU
oracle's stream; parity tests hand the very same tensors to both sides.
"""
from __future__ import annotations

import torch

FP8 = torch.float8_e4m3fn
BLOCK = 128


def quantize_blockwise(w: torch.Tensor):
    n, k = w.shape
    wb = w.view(n // BLOCK, BLOCK, k // BLOCK, BLOCK)
    s = wb.abs().amax(dim=(1, 3)).clamp(min=1e-12) / 448.0
    q = (wb / s[:, None, :, None]).clamp(-448.0, 448.0).to(FP8).view(n, k)
    return q, s.contiguous()


@torch.no_grad()
def make_layer_weights(hidden: int, experts: int, inter: int, shared_inter: int = 0, shared_gate: bool = True,
                       seed: int = 0, device="cuda", std: float = 0.02, fused_gate_up: bool = False) -> dict:
    g = torch.Generator(device=device).manual_seed(seed)

    def randn(*shape):
        return torch.randn(*shape, generator=g, device=device, dtype=torch.float32) * std

    w = {"moe.gate.weight": randn(experts, hidden).to(torch.bfloat16)}
    gq = torch.empty(experts, inter, hidden, dtype=FP8, device=device)
    uq = torch.empty_like(gq)
    dq = torch.empty(experts, hidden, inter, dtype=FP8, device=device)
    gs = torch.empty(experts, inter // BLOCK, hidden // BLOCK, dtype=torch.float32, device=device)
    us = torch.empty_like(gs)
    ds = torch.empty(experts, hidden // BLOCK, inter // BLOCK, dtype=torch.float32, device=device)
    for e in range(experts):
        gq[e], gs[e] = quantize_blockwise(randn(inter, hidden))
        uq[e], us[e] = quantize_blockwise(randn(inter, hidden))
        dq[e], ds[e] = quantize_blockwise(randn(hidden, inter))
    if fused_gate_up:
        w["moe.experts.gate_up_proj.weight"] = torch.cat([gq, uq], dim=1)
        w["moe.experts.gate_up_proj.weight_scale_inv"] = torch.cat([gs, us], dim=1)
        del gq, uq
    else:
        w["moe.experts.gate_proj.weight"], w["moe.experts.gate_proj.weight_scale_inv"] = gq, gs
        w["moe.experts.up_proj.weight"], w["moe.experts.up_proj.weight_scale_inv"] = uq, us
    w["moe.experts.down_proj.weight"], w["moe.experts.down_proj.weight_scale_inv"] = dq, ds
    if shared_inter:
        for name, shape in (("gate_proj", (shared_inter, hidden)), ("up_proj", (shared_inter, hidden)),
                            ("down_proj", (hidden, shared_inter))):
            q, s = quantize_blockwise(randn(*shape))
            w[f"moe.shared_expert.{name}.weight"] = q
            w[f"moe.shared_expert.{name}.weight_scale_inv"] = s
        if shared_gate:
            w["moe.shared_expert_gate.weight"] = randn(1, hidden).to(torch.bfloat16)
    return w


def make_hidden(tokens: int, hidden: int, seed: int, device="cuda") -> torch.Tensor:
    g = torch.Generator(device=device).manual_seed(seed)
    return torch.randn(tokens, hidden, generator=g, device=device).to(torch.bfloat16)


def uniform_logits(tokens: int, experts: int, seed: int, device="cuda") -> torch.Tensor:
    g = torch.Generator(device=device).manual_seed(seed)
    return torch.rand(tokens, experts, generator=g, device=device)


def zipf_bias(experts: int, s: float = 1.2, seed: int = 0, device="cuda") -> torch.Tensor:
    """``log p_{pi(e)}`` with ``p_i ∝ i^-s`` over a seeded permutation (expert popularity)."""
    g = torch.Generator().manual_seed(seed)
    ranks = torch.arange(1, experts + 1, dtype=torch.float64)
    p = ranks.pow(-s)
    p = p / p.sum()
    perm = torch.randperm(experts, generator=g)
    return p.log()[perm].float().to(device)


def to_cpu(weights: dict, experts=None) -> dict:
    """CPU copy of a weights dict, optionally only some routed experts (kept in place, the others
    zero-free: their slots are left out by indexing ``experts``)."""
    out = {}
    for k, v in weights.items():
        if not torch.is_tensor(v):
            out[k] = v
        elif k.startswith("moe.experts.") and experts is not None:
            idx = torch.as_tensor(sorted(experts), device=v.device)
            full = torch.zeros((v.shape[0],) + tuple(v.shape[1:]), dtype=v.dtype)
            full[idx.cpu()] = v[idx].cpu()
            out[k] = full
        else:
            out[k] = v.cpu()
    return out
