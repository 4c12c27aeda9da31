"""CPU oracle for muserve's FP8 MoE path (TEST INFRASTRUCTURE ONLY).

This module restates, in plain torch-on-CPU code, the algorithm of the reference's
active MoE layer, ``muserve/model/qwen35_layer_v2.py:561-675`` (``moe_forward``), stage
by stage, so that every intermediate of the CUDA path can be checked against it.

Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference``
legs of ``bench.py`` may import this module, and only as the checker or the timed CPU
baseline.  The product path (``muserve_b200``) never calls it.

Parity status
-------------
* Router, permutation, padding, FP8 activation quantisation, SwiGLU, unsort, weighted
  combine and the shared-expert glue are restated from the reference lines cited on each
  function.  They are pinned against the reference's own ``moe_forward`` executed on this
  CPU (``tests/golden/make_golden.py`` imports the reference, stubs the MUSA-only modules
  and records every intermediate).
* The two FP8 GEMMs live in the third-party library ``mate 0.2.1+mu436``
  (``muserve/docs/SPEC.md:88``), which is neither vendored nor installed.  Their
  arithmetic is restated from the call sites (``qwen35_layer_v2.py:102-106,613-618,
  638-643``; ``qwen35_layer.py:496`` for the ``-1`` rows) as "dequantise with the
  per-row x per-128 activation scale and the 128x128 weight scale, multiply in fp32, round
  to bf16".  No reference test pins their results, so for the GEMMs parity is UNPINNED:
  the golden run uses this same restatement inside its ``mate.gemm`` stub.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch
import torch.nn.functional as F

FP8 = torch.float8_e4m3fn
FP8_MAX = 448.0
BLOCK = 128


# ─────────────────────────────────────────────────────────────────────────────
# FP8 helpers
# ─────────────────────────────────────────────────────────────────────────────

def fast_fp8_quantize(x: torch.Tensor, block_size: int = BLOCK):
    """Per-row, per-128-channel e4m3 quantisation.

    Restates ``qwen35_layer_v2.py:71-86``: ``s = clamp(amax(|x|), 1e-12) / 448`` in fp32,
    ``q = clamp(x / s, -448, 448) -> float8_e4m3fn``.  Returns ``(q [M,K], s [M,K/128])``.
    """
    x2 = x.reshape(-1, x.shape[-1])
    m, k = x2.shape
    assert k % block_size == 0, f"K={k} not divisible by block_size={block_size}"
    xb = x2.view(m, k // block_size, block_size).float()
    s = xb.abs().amax(dim=-1).clamp(min=1e-12) / FP8_MAX
    q = (xb / s.unsqueeze(-1)).clamp(-FP8_MAX, FP8_MAX).to(FP8).view(m, k).contiguous()
    return q, s.contiguous()


def dequant_weight(w: torch.Tensor, s: torch.Tensor) -> torch.Tensor:
    """fp32 value of a 128x128 block-scaled e4m3 weight ``w [N,K]`` with ``s [N/128,K/128]``."""
    n, k = w.shape
    if n % BLOCK == 0 and k % BLOCK == 0:
        # the same per-element products, by broadcasting instead of materialising the scales
        wb = w.float().view(n // BLOCK, BLOCK, k // BLOCK, BLOCK)
        return (wb * s.float()[:, None, :, None]).view(n, k)
    sf = s.float().repeat_interleave(BLOCK, 0)[:n].repeat_interleave(BLOCK, 1)[:, :k]
    return w.float() * sf


def dequant_act(a: torch.Tensor, s: torch.Tensor) -> torch.Tensor:
    """fp32 value of a per-row per-128 scaled e4m3 activation ``a [M,K]``, ``s [M,K/128]``."""
    return a.float() * s.float().repeat_interleave(BLOCK, 1)[:, : a.shape[1]]


def gemm_fp8_nt_groupwise(a, b, a_scale, b_scale, scale_granularity_mnk=(1, 128, 128),
                          out_dtype=torch.bfloat16):
    """Restated ``mate.gemm.gemm_fp8_nt_groupwise`` (call site ``qwen35_layer_v2.py:102-106``).

    ``out[m,n] = sum_k (a[m,k] a_s[m,k/128]) (b[n,k] b_s[n/128,k/128])``, fp32, then rounded
    to ``out_dtype``.  Third-party semantics inferred from the call site: parity unpinned.
    """
    assert tuple(scale_granularity_mnk) == (1, 128, 128)
    return (dequant_act(a, a_scale) @ dequant_weight(b, b_scale).t()).to(out_dtype)


def ragged_m_moe_gemm_8bit(a_pair, w_pair, m_indices, out):
    """Restated ``mate.gemm.ragged_m_moe_gemm_8bit`` (call sites ``qwen35_layer_v2.py:613-618``,
    ``:638-643``; ``qwen35_layer.py:534-546``).

    Row ``m`` of ``out`` is ``gemm(a[m], w[m_indices[m]])`` rounded to bf16; rows whose index
    is ``-1`` are left untouched (``qwen35_layer.py:496``).  Parity unpinned (third-party).
    """
    a, a_s = a_pair
    w, w_s = w_pair
    ids = m_indices.long()
    a_deq = dequant_act(a, a_s)
    for e in torch.unique(ids).tolist():
        if e < 0:
            continue
        rows = (ids == e).nonzero(as_tuple=True)[0]
        out[rows] = (a_deq[rows] @ dequant_weight(w[e], w_s[e]).t()).to(out.dtype)
    return out


def bf16_linear(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """``F.linear`` in bf16 (``qwen35_layer_v2.py:110-112``)."""
    return F.linear(x, w)


def fp8_linear(x: torch.Tensor, w: torch.Tensor, w_s: torch.Tensor) -> torch.Tensor:
    """Quantise ``x`` per 128 channels, then block-scaled GEMM (``qwen35_layer_v2.py:89-107``)."""
    shp = x.shape
    xq, xs = fast_fp8_quantize(x.reshape(-1, shp[-1]))
    return gemm_fp8_nt_groupwise(xq, w, xs, w_s).reshape(*shp[:-1], w.shape[0])


# ─────────────────────────────────────────────────────────────────────────────
# Router and permutation
# ─────────────────────────────────────────────────────────────────────────────

def route(logits: torch.Tensor, k: int, weight_dtype=torch.bfloat16):
    """Softmax -> top-k -> renormalise -> cast (``qwen35_layer_v2.py:568-572``).

    ``logits`` is the fp32 view of the router GEMM output.  Returns
    ``(topk_w [T,k] weight_dtype, topk_ids [T,k] int64)``.  The top-k order among equal
    scores is whatever torch's CPU kernel produces; the CUDA router reproduces it.
    """
    scores = torch.softmax(logits.float(), dim=-1)
    w, ids = torch.topk(scores, k, dim=-1)
    w = w / w.sum(dim=-1, keepdim=True)
    return w.to(weight_dtype), ids


def route_biased(logits: torch.Tensor, logit_bias: torch.Tensor, k: int, weight_dtype=torch.bfloat16):
    """:func:`route` on ``logits + logit_bias`` (fp32 add): the 60-layer stack benchmark's
    expert-popularity prior on top of the router logits (not a reference op)."""
    return route(logits.float() + logit_bias.float(), k, weight_dtype)


def rms_norm_gemma(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """Gemma-style RMS norm (``qwen35_layer_v2.py:59-62``): ``w = bf16(1 + float(weight))``,
    then ``F.rms_norm`` on the bf16 input, which on the CPU computes in fp32 and rounds once."""
    w = (1.0 + weight.float()).to(x.dtype)
    return torch.nn.functional.rms_norm(x, (x.shape[-1],), w, eps).to(x.dtype)


def moe_block(h: torch.Tensor, weights: dict, num_experts: int, k: int, logit_bias=None, eps: float = 1e-6):
    """The MoE half of the decode layer (``qwen35_layer_v2.py:712-715``):
    ``h + moe_forward(rms_norm_gemma(h, post_attention_layernorm.weight))``, with the router
    logits from the bf16 gate GEMM (plus an optional prior) routed by :func:`route`."""
    x2 = rms_norm_gemma(h, weights["post_attention_layernorm.weight"], eps)
    logits = bf16_linear(x2, weights["moe.gate.weight"]).float()
    if logit_bias is not None:
        logits = logits + logit_bias.float()
    return h + moe_forward(x2, weights, num_experts, k, logits=logits)


def moe_gate(hidden: torch.Tensor, gate_weight: torch.Tensor, k: int):
    """Kernel-layer router with fp32 logits (``muserve/kernels/moe_dispatch.py:8-24``)."""
    logits = F.linear(hidden.float(), gate_weight.float())
    scores = torch.softmax(logits, dim=-1)
    w, ids = torch.topk(scores, k, dim=-1)
    w = w / w.sum(dim=-1, keepdim=True)
    return ids.to(torch.int32), w


@dataclass
class Permutation:
    """Outputs of the dispatch bookkeeping (``qwen35_layer_v2.py:574-605``)."""
    local_mask: torch.Tensor          # [T*k] bool
    local_indices: torch.Tensor       # [P_local] int64 flat slot of each local row
    sort_order: torch.Tensor          # [P_local] int64 (argsort(local ids, stable))
    inverse_order: torch.Tensor       # [P_local] int64
    sorted_expert_ids: torch.Tensor   # [Mpad] int32, -1 padding
    sorted_token_idx: torch.Tensor    # [P_local] int64 token of each sorted row
    num_local: int
    padded_m: int
    expert_counts: torch.Tensor = field(default=None)  # [E_local] int64


def permute(topk_ids: torch.Tensor, num_experts: int, tp: int = 1, rank: int = 0,
            alignment: int = 128) -> Permutation:
    """Expand, filter local experts, stable sort, pad (``qwen35_layer_v2.py:574-605``)."""
    t, k = topk_ids.shape
    flat_ids = topk_ids.reshape(-1)
    token_idx = torch.arange(t).repeat_interleave(k)               # :536-540
    local_mask = (flat_ids % tp) == rank                            # :581
    local_expert_ids = flat_ids[local_mask] // tp                   # :582
    local_indices = torch.where(local_mask)[0]                      # :653
    num_local = int(local_expert_ids.numel())
    sort_order = local_expert_ids.argsort(stable=True)              # :587
    sorted_expert_ids = local_expert_ids[sort_order].to(torch.int32)  # :589
    inverse_order = sort_order.argsort()                            # :590
    padded_m = ((num_local + alignment - 1) // alignment) * alignment  # :595
    if padded_m > num_local:                                        # :596-602
        sorted_expert_ids = torch.cat(
            [sorted_expert_ids, torch.full((padded_m - num_local,), -1, dtype=torch.int32)])
    counts = torch.bincount(local_expert_ids, minlength=num_experts // tp)
    return Permutation(local_mask, local_indices, sort_order, inverse_order,
                       sorted_expert_ids, token_idx[local_mask][sort_order], num_local,
                       padded_m, counts)


# ─────────────────────────────────────────────────────────────────────────────
# Whole layer
# ─────────────────────────────────────────────────────────────────────────────

def fused_gate_up(weights: dict):
    """``cat([gate, up], dim=1)`` of routed-expert weights and scales (``qwen35_layer_v2.py:543-558``).
    Unlike the reference this does not mutate ``weights``."""
    if "moe.experts.gate_up_proj.weight" in weights:
        return (weights["moe.experts.gate_up_proj.weight"],
                weights["moe.experts.gate_up_proj.weight_scale_inv"])
    w = torch.cat([weights["moe.experts.gate_proj.weight"],
                   weights["moe.experts.up_proj.weight"]], dim=1)
    s = torch.cat([weights["moe.experts.gate_proj.weight_scale_inv"],
                   weights["moe.experts.up_proj.weight_scale_inv"]], dim=1)
    return w, s


def moe_forward_stages(hidden: torch.Tensor, weights: dict, num_experts: int, k: int,
                       tp: int = 1, rank: int = 0, logits: torch.Tensor | None = None,
                       all_reduce=None) -> dict:
    """Every intermediate of ``moe_forward`` (``qwen35_layer_v2.py:561-675``), TP placement
    ``expert % tp == rank`` as in the reference.

    ``logits`` (fp32 ``[T,E]``) replaces the router GEMM when given, so the CUDA path and the
    oracle can be compared on identical logits.  ``all_reduce`` is called on the
    ``[T*k, H]`` buffer when ``tp > 1`` (``:657``).
    """
    out = {}
    total, hsz = hidden.shape
    if logits is None:
        logits = bf16_linear(hidden, weights["moe.gate.weight"]).float()       # :568
    out["logits"] = logits
    topk_w, topk_ids = route(logits, k)                                          # :569-572
    out["topk_w"], out["topk_ids"] = topk_w, topk_ids
    perm = permute(topk_ids, num_experts, tp, rank)                              # :574-605
    out["perm"] = perm
    nl, mp = perm.num_local, perm.padded_m
    sorted_tokens = hidden[perm.sorted_token_idx]                                # :578,588
    pad = torch.zeros(mp - nl, hsz, dtype=hidden.dtype)
    sorted_tokens_padded = torch.cat([sorted_tokens, pad], 0)                    # :597-599
    w_gu, s_gu = fused_gate_up(weights)                                          # :609
    inter = w_gu.shape[1] // 2
    x_fp8, x_scale = fast_fp8_quantize(sorted_tokens_padded)                     # :612
    out["x_fp8"], out["x_scale"] = x_fp8, x_scale
    gate_up = torch.empty(mp, 2 * inter, dtype=torch.bfloat16)
    ragged_m_moe_gemm_8bit((x_fp8, x_scale), (w_gu, s_gu), perm.sorted_expert_ids, gate_up)
    gate_up = gate_up[:nl]                                                       # :619
    out["gate_up"] = gate_up
    act = F.silu(gate_up[:, :inter]) * gate_up[:, inter:]                        # :622-624
    out["act"] = act
    act_padded = torch.zeros(mp, inter, dtype=act.dtype)                         # :631-634
    act_padded[:nl] = act
    act_fp8, act_scale = fast_fp8_quantize(act_padded)                           # :637
    out["act_fp8"], out["act_scale"] = act_fp8, act_scale
    down = torch.empty(mp, hsz, dtype=torch.bfloat16)
    ragged_m_moe_gemm_8bit((act_fp8, act_scale), (weights["moe.experts.down_proj.weight"],
                           weights["moe.experts.down_proj.weight_scale_inv"]),
                           perm.sorted_expert_ids, down)                         # :638-643
    down = down[:nl]
    out["down"] = down
    unsorted = down[perm.inverse_order]                                          # :649
    full = torch.zeros(total * k, hsz, dtype=hidden.dtype)                       # :652
    full[perm.local_indices] = unsorted                                          # :653-654
    out["full"] = full
    if tp > 1 and all_reduce is not None:
        all_reduce(full)                                                         # :657
    output = (full.reshape(total, k, hsz) * topk_w.unsqueeze(-1)).sum(dim=1)     # :660-662
    out["routed"] = output
    if "moe.shared_expert.gate_proj.weight" in weights:                          # :665-673
        sg = fp8_linear(hidden, weights["moe.shared_expert.gate_proj.weight"],
                        weights["moe.shared_expert.gate_proj.weight_scale_inv"])
        su = fp8_linear(hidden, weights["moe.shared_expert.up_proj.weight"],
                        weights["moe.shared_expert.up_proj.weight_scale_inv"])
        so = F.silu(sg) * su
        sd = fp8_linear(so, weights["moe.shared_expert.down_proj.weight"],
                        weights["moe.shared_expert.down_proj.weight_scale_inv"])
        out["shared_down"] = sd
        if "moe.shared_expert_gate.weight" in weights:
            gv = torch.sigmoid(bf16_linear(hidden, weights["moe.shared_expert_gate.weight"]))
            out["shared_gate_val"] = gv
            sd = sd * gv
        output = output + sd
    out["output"] = output
    return out


def moe_forward(hidden: torch.Tensor, weights: dict, num_experts: int, k: int, **kw):
    """Output of ``qwen35_layer_v2.moe_forward`` (``:561-675``)."""
    return moe_forward_stages(hidden, weights, num_experts, k, **kw)["output"]


def moe_forward_tokens(hidden: torch.Tensor, weights: dict, topk_w: torch.Tensor,
                       topk_ids: torch.Tensor, expert_fn=None, shared_gate_logit: torch.Tensor | None = None,
                       combine: str = "v2"):
    """Per-token restatement of the same layer for large shapes, given the routing.

    Every output row depends only on its own token (activation scales are per row), so a
    sample of tokens can be checked at full size.  ``expert_fn(e)`` returns
    ``(w_gate_up [2I,H], s_gate_up, w_down [H,I], s_down)`` of routed expert ``e`` on the CPU
    (default: read from ``weights``), so only touched experts are ever dequantised.
    ``combine``: ``"v2"`` (``qwen35_layer_v2.py:660-662``), ``"dispatch"``
    (``moe_dispatch.py:75-77``, fp32 weights) or ``"batched"`` (``batched_moe.py:153-158``).
    Same arithmetic as :func:`moe_forward_stages` at TP=1.
    """
    t, hsz = hidden.shape
    k = topk_ids.shape[1]
    if expert_fn is None:
        w_gu, s_gu = fused_gate_up(weights)

        def expert_fn(e):
            return (w_gu[e], s_gu[e], weights["moe.experts.down_proj.weight"][e],
                    weights["moe.experts.down_proj.weight_scale_inv"][e])
    xq, xs = fast_fp8_quantize(hidden)
    xd = dequant_act(xq, xs)
    full = torch.zeros(t, k, hsz, dtype=torch.bfloat16)
    for e in torch.unique(topk_ids).tolist():
        tok, slot = (topk_ids == e).nonzero(as_tuple=True)
        wgu, sgu, wd, sd_ = expert_fn(e)
        inter = wgu.shape[0] // 2
        gu = (xd[tok] @ dequant_weight(wgu, sgu).t()).to(torch.bfloat16)
        a = F.silu(gu[:, :inter]) * gu[:, inter:]
        aq, as_ = fast_fp8_quantize(a)
        d = (dequant_act(aq, as_) @ dequant_weight(wd, sd_).t()).to(torch.bfloat16)
        full[tok, slot] = d
    if combine == "v2":
        output = (full * topk_w.unsqueeze(-1)).sum(dim=1)
    else:
        output = torch.zeros(t, hsz, dtype=torch.bfloat16)
        order = torch.argsort(topk_ids, dim=1, stable=True)
        for j in range(k):
            sel = order[:, j]
            d = full[torch.arange(t), sel]
            w = topk_w[torch.arange(t), sel].unsqueeze(-1)
            if combine == "dispatch":
                output = (output.float() + d.float() * w.float()).to(torch.bfloat16)
            else:
                output = output + d * w.to(torch.bfloat16)
    if "moe.shared_expert.gate_proj.weight" in weights:
        sg = fp8_linear(hidden, weights["moe.shared_expert.gate_proj.weight"],
                        weights["moe.shared_expert.gate_proj.weight_scale_inv"])
        su = fp8_linear(hidden, weights["moe.shared_expert.up_proj.weight"],
                        weights["moe.shared_expert.up_proj.weight_scale_inv"])
        sd = fp8_linear(F.silu(sg) * su, weights["moe.shared_expert.down_proj.weight"],
                        weights["moe.shared_expert.down_proj.weight_scale_inv"])
        if "moe.shared_expert_gate.weight" in weights or shared_gate_logit is not None:
            if shared_gate_logit is None:
                shared_gate_logit = bf16_linear(hidden, weights["moe.shared_expert_gate.weight"])
            sd = sd * torch.sigmoid(shared_gate_logit)
        output = output + sd
    return output


# ─────────────────────────────────────────────────────────────────────────────
# Synthetic weights (the reference has no public checkpoint here)
# ─────────────────────────────────────────────────────────────────────────────

def quantize_weight_blockwise(w: torch.Tensor):
    """128x128 block quantisation of an fp32 ``[N,K]`` weight: ``s = amax/448`` (the
    ``*_weight_scale_inv`` convention of ``loader.py:120-125``), ``q = clamp(w/s) -> e4m3``."""
    n, k = w.shape
    wb = w.view(n // BLOCK, BLOCK, k // BLOCK, BLOCK).float()
    s = wb.abs().amax(dim=(1, 3)).clamp(min=1e-12) / FP8_MAX
    q = (wb / s[:, None, :, None]).clamp(-FP8_MAX, FP8_MAX).to(FP8).view(n, k)
    return q, s.contiguous()


def make_layer_weights(hidden_size: int, num_experts: int, inter: int, shared_inter: int = 0,
                       shared_gate: bool = True, seed: int = 0, std: float = 0.02,
                       device="cpu", experts: range | None = None) -> dict:
    """Seeded synthetic MoE layer in the reference's weights-dict layout (``loader.py:212-264``).

    Draw order from one ``torch.Generator(device).manual_seed(seed)``: router gate
    ``[E,H]``; then per expert ``e``: gate ``[I,H]``, up ``[I,H]``, down ``[H,I]`` (fp32
    ``N(0,std)``, block-quantised); then shared gate/up/down; then ``shared_expert_gate [1,H]``.
    ``experts`` restricts which routed experts are stored (the draws for the others are still
    made so the stream stays aligned).
    """
    g = torch.Generator(device=device).manual_seed(seed)
    h, e_n, i_n = hidden_size, num_experts, inter

    def randn(*shape):
        return torch.randn(*shape, generator=g, device=device, dtype=torch.float32) * std

    w = {"moe.gate.weight": randn(e_n, h).to(torch.bfloat16)}
    keep = list(range(e_n)) if experts is None else list(experts)
    gq, gs, uq, us, dq, ds = [], [], [], [], [], []
    for e in range(e_n):
        gw, uw, dw = randn(i_n, h), randn(i_n, h), randn(h, i_n)
        if e in keep:
            for src, qs, ss in ((gw, gq, gs), (uw, uq, us), (dw, dq, ds)):
                q, s = quantize_weight_blockwise(src)
                qs.append(q)
                ss.append(s)
    w["moe.experts.gate_proj.weight"] = torch.stack(gq)
    w["moe.experts.gate_proj.weight_scale_inv"] = torch.stack(gs)
    w["moe.experts.up_proj.weight"] = torch.stack(uq)
    w["moe.experts.up_proj.weight_scale_inv"] = torch.stack(us)
    w["moe.experts.down_proj.weight"] = torch.stack(dq)
    w["moe.experts.down_proj.weight_scale_inv"] = torch.stack(ds)
    if shared_inter:
        for name, shape in (("gate_proj", (shared_inter, h)), ("up_proj", (shared_inter, h)),
                            ("down_proj", (h, shared_inter))):
            q, s = quantize_weight_blockwise(randn(*shape))
            w[f"moe.shared_expert.{name}.weight"] = q
            w[f"moe.shared_expert.{name}.weight_scale_inv"] = s
        if shared_gate:
            w["moe.shared_expert_gate.weight"] = randn(1, h).to(torch.bfloat16)
    return w


def make_hidden(tokens: int, hidden_size: int, seed: int, device="cpu") -> torch.Tensor:
    """``x ~ N(0,1)`` bf16 ``[T,H]`` from ``Generator(device).manual_seed(seed)``."""
    g = torch.Generator(device=device).manual_seed(seed)
    return torch.randn(tokens, hidden_size, generator=g, device=device).to(torch.bfloat16)


def zipf_bias(num_experts: int, s: float = 1.2, seed: int = 0) -> torch.Tensor:
    """Expert-popularity prior ``log p_{pi(e)}``, ``p_i ∝ i^-s`` over a seeded permutation."""
    g = torch.Generator().manual_seed(seed)
    ranks = torch.arange(1, num_experts + 1, dtype=torch.float64)
    p = ranks.pow(-s)
    p = p / p.sum()
    perm = torch.randperm(num_experts, generator=g)
    return p.log()[perm].float()


def decode_bytes(n_touched: int, hidden_size: int, inter: int, shared_inter: int,
                 num_experts: int, tokens: int) -> int:
    """Algorithmic HBM bytes of one decode layer: weights + scales of each touched expert and of
    the shared expert, the router gate, the shared-expert gate, and hidden in + out."""
    def expert_bytes(i_n):
        w = 3 * hidden_size * i_n
        s = ((2 * i_n // BLOCK) * (hidden_size // BLOCK) + (hidden_size // BLOCK) * (i_n // BLOCK)) * 4
        return w + s
    return (n_touched * expert_bytes(inter) + (expert_bytes(shared_inter) if shared_inter else 0)
            + num_experts * hidden_size * 2 + hidden_size * 2 + 2 * tokens * hidden_size * 2)


def prefill_flops(hidden_size: int, inter: int, shared_inter: int, tokens: int, k: int) -> int:
    """FP8 tensor FLOPs of one layer: ``6 H I`` per (token, expert) pair plus the shared expert."""
    return 6 * hidden_size * inter * tokens * k + 6 * hidden_size * shared_inter * tokens


def ceil_div(a: int, b: int) -> int:
    return -(-a // b)


__all__ = [n for n in dir() if not n.startswith("_") and n not in ("annotations", "math")]
