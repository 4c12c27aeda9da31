"""The CPU oracle reproduces the reference's own moe_forward (golden fixtures made by
tests/golden/make_golden.py from the reference run on CPU)."""
import hashlib

import pytest
import torch

from conftest import load_golden
from oracle import moe_oracle as orc


def sha(t):
    t = t.contiguous()
    t = t.view(torch.uint8) if t.dtype == torch.float8_e4m3fn else (t.view(torch.int16) if t.dtype == torch.bfloat16 else t)
    return hashlib.sha256(t.numpy().tobytes()).hexdigest()


def run_oracle(g, logits=None):
    c = g["cfg"]
    w = orc.make_layer_weights(c["hidden"], c["experts"], c["inter"], c["shared"], seed=c["wseed"])
    x = orc.make_hidden(c["tokens"], c["hidden"], c["xseed"])
    assert sha(x) == g["hidden_sha"], "seeded input generation changed"
    return orc.moe_forward_stages(x, w, c["experts"], c["k"], logits=logits), w, x


@pytest.mark.parametrize("case", ["c0", "small"])
def test_oracle_matches_reference_layer(case):
    g = load_golden(case)
    st, _, _ = run_oracle(g)
    assert torch.equal(st["topk_ids"], g["topk_ids"])
    assert torch.equal(st["topk_w"], g["topk_w"])
    assert torch.equal(st["perm"].sort_order, g["sort_order"])
    assert torch.equal(st["perm"].inverse_order, g["inverse_order"])
    assert torch.equal(st["perm"].sorted_expert_ids, g["sorted_expert_ids"])
    assert torch.equal(st["x_scale"], g["x_scale"])
    assert torch.equal(st["act_scale"], g["act_scale"])
    assert sha(st["x_fp8"]) == g["x_fp8_sha"]
    assert sha(st["act_fp8"]) == g["act_fp8_sha"]
    nl = st["perm"].num_local
    mp = st["perm"].padded_m
    gu = torch.zeros(mp, st["gate_up"].shape[1], dtype=torch.bfloat16)
    # the reference's buffers hold padding rows written by the GEMM: compare the valid rows
    if "gate_up" in g:
        assert torch.equal(st["gate_up"], g["gate_up"][:nl])
        assert torch.equal(st["down"], g["down"][:nl])
    else:
        assert torch.equal(st["gate_up"][:4], g["gate_up_rows"])
        assert torch.equal(st["down"][:4], g["down_rows"])
    assert torch.equal(st["output"], g["output"])
    if "shared_down" in g:
        assert torch.equal(st["shared_down"], g["shared_down"])
    del gu


@pytest.mark.parametrize("case", ["route_unif", "route_bf16"])
def test_oracle_routing_full_shape(case):
    g = load_golden(case)
    w, ids = orc.route(g["logits"], g["cfg"]["k"])
    assert torch.equal(ids, g["topk_ids"]) and torch.equal(w, g["topk_w"])
    p = orc.permute(ids, g["cfg"]["experts"])
    assert torch.equal(p.sort_order, g["sort_order"])
    assert torch.equal(p.inverse_order, g["inverse_order"])
    assert torch.equal(p.sorted_expert_ids, g["sorted_expert_ids"])


def test_oracle_tp2_expert_placement_matches_reference():
    """V2 at TP=2 (experts e % 2 == rank, [T*k,H] all-reduce, then combine) reproduced by the
    oracle with the all-reduce done in process (each slot is produced by exactly one rank, so
    the bf16 sum adds one nonzero and is exact)."""
    g = load_golden("c0_tp2")
    c = g["cfg"]
    w = orc.make_layer_weights(c["hidden"], c["experts"], c["inter"], c["shared"], seed=c["wseed"])
    x = orc.make_hidden(c["tokens"], c["hidden"], c["xseed"])
    fulls = []
    for r in range(2):
        wl = {k: (v[r::2].contiguous() if k.startswith("moe.experts.") else v) for k, v in w.items()}
        st = orc.moe_forward_stages(x, wl, c["experts"], c["k"], tp=2, rank=r)
        fulls.append(st["full"])
        assert torch.equal(st["perm"].sort_order, g["sort_order"][r])
        assert torch.equal(st["perm"].sorted_expert_ids, g["sorted_expert_ids"][r])
    total = fulls[0] + fulls[1]
    routed = (total.reshape(c["tokens"], c["k"], -1) * st["topk_w"].unsqueeze(-1)).sum(1)
    out = routed + st["shared_down"] * st["shared_gate_val"]
    assert torch.equal(out, g["output"])


def test_per_token_oracle_equals_staged_oracle():
    g = load_golden("c0")
    st, w, x = run_oracle(g)
    out = orc.moe_forward_tokens(x, w, st["topk_w"], st["topk_ids"])
    assert torch.equal(out, st["output"])


def test_rms_norm_gemma_oracle_is_one_rounding():
    """The oracle's rms_norm_gemma (qwen35_layer_v2.py:59-62, torch's rms_norm on bf16 input)
    equals an independent numpy restatement: w = bf16(1 + weight), x * (1/sqrt(mean(x^2) + eps))
    * w in fp32, rounded to bf16 once.  The GPU kernel is tested against this oracle."""
    import numpy as np
    from oracle import moe_oracle as orc
    g = torch.Generator().manual_seed(21)
    x = (torch.randn(16, 2048, generator=g) * 3).to(torch.bfloat16)
    w = (torch.randn(2048, generator=g) * 0.1).to(torch.bfloat16)
    out = orc.rms_norm_gemma(x, w)
    xf = x.float().numpy()
    weff = (1.0 + w.float()).to(torch.bfloat16).float().numpy()
    ms = (xf.astype(np.float64) ** 2).mean(axis=1, keepdims=True)
    rstd = (np.float32(1.0) / np.sqrt(ms.astype(np.float32) + np.float32(1e-6))).astype(np.float32)
    ref = torch.from_numpy((xf * rstd * weff).astype(np.float32)).to(torch.bfloat16)
    d = (out.view(torch.int16).int() - ref.view(torch.int16).int()).abs()
    # the mean of squares is summed in another order here (float64): rstd may move by an ulp
    assert d.max().item() <= 1 and (d == 0).float().mean().item() >= 0.99


def test_route_biased_oracle():
    """The stack benchmark's prior is a plain fp32 add before the reference's routing."""
    from oracle import moe_oracle as orc
    g = torch.Generator().manual_seed(22)
    lg = torch.randn(8, 64, generator=g)
    b = orc.zipf_bias(64, 1.2, seed=3)
    w1, i1 = orc.route_biased(lg, b, 6)
    w2, i2 = orc.route(lg + b, 6)
    assert torch.equal(i1, i2) and torch.equal(w1, w2)
    # a Zipf prior concentrates routing on the popular experts
    _, ib = orc.route(torch.randn(4096, 64, generator=g) + b, 6)
    top = torch.argsort(b, descending=True)[:6]
    assert torch.isin(ib, top).float().mean() > 0.3
