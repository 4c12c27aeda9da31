"""Router kernel: ids bit-exact with torch's CPU top-k (the reference's own op), weights
within one bf16 ulp.  qwen35_layer_v2.py:569-572, moe_dispatch.py:20-24."""
import pytest
import torch

from conftest import load_golden
from muserve_b200 import moe
from oracle.ctopk import topk_torch_cpu_order

pytestmark = pytest.mark.gpu


def bf16_ulp_diff(a, b):
    return (a.cpu().view(torch.int16).int() - b.cpu().view(torch.int16).int()).abs().max().item()


def score_collision_rows(logits):
    """Rows where two distinct logits give equal fp32 softmax scores on the CPU (the only case
    where selecting on logits can differ from torch selecting on scores)."""
    s = torch.softmax(logits, -1)
    rows = []
    for t in range(logits.shape[0]):
        ss, order = torch.sort(s[t])
        ls = logits[t][order]
        if ((ss[1:] == ss[:-1]) & (ls[1:] != ls[:-1])).any():
            rows.append(t)
    return rows


@pytest.mark.parametrize("case", ["route_unif", "route_bf16"])
def test_router_matches_reference_golden(cuda, case):
    g = load_golden(case)
    k = g["cfg"]["k"]
    w, ids = moe.route_topk(g["logits"].to(cuda), k)
    torch.cuda.synchronize()
    bad = set(score_collision_rows(g["logits"]))
    good = [t for t in range(ids.shape[0]) if t not in bad]
    assert torch.equal(ids.cpu()[good], g["topk_ids"][good])
    assert bf16_ulp_diff(w[good], g["topk_w"][good]) <= 1


@pytest.mark.parametrize("E,k", [(512, 10), (64, 8), (512, 8), (1024, 16), (128, 1), (8, 8), (256, 4)])
@pytest.mark.parametrize("T", [1, 37, 2048])
def test_router_tie_heavy_bf16_logits(cuda, E, k, T):
    g = torch.Generator().manual_seed(E + 31 * k + T)
    x = (torch.randn(T, E, generator=g) * 1.28).to(torch.bfloat16).float()
    w, ids = moe.route_topk(x.to(cuda), k, w_dtype=torch.float32)
    ref_w, ref_ids = torch.topk(torch.softmax(x, -1), k, -1)
    ref_w = ref_w / ref_w.sum(-1, keepdim=True)
    assert torch.equal(ids.cpu(), ref_ids)
    torch.testing.assert_close(w.cpu(), ref_w, rtol=2e-6, atol=1e-7)


@pytest.mark.parametrize("E,k", [(512, 10), (256, 8), (64, 6), (16, 16)])
def test_router_fp32_rows_with_planted_ties(cuda, E, k):
    """fp32 logits: distinct rows take the register fast path, rows with a tie among the k+1
    largest (signed zeros included) fall back to the replay; both must match torch."""
    g = torch.Generator().manual_seed(E * 7 + k)
    T = 64
    x = torch.randn(T, E, generator=g)
    for t in range(T):
        order = torch.argsort(x[t], descending=True)
        kind = t % 5
        if kind == 1:  # the two largest are +0 and -0
            x[t] = -x[t].abs() - 0.1
            x[t, order[3]] = 0.0
            x[t, order[E // 2]] = -0.0
        elif kind == 2 and k < E:  # tie between ranks k-1 and k
            x[t, order[k]] = x[t, order[k - 1]]
        elif kind == 3:  # tie at the top
            x[t, order[1]] = x[t, order[0]]
        elif kind == 4 and k + 1 < E:  # tie just below the selection
            x[t, order[k + 1]] = x[t, order[k]]
    w, ids = moe.route_topk(x.to(cuda), k, w_dtype=torch.float32)
    ref_w, ref_ids = torch.topk(torch.softmax(x, -1), k, -1)
    ref_w = ref_w / ref_w.sum(-1, keepdim=True)
    assert torch.equal(ids.cpu(), ref_ids)
    torch.testing.assert_close(w.cpu(), ref_w, rtol=2e-6, atol=1e-7)


def test_topk_select_on_cpu_scores_is_exact(cuda):
    """Given the very same fp32 scores, the ids equal torch.topk's, whatever the ties."""
    g = torch.Generator().manual_seed(5)
    s = torch.softmax(torch.rand(4096, 512, generator=g), -1)
    s[::9, 100:110] = s[::9, 3:4]  # planted exact ties
    v, ids = moe.topk_select(s.to(cuda), 10)
    rv, rids = torch.topk(s, 10, -1)
    assert torch.equal(ids.cpu(), rids) and torch.equal(v.cpu(), rv)


def test_router_nan_and_inf_rows(cuda):
    x = torch.randn(6, 64)
    x[1, 7] = float("nan")
    x[3, 2] = float("inf")
    x[4] = 0.0
    _, ids = moe.route_topk(x.to(cuda), 8, w_dtype=torch.float32)
    _, rids = torch.topk(torch.softmax(x, -1), 8, -1)
    assert torch.equal(ids.cpu(), rids)


def test_moe_gate_api(cuda):
    from muserve_b200.kernels.moe_dispatch import moe_gate
    from oracle import moe_oracle as orc
    g = torch.Generator().manual_seed(9)
    h = torch.randn(33, 512, generator=g).to(torch.bfloat16)
    gw = (torch.randn(64, 512, generator=g) * 0.02).to(torch.bfloat16)
    ids, w = moe_gate(h.to(cuda), gw.to(cuda), top_k=6)
    rids, rw = orc.moe_gate(h, gw, 6)
    assert ids.dtype == torch.int32 and w.dtype == torch.float32
    # fp32 logits from two GEMM implementations may differ in the last bits: compare where the
    # CPU logits order is unambiguous
    assert (ids.cpu() == rids).float().mean() > 0.99
    torch.testing.assert_close(w.cpu()[(ids.cpu() == rids).all(-1)], rw[(ids.cpu() == rids).all(-1)],
                               rtol=1e-4, atol=1e-6)
