"""Router from the hidden states on the tensor cores (qwen35_layer_v2.py:567-572,
kernels/moe_dispatch.py:8-24): the logits against an fp64 product of the same bf16 inputs, the
bf16-rounded logits against that product rounded to bf16, and the routing against the oracle on
the kernel's own logits (ids identical, weights within 1 bf16 ulp; the reference's bar for the
router).  Shapes cover the split-K path (small T), the unsplit path (T = 8192), partial token and
expert tiles, and E not a multiple of 32."""
import pytest
import torch

from muserve_b200 import moe
from muserve_b200.kernels.moe_dispatch import moe_gate
from oracle import moe_oracle as orc

pytestmark = pytest.mark.gpu

SHAPES = [(1, 512, 64, 4), (64, 4096, 512, 10), (300, 2048, 64, 8), (129, 1024, 48, 6), (8192, 4096, 512, 10)]


def _inputs(t, h, e, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(t, h, generator=g).to(torch.bfloat16)
    w = (torch.randn(e, h, generator=g) * 0.02).to(torch.bfloat16)
    return x, w


@pytest.mark.parametrize("t,h,e,k", SHAPES)
def test_router_logits_and_routing(cuda, t, h, e, k):
    x, w = _inputs(t, h, e, 100 + t)
    xd, wd = x.to(cuda), w.to(cuda)
    ref = x.double() @ w.double().t()
    bound = x.double().abs() @ w.double().abs().t()
    # fp32 logits (moe_gate): within fp32 accumulation error of the exact product
    w32, ids32, lg32 = moe.router_from_hidden(xd, wd, k, round_logits_bf16=False, w_dtype=torch.float32,
                                              return_logits=True)
    assert ((lg32.cpu().double() - ref).abs() <= 2e-6 * bound + 1e-30).all()
    # bf16-rounded logits (v2): exactly the bf16 rounding of the fp32 logits, so within bf16's
    # unit roundoff (2^-8) plus the fp32 sum's error of the exact product
    wb, idsb, lgb = moe.router_from_hidden(xd, wd, k, return_logits=True)
    assert torch.equal(lgb.cpu(), lg32.cpu().to(torch.bfloat16).float())
    b = lgb.cpu().double()
    assert ((b - ref).abs() <= 2.0 ** -8 * b.abs() + 2e-6 * bound + 1e-30).all()
    # routing on the kernel's own logits, as the oracle computes it
    rw, rid = orc.route(lgb.cpu(), k)
    assert torch.equal(idsb.cpu().long(), rid)
    assert (wb.cpu().view(torch.int16).int() - rw.view(torch.int16).int()).abs().max() <= 1
    rw32, rid32 = orc.route(lg32.cpu(), k, weight_dtype=torch.float32)
    assert torch.equal(ids32.cpu().long(), rid32)
    assert torch.allclose(w32.cpu(), rw32, rtol=1e-6, atol=1e-7)
    # deterministic (fixed split order)
    wb2, idsb2 = moe.router_from_hidden(xd, wd, k)
    assert torch.equal(wb2, wb) and torch.equal(idsb2, idsb)
    moe.check_device_error()


def test_moe_gate_uses_fp32_logits(cuda):
    x, w = _inputs(64, 2048, 64, 7)
    ids, tw = moe_gate(x.to(cuda), w.to(cuda), top_k=8)
    assert ids.dtype == torch.int32 and tw.dtype == torch.float32
    logits = (x.float() @ w.float().t())
    rw, rid = orc.route(logits, 8, weight_dtype=torch.float32)
    same = (ids.cpu().long() == rid).all(-1)
    assert same.float().mean() >= 0.95  # fp32 sums in another order may swap near-tied experts
    assert torch.allclose(tw.cpu()[same], rw[same], rtol=1e-5, atol=1e-6)
