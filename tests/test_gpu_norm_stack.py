"""The decode layer's MoE half around the path: the Gemma RMSNorm in front of the router
(qwen35_layer_v2.py:59-62 at :713-714) with the residual add fused in (:715), the router with
an additive logit prior (the 60-layer stack benchmark's Zipf popularity), and the graphed
stack of normed layers, all against the CPU oracle."""
import pytest
import torch

from conftest import assert_close_bf16
from muserve_b200 import moe
from muserve_b200.graph import GraphedMoEStack
from oracle import moe_oracle as orc

pytestmark = pytest.mark.gpu


def bf16_ulps(a, b):
    ia = a.cpu().contiguous().view(torch.int16).int()
    ib = b.cpu().contiguous().view(torch.int16).int()
    return (ia - ib).abs()


@pytest.mark.parametrize("T,H", [(1, 4096), (37, 4096), (128, 2048), (5, 136), (3, 16384), (300, 1024)])
@pytest.mark.parametrize("with_add", [False, True])
def test_add_rms_norm_matches_oracle(cuda, T, H, with_add):
    g = torch.Generator().manual_seed(T * 131 + H + with_add)
    h = (torch.randn(T, H, generator=g) * 3).to(torch.bfloat16)
    y = (torch.randn(T, H, generator=g)).to(torch.bfloat16) if with_add else None
    w = (torch.randn(H, generator=g) * 0.1).to(torch.bfloat16)
    hd = h.to(cuda)
    out = moe.add_rms_norm_gemma(hd, w.to(cuda), add=None if y is None else y.to(cuda))
    torch.cuda.synchronize()
    h_ref = h + y if with_add else h
    assert torch.equal(hd.cpu(), h_ref)  # the fused residual add is one bf16 rounding, bit-exact
    ref = orc.rms_norm_gemma(h_ref, w)
    d = bf16_ulps(out, ref)
    # the sum of squares runs in another order than on the host: rstd may move by an ulp
    assert d.max().item() <= 1
    assert (d == 0).float().mean().item() >= 0.99


def test_add_only(cuda):
    g = torch.Generator().manual_seed(3)
    h = torch.randn(17, 4096, generator=g).to(torch.bfloat16)
    y = torch.randn(17, 4096, generator=g).to(torch.bfloat16)
    hd = h.to(cuda)
    r = moe.add_rms_norm_gemma(hd, None, add=y.to(cuda), norm=False)
    assert r.data_ptr() == hd.data_ptr()
    assert torch.equal(hd.cpu(), h + y)


def test_v2_rms_norm_gemma_api(cuda):
    from muserve_b200.model import qwen35_layer_v2 as v2
    g = torch.Generator().manual_seed(4)
    x = torch.randn(2, 5, 4096, generator=g).to(torch.bfloat16)
    w = (torch.randn(4096, generator=g) * 0.1).to(torch.bfloat16)
    out = v2.rms_norm_gemma(x.to(cuda), w.to(cuda))
    assert out.shape == x.shape
    assert bf16_ulps(out, orc.rms_norm_gemma(x, w)).max().item() <= 1


@pytest.mark.parametrize("T,H,E,k", [(64, 4096, 512, 10), (128, 2048, 64, 8), (7, 1024, 128, 4)])
def test_router_logit_bias(cuda, T, H, E, k):
    g = torch.Generator().manual_seed(T + H + E)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    gw = (torch.randn(E, H, generator=g) * 0.02).to(torch.bfloat16)
    bias = orc.zipf_bias(E, 1.2, seed=E)
    w, ids, lg = moe.router_from_hidden(x.to(cuda), gw.to(cuda), k, logit_bias=bias.to(cuda), return_logits=True)
    torch.cuda.synchronize()
    logits = lg.cpu()
    # the returned logits exclude the prior and are the bf16 GEMM output
    assert torch.equal(logits, logits.to(torch.bfloat16).float())
    ref_w, ref_ids = orc.route_biased(logits, bias, k)
    assert torch.equal(ids.cpu().long(), ref_ids)
    assert bf16_ulps(w, ref_w).max().item() <= 1
    # the prior moves the routing toward the popular experts
    w0, ids0 = moe.router_from_hidden(x.to(cuda), gw.to(cuda), k)
    assert not torch.equal(ids0.cpu(), ids.cpu())


def _normed_layers(cuda, n, h=512, e=32, inter=256, seed=80):
    out = []
    for i in range(n):
        w = orc.make_layer_weights(h, e, inter, inter, seed=seed + i)
        g = torch.Generator().manual_seed(seed + 100 + i)
        w["post_attention_layernorm.weight"] = (torch.randn(h, generator=g) * 0.1).to(torch.bfloat16)
        out.append({kk: v.to(cuda) for kk, v in w.items() if torch.is_tensor(v)})
    return out


def test_normed_stack_matches_oracle_and_graph(cuda):
    n, T, E, k = 3, 16, 32, 4
    layers = _normed_layers(cuda, n)
    biases = [orc.zipf_bias(E, 1.2, seed=90 + i).to(cuda) for i in range(n)]
    x0 = orc.make_hidden(T, 512, 91).to(cuda)
    stack = GraphedMoEStack(layers, batch_size=T, top_k=k, norm=True, logit_biases=biases)
    got = stack.eager(x0)
    # the fused add + next norm equals one layer at a time
    h = x0
    for i in range(n):
        one = GraphedMoEStack([layers[i]], batch_size=T, top_k=k, norm=True, logit_biases=[biases[i]])
        h_next = one.eager(h)
        cpu_w = {kk: v.cpu() for kk, v in layers[i].items()}
        ref = orc.moe_block(h.cpu(), cpu_w, E, k, logit_bias=biases[i].cpu())
        assert_close_bf16(h_next.cpu().float(), ref.float())
        h = h_next
    assert torch.equal(got, h)
    # graph replay is bit-identical to the eager step
    stack.capture(x0)
    assert torch.equal(stack.run(x0), got)
    moe.check_device_error()
    stack.close()
