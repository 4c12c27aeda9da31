"""Large-batch data path: above 8192 routed rows the layer counts rows in many blocks
(multi-block dispatch), quantises each token once and gathers its e4m3 rows into expert order.
Checked on every token against the CPU oracle, with and without the shared expert and in the
three combine orders (qwen35_layer_v2.py:660-662, moe_dispatch.py:75-77,
batched_moe.py:153-158).  Tolerance: bf16 max-abs-rel <= 2e-2 and cosine >= 0.9999."""
import pytest
import torch

from conftest import assert_close_bf16
from muserve_b200 import _lib, moe
from oracle import moe_oracle as orc

pytestmark = pytest.mark.gpu

H, E, K, INTER, TOKENS = 512, 64, 8, 512, 1100  # 8800 routed rows


@pytest.fixture(scope="module")
def layer(cuda):
    w = orc.make_layer_weights(H, E, INTER, INTER, seed=31)
    x = orc.make_hidden(TOKENS, H, 32)
    logits = torch.nn.functional.linear(x, w["moe.gate.weight"]).float()
    wd = {k: v.to(cuda) for k, v in w.items() if torch.is_tensor(v)}
    return w, x, logits, wd


@pytest.mark.parametrize("combine,mode,wdt", [("v2", _lib.COMBINE_V2, torch.bfloat16),
                                              ("dispatch", _lib.COMBINE_DISPATCH, torch.float32),
                                              ("batched", _lib.COMBINE_BATCHED, torch.bfloat16)])
def test_gather_path_all_tokens(cuda, layer, combine, mode, wdt):
    w, x, logits, wd = layer
    out, tw, tid = moe.moe_layer(x.to(cuda), wd, top_k=K, num_experts=E, router_logits=logits.to(cuda),
                                 combine_mode=mode, weights_dtype=wdt, return_routing=True)
    rw, rid = orc.route(logits, K)
    assert torch.equal(tid.cpu().long(), rid)
    ref = orc.moe_forward_tokens(x, w, tw.cpu(), tid.cpu().long(), combine=combine)
    assert_close_bf16(out.cpu(), ref)
    moe.check_device_error()


def test_gather_path_routed_only(cuda, layer):
    w, x, logits, wd = layer
    routed = {k: v for k, v in wd.items() if not k.startswith("moe.shared")}
    out, tw, tid = moe.moe_layer(x.to(cuda), routed, top_k=K, num_experts=E, router_logits=logits.to(cuda),
                                 return_routing=True)
    ref = orc.moe_forward_tokens(x, {k: v for k, v in w.items() if not k.startswith("moe.shared")}, tw.cpu(),
                                 tid.cpu().long())
    assert_close_bf16(out.cpu(), ref)
    moe.check_device_error()


def test_gather_path_matches_per_row_quantisation(cuda, layer):
    """The same 1100 tokens split in two calls of 550 (4400 rows each, per-row quantisation)
    give bit-identical outputs: quantising a token once and gathering equals quantising each
    of its rows."""
    w, x, logits, wd = layer
    xd, ld = x.to(cuda), logits.to(cuda)
    big = moe.moe_layer(xd, wd, top_k=K, num_experts=E, router_logits=ld)
    halves = [moe.moe_layer(xd[i:i + 550].contiguous(), wd, top_k=K, num_experts=E,
                            router_logits=ld[i:i + 550].contiguous()) for i in (0, 550)]
    assert torch.equal(big, torch.cat(halves))
    moe.check_device_error()
