"""Host-side logic that needs no GPU: TP weight layouts and their equivalence on the oracle."""
import pytest
import torch

from conftest import assert_close_bf16
from muserve_b200 import loader
from oracle import moe_oracle as orc


@pytest.fixture(scope="module")
def layer():
    h, e, k, i = 256, 16, 4, 256
    w = orc.make_layer_weights(h, e, i, 256, seed=7)
    x = orc.make_hidden(24, h, 8)
    return w, x, e, k


def test_intermediate_sharding_slices(layer):
    w, _, e, _ = layer
    s = loader.shard_moe_weights(w, 2, 1, "inter")
    assert s["moe.layout"] == "inter"
    assert s["moe.experts.gate_proj.weight"].shape == (e, 128, 256)
    assert torch.equal(s["moe.experts.gate_proj.weight"].view(torch.uint8),
                       w["moe.experts.gate_proj.weight"][:, 128:].view(torch.uint8))
    assert torch.equal(s["moe.experts.down_proj.weight_scale_inv"], w["moe.experts.down_proj.weight_scale_inv"][:, :, 1:])
    assert s["moe.shared_expert.down_proj.weight"].shape == (256, 128)
    assert s["moe.gate.weight"] is w["moe.gate.weight"]


def test_intermediate_sharding_sums_to_full_layer(layer):
    """Sum over ranks of per-rank partial layers (router replicated, I sharded) equals the
    TP=1 layer up to bf16 rounding of the partial sums."""
    w, x, e, k = layer
    full = orc.moe_forward(x, w, e, k)
    parts = [orc.moe_forward(x, loader.shard_moe_weights(w, 2, r, "inter"), e, k) for r in range(2)]
    # the shared-expert gate multiplies each partial; sum in fp32 as an all-reduce would
    tot = (parts[0].float() + parts[1].float()).to(torch.bfloat16)
    assert_close_bf16(tot, full)


def test_expert_placement_slices(layer):
    w, _, e, _ = layer
    s = loader.shard_moe_weights(w, 4, 3, "expert")
    assert s["moe.experts.down_proj.weight"].shape[0] == e // 4
    assert torch.equal(s["moe.experts.up_proj.weight_scale_inv"][1], w["moe.experts.up_proj.weight_scale_inv"][7])


def test_fuse_gate_up_layout(layer):
    w, _, _, _ = layer
    f = loader.fuse_gate_up(w)
    assert f["moe.experts.gate_up_proj.weight"].shape[1] == 2 * w["moe.experts.gate_proj.weight"].shape[1]
    assert "moe.experts.gate_proj.weight" not in f


def test_stack_per_expert():
    w = {f"moe.expert_{e}.gate_proj.weight": torch.full((2, 3), float(e)) for e in range(3)}
    loader.stack_per_expert(w, 3)
    assert w["moe.experts.gate_proj.weight"].shape == (3, 2, 3)
    assert "moe.expert_0.gate_proj.weight" not in w
