"""HF checkpoint loader (muserve/loader.py:87-264): a small synthetic FP8 checkpoint written as
safetensors shards with an index, read back in both TP layouts and compared with the
in-memory layouts of the same weights (loader.shard_moe_weights, loader.fuse_gate_up)."""
import json
import os

import pytest
import torch

from muserve_b200 import checkpoint, loader
from oracle import moe_oracle as orc

safetensors = pytest.importorskip("safetensors.torch")

H, E, INTER, LAYER = 256, 8, 256, 3


def _bf16_scales(w: dict) -> dict:
    """The checkpoint stores scales in bf16; the loader widens them to fp32 exactly."""
    return {k: (v.to(torch.bfloat16).float() if k.endswith("scale_inv") else v) for k, v in w.items()}


@pytest.fixture(scope="module")
def ckpt(tmp_path_factory):
    ref = _bf16_scales(orc.make_layer_weights(H, E, INTER, INTER, seed=41))
    p = checkpoint.layer_prefix(LAYER)
    hf = {p + "mlp.gate.weight": ref["moe.gate.weight"],
          p + "mlp.shared_expert_gate.weight": ref["moe.shared_expert_gate.weight"],
          "model.language_model.layers.0.input_layernorm.weight": torch.ones(H, dtype=torch.bfloat16)}
    for proj in ("gate_proj", "up_proj", "down_proj"):
        hf[p + f"mlp.shared_expert.{proj}.weight"] = ref[f"moe.shared_expert.{proj}.weight"]
        hf[p + f"mlp.shared_expert.{proj}.weight_scale_inv"] = ref[f"moe.shared_expert.{proj}.weight_scale_inv"].to(torch.bfloat16)
        for e in range(E):
            hf[p + f"mlp.experts.{e}.{proj}.weight"] = ref[f"moe.experts.{proj}.weight"][e].contiguous()
            hf[p + f"mlp.experts.{e}.{proj}.weight_scale_inv"] = \
                ref[f"moe.experts.{proj}.weight_scale_inv"][e].to(torch.bfloat16).contiguous()
    d = tmp_path_factory.mktemp("ckpt")
    names = sorted(hf)
    shards = {"model-00001-of-00002.safetensors": names[::2], "model-00002-of-00002.safetensors": names[1::2]}
    wmap = {}
    for fn, keys in shards.items():
        safetensors.save_file({k: hf[k] for k in keys}, os.path.join(d, fn))
        wmap.update({k: fn for k in keys})
    with open(os.path.join(d, "model.safetensors.index.json"), "w") as f:
        json.dump({"metadata": {}, "weight_map": wmap}, f)
    return str(d), ref


def _same(a: dict, b: dict):
    ka = {k for k, v in a.items() if torch.is_tensor(v)}
    kb = {k for k, v in b.items() if torch.is_tensor(v)}
    assert ka == kb
    for k in ka:
        assert a[k].dtype == b[k].dtype and a[k].shape == b[k].shape, k
        if a[k].dtype == torch.float8_e4m3fn:
            assert torch.equal(a[k].view(torch.uint8), b[k].view(torch.uint8)), k
        else:
            assert torch.equal(a[k], b[k]), k
        assert a[k].is_contiguous(), k


@pytest.mark.parametrize("tp,rank", [(1, 0), (2, 1), (4, 2)])
def test_expert_layout(ckpt, tp, rank):
    path, ref = ckpt
    got = checkpoint.load_moe_layer(path, LAYER, tp=tp, rank=rank, layout="expert")
    want = loader.fuse_gate_up(loader.shard_moe_weights(ref, tp, rank, "expert"))
    _same(got, want)
    assert got["moe.layout"] == "expert"
    assert got["moe.experts.gate_up_proj.weight_scale_inv"].dtype == torch.float32


@pytest.mark.parametrize("tp,rank", [(2, 0), (2, 1)])
def test_inter_layout(ckpt, tp, rank):
    path, ref = ckpt
    got = checkpoint.load_moe_layer(path, LAYER, tp=tp, rank=rank, layout="inter")
    want = loader.fuse_gate_up(loader.shard_moe_weights(ref, tp, rank, "inter"))
    _same(got, want)


def test_unfused(ckpt):
    path, ref = ckpt
    got = checkpoint.load_moe_layer(path, LAYER, fuse_gate_up=False)
    _same(got, loader.shard_moe_weights(ref, 1, 0, "expert"))


def test_errors(ckpt):
    path, _ = ckpt
    with pytest.raises(KeyError):
        checkpoint.load_moe_layer(path, LAYER + 1)
    with pytest.raises(ValueError):
        checkpoint.load_moe_layer(path, LAYER, tp=4, rank=0, layout="inter")  # 256 / 4 is not whole 128-blocks
    with pytest.raises(ValueError):
        checkpoint.load_moe_layer(path, LAYER, tp=3, rank=0, layout="expert")
    idx = checkpoint.load_index(path)
    idx.pop(checkpoint.layer_prefix(LAYER) + "mlp.experts.5.down_proj.weight")
    with pytest.raises(KeyError):
        checkpoint.load_moe_layer(path, LAYER, weight_index=idx)
