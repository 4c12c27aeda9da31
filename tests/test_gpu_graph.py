"""CUDA-graph capture of a stack of MoE layers (muserve/model/graph_decode.py:23-113): the
replayed graph gives bit-identical results to the same step run eagerly, for the captured
input and for new inputs copied into the static buffer, and the self-feeding step chains."""
import pytest
import torch

from muserve_b200 import moe
from muserve_b200.graph import GraphedMoEStack
from oracle import moe_oracle as orc

pytestmark = pytest.mark.gpu


def _layers(cuda, n, h=512, e=32, inter=256, seed=50):
    out = []
    for i in range(n):
        w = orc.make_layer_weights(h, e, inter, inter, seed=seed + i)
        out.append({k: v.to(cuda) for k, v in w.items() if torch.is_tensor(v)})
    return out


def test_graph_replay_matches_eager(cuda):
    layers = _layers(cuda, 3)
    x0 = orc.make_hidden(16, 512, 60).to(cuda)
    g = GraphedMoEStack(layers, batch_size=16, top_k=4)
    g.capture(x0)
    want0 = g.eager(x0.clone())
    assert torch.equal(g.run(x0), want0)
    x1 = orc.make_hidden(16, 512, 61).to(cuda)
    want1 = g.eager(x1.clone())
    got1 = g.run(x1).clone()
    assert torch.equal(got1, want1)
    assert torch.equal(g.run(x1), got1)  # replays are deterministic
    moe.check_device_error()
    g.close()


def test_graph_self_feeding_steps(cuda):
    layers = _layers(cuda, 2, seed=70)
    x = orc.make_hidden(8, 512, 71).to(cuda)
    g = GraphedMoEStack(layers, batch_size=8, top_k=4, self_feed=True)
    g.capture(x)
    # capture() records without running, so the static input still holds x; each step() then
    # advances it
    ref = x.clone()
    g.inp.copy_(x)
    for _ in range(3):
        ref = g.eager(ref)
        out = g.step()
        assert torch.equal(out, ref)
        assert torch.equal(g.inp, ref)
    moe.check_device_error()
    g.close()


def test_graph_full_shape_decode(cuda):
    """One full-shape layer (H=4096, 512 experts top-10, I=1024 + shared) at 64 tokens."""
    from muserve_b200 import synthetic
    w = synthetic.make_layer_weights(4096, 512, 1024, 1024, seed=1, device=cuda)
    x = synthetic.make_hidden(64, 4096, seed=2, device=cuda)
    g = GraphedMoEStack([w], batch_size=64, top_k=10)
    g.capture(x)
    assert torch.equal(g.run(x), g.eager(x.clone()))
    moe.check_device_error()
    g.close()
    del w
    torch.cuda.empty_cache()
