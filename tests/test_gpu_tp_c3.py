"""Tensor parallelism at BASELINE config 3's shapes on one GPU: H=4096, 512 experts top-10 + the
shared expert, I=1024, 256 tokens.  Every rank's partial layer is computed with that rank's
weight shard (muserve_b200.loader.shard_moe_weights) and the partials are summed, as the
all-reduce of muserve/distributed.py:62-64 would, then compared with the unsharded oracle on
all 256 tokens.

Mode "inter" (the benchmark's layout) at TP 2, 4 and 8 runs I/TP = 512, 256 and 128 per rank:
I/TP = 128 (TP 8) takes the weights-on-M down GEMM and the 2-accumulator gate_up variant with
a single 128-channel block, the kernels the 8-GPU benchmark runs.  Mode "expert" (the
reference's own e % tp == rank placement, loader.py:230-264) runs at TP 8, with rank 0 adding
the shared expert.  The partials are summed in fp32 and rounded once (what the fused
all-reduce computes); they differ from the unsharded layer by bf16 rounding of each partial.
Tolerance: bf16 max-abs-rel <= 2e-2 and cosine >= 0.9999."""
import pytest
import torch

from conftest import assert_close_bf16
from muserve_b200 import moe, synthetic
from muserve_b200.loader import shard_moe_weights
from oracle import moe_oracle as orc

pytestmark = pytest.mark.gpu

H, E, K, INTER, T = 4096, 512, 10, 1024, 256


@pytest.fixture(scope="module")
def c3(cuda):
    w = synthetic.make_layer_weights(H, E, INTER, INTER, seed=1, device=cuda)
    x = synthetic.make_hidden(T, H, seed=2, device=cuda)
    logits = synthetic.uniform_logits(T, E, seed=3, device=cuda)
    tw, tid = moe.route_topk(logits, K, ids_dtype=torch.int32)

    def fetch(e):
        gu = torch.cat([w["moe.experts.gate_proj.weight"][e], w["moe.experts.up_proj.weight"][e]], 0).cpu()
        gs = torch.cat([w["moe.experts.gate_proj.weight_scale_inv"][e],
                        w["moe.experts.up_proj.weight_scale_inv"][e]], 0).cpu()
        return gu, gs, w["moe.experts.down_proj.weight"][e].cpu(), w["moe.experts.down_proj.weight_scale_inv"][e].cpu()
    shared = {k: v.cpu() for k, v in w.items() if k.startswith("moe.shared")}
    ref = orc.moe_forward_tokens(x.cpu(), shared, tw.cpu(), tid.cpu().long(), expert_fn=fetch)
    yield w, x, logits, ref
    del w
    torch.cuda.empty_cache()


@pytest.mark.parametrize("tp", [2, 4, 8])
def test_c3_inter_sharded(c3, tp):
    w, x, logits, ref = c3
    total = torch.zeros(T, H, dtype=torch.float32, device=x.device)
    for rank in range(tp):
        wr = {k: v for k, v in shard_moe_weights(w, tp, rank, "inter").items() if torch.is_tensor(v)}
        assert wr["moe.experts.gate_proj.weight"].shape[1] == INTER // tp
        total += moe.moe_layer(x, wr, top_k=K, num_experts=E, router_logits=logits).float()
        del wr
    moe.check_device_error()
    assert_close_bf16(total.to(torch.bfloat16), ref)


def test_c3_expert_placed_tp8(c3):
    w, x, logits, ref = c3
    tp = 8
    total = torch.zeros(T, H, dtype=torch.float32, device=x.device)
    for rank in range(tp):
        wr = {k: v for k, v in shard_moe_weights(w, tp, rank, "expert").items() if torch.is_tensor(v)}
        total += moe.moe_layer(x, wr, top_k=K, num_experts=E, router_logits=logits, placement=1, tp=tp, rank=rank,
                               add_shared=(rank == 0)).float()
        del wr
    moe.check_device_error()
    assert_close_bf16(total.to(torch.bfloat16), ref)
