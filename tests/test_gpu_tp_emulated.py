"""Tensor parallelism on one GPU: every rank's partial layer computed with that rank's weight
shard (muserve_b200.loader.shard_moe_weights) and summed on the host, as the NCCL all-reduce
would (muserve/distributed.py:62-64), against the unsharded oracle.

Mode "inter": the expert intermediate split into TP column/row shards (loader.py:52-61),
every rank routes all tokens.  Mode "expert": whole experts placed e % tp == rank
(loader.py:232), each rank computes its local experts (placement=1) and rank 0 adds the shared
expert.  Sums of bf16 partials differ from the single-GPU layer by bf16 rounding only.
Tolerance: bf16 max-abs-rel <= 2e-2 and cosine >= 0.9999."""
import pytest
import torch

from conftest import assert_close_bf16
from muserve_b200 import moe
from muserve_b200.loader import shard_moe_weights
from oracle import moe_oracle as orc

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("tp", [2, 4])
@pytest.mark.parametrize("tokens", [24, 600])
def test_inter_sharded_partials_sum_to_the_layer(cuda, tp, tokens):
    h, e, k, inter = 512, 32, 4, 512
    w = orc.make_layer_weights(h, e, inter, inter, seed=21)
    x = orc.make_hidden(tokens, h, 22)
    logits = torch.nn.functional.linear(x, w["moe.gate.weight"]).float()
    ref = orc.moe_forward(x, w, e, k, logits=logits)
    total = torch.zeros(tokens, h, dtype=torch.float32)
    for rank in range(tp):
        wr = {kk: v.to(cuda) for kk, v in shard_moe_weights(w, tp, rank, "inter").items() if torch.is_tensor(v)}
        part = moe.moe_layer(x.to(cuda), wr, top_k=k, num_experts=e, router_logits=logits.to(cuda))
        total += part.float().cpu()
    moe.check_device_error()
    assert_close_bf16(total.to(torch.bfloat16), ref)


@pytest.mark.parametrize("tp", [2, 4])
def test_expert_placed_partials_sum_to_the_layer(cuda, tp):
    h, e, k, inter, tokens = 512, 32, 4, 256, 40
    w = orc.make_layer_weights(h, e, inter, inter, seed=23)
    x = orc.make_hidden(tokens, h, 24)
    logits = torch.nn.functional.linear(x, w["moe.gate.weight"]).float()
    ref = orc.moe_forward(x, w, e, k, logits=logits)
    total = torch.zeros(tokens, h, dtype=torch.float32)
    for rank in range(tp):
        wr = {kk: (v.to(cuda) if torch.is_tensor(v) else v) for kk, v in shard_moe_weights(w, tp, rank, "expert").items()}
        part = moe.moe_layer(x.to(cuda), {kk: v for kk, v in wr.items() if torch.is_tensor(v)}, top_k=k,
                             num_experts=e, router_logits=logits.to(cuda), placement=1, tp=tp, rank=rank,
                             add_shared=(rank == 0))
        total += part.float().cpu()
    moe.check_device_error()
    assert_close_bf16(total.to(torch.bfloat16), ref)
