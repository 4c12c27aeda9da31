"""Dispatch bookkeeping bit-exact with the reference (qwen35_layer_v2.py:574-605)."""
import pytest
import torch

from conftest import load_golden
from muserve_b200 import moe
from oracle import moe_oracle as orc

pytestmark = pytest.mark.gpu


def check(ids, E, tp=1, rank=0, dev=None):
    so, io, se, cnt, nl = moe.permute(ids.to(dev), E, tp=tp, rank=rank)
    ref = orc.permute(ids.cpu().long(), E, tp, rank)
    n = int(nl.item())
    assert n == ref.num_local
    assert torch.equal(so.cpu()[:n], ref.sort_order)
    assert torch.equal(io.cpu()[:n], ref.inverse_order)
    assert torch.equal(se.cpu()[:ref.padded_m], ref.sorted_expert_ids)
    assert torch.equal(cnt.cpu().long(), ref.expert_counts)


@pytest.mark.parametrize("case", ["c0", "route_unif", "route_bf16"])
def test_permute_golden(cuda, case):
    g = load_golden(case)
    so, io, se, cnt, nl = moe.permute(g["topk_ids"].to(cuda), g["cfg"]["experts"])
    n = int(nl.item())
    assert n == g["num_local"]
    assert torch.equal(so.cpu()[:n], g["sort_order"])
    assert torch.equal(io.cpu()[:n], g["inverse_order"])
    assert torch.equal(se.cpu()[:g["sorted_expert_ids"].numel()], g["sorted_expert_ids"])


@pytest.mark.parametrize("tp", [2, 4, 8])
def test_permute_expert_placement(cuda, tp):
    g = torch.Generator().manual_seed(tp)
    ids = torch.stack([torch.randperm(512, generator=g)[:10] for _ in range(256)])
    for rank in range(tp):
        check(ids, 512, tp, rank, cuda)


@pytest.mark.parametrize("T,k,E", [(1, 1, 8), (1, 10, 512), (3000, 8, 64), (8192, 10, 512), (5, 4, 1024)])
def test_permute_shapes(cuda, T, k, E):
    g = torch.Generator().manual_seed(T + k)
    ids = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)]).int()
    check(ids, E, dev=cuda)


def test_permute_all_on_one_expert_per_slot(cuda):
    ids = torch.arange(4).repeat(700, 1)  # every token routes to experts 0..3
    check(ids, 16, dev=cuda)
