"""The C restatement of torch's CPU top-k order (the order the CUDA router replays) agrees
with torch.topk on tie-heavy inputs, NaN rows, and both libstdc++ code paths."""
import pytest
import torch

from oracle.ctopk import topk_torch_cpu_order


@pytest.mark.parametrize("E,k", [(512, 10), (64, 8), (512, 8), (1024, 16), (16, 4), (33, 3), (7, 7)])
def test_c_topk_equals_torch(E, k):
    g = torch.Generator().manual_seed(E * 100 + k)
    x = (torch.randn(2000, E, generator=g) * 1.28).to(torch.bfloat16).float()
    x[::13, 0] = float("nan")
    x[5::17] = 0.25  # whole rows tied
    s = torch.softmax(x, -1)
    v, i = torch.topk(s, k, -1)
    v2, i2 = topk_torch_cpu_order(s, k)
    assert torch.equal(i, i2)
    assert torch.equal(v.nan_to_num(7.0), v2.nan_to_num(7.0))


def test_lowest_index_rule_is_not_torch_order():
    """Documents why the router replays libstdc++: a 'lowest index first' tie rule differs."""
    g = torch.Generator().manual_seed(1)
    x = (torch.randn(4000, 512, generator=g) * 1.28).to(torch.bfloat16).float()
    _, i = torch.topk(x, 10, -1)
    stable = torch.argsort(-x, dim=-1, stable=True)[:, :10]
    assert (i != stable).any(-1).float().mean() > 0.05
