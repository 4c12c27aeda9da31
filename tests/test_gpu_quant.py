"""Per-row per-128 e4m3 quantisation bit-exact with _fast_fp8_quantize (qwen35_layer_v2.py:71-86)."""
import hashlib

import pytest
import torch

from conftest import load_golden
from muserve_b200 import moe
from oracle import moe_oracle as orc

pytestmark = pytest.mark.gpu


def exact(q, s, rq, rs):
    assert torch.equal(q.cpu().view(torch.uint8), rq.view(torch.uint8))
    assert torch.equal(s.cpu().nan_to_num(-1.0), rs.nan_to_num(-1.0))


def test_quant_golden_c0(cuda):
    g = load_golden("c0")
    c = g["cfg"]
    x = orc.make_hidden(c["tokens"], c["hidden"], c["xseed"])
    p = orc.permute(g["topk_ids"], c["experts"])
    rows = torch.cat([x[p.sorted_token_idx], torch.zeros(p.padded_m - p.num_local, c["hidden"], dtype=x.dtype)])
    q, s = moe.fp8_quant_128(rows.to(cuda))
    assert hashlib.sha256(q.cpu().view(torch.uint8).numpy().tobytes()).hexdigest() == g["x_fp8_sha"]
    assert torch.equal(s.cpu(), g["x_scale"])


@pytest.mark.parametrize("scale", [1.0, 1e-3, 1e3, 1e-30, 3e35])
@pytest.mark.parametrize("M,K", [(1, 128), (37, 4096), (700, 1024), (64, 2048)])
def test_quant_random(cuda, scale, M, K):
    g = torch.Generator().manual_seed(M + K)
    x = (torch.randn(M, K, generator=g) * scale).to(torch.bfloat16)
    x[0, :128] = 0  # an all-zero block -> scale 1e-12/448
    q, s = moe.fp8_quant_128(x.to(cuda))
    exact(q, s, *orc.fast_fp8_quantize(x))


def test_quant_special_values(cuda):
    x = torch.randn(4, 256).to(torch.bfloat16)
    x[1, 5] = float("nan")
    x[2, 130] = float("inf")
    x[3, 0] = -float("inf")
    q, s = moe.fp8_quant_128(x.to(cuda))
    rq, rs = orc.fast_fp8_quantize(x)
    assert torch.equal(s.cpu().isnan(), rs.isnan())
    # invalid operations (inf/inf) give a NaN whose sign is platform-defined (x86: negative
    # default NaN -> e4m3 0xFF; GPU: 0x7F): compare NaN-ness there, bytes everywhere else
    qb, rb = q.cpu().view(torch.uint8), rq.view(torch.uint8)
    rnan = (rb & 0x7F) == 0x7F
    assert torch.equal((qb & 0x7F) == 0x7F, rnan)
    assert torch.equal(qb[~rnan], rb[~rnan])


def test_quant_gather_and_kb_major(cuda):
    x = torch.randn(50, 512).to(torch.bfloat16)
    idx = torch.tensor([3, 3, 49, 0, 17], dtype=torch.int32)
    q, s = moe.fp8_quant_128(x.to(cuda), row_index=idx.to(cuda), scale_kb_major=True)
    exact(q, s.contiguous(), *orc.fast_fp8_quantize(x[idx.long()]))
