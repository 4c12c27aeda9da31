"""Block-scaled FP8 GEMMs on tcgen05 vs the oracle's restatement of the mate ops
(gemm_fp8_nt_groupwise, ragged_m_moe_gemm_8bit; qwen35_layer_v2.py:102-106, 613-618, 638-643).
Tolerance: bf16 max-abs-rel <= 2e-2 and cosine >= 0.9999."""
import pytest
import torch

from conftest import assert_close_bf16
from muserve_b200 import moe
from muserve_b200.kernels.fp8_matmul import w8a8_block_fp8_matmul
from muserve_b200.mate import gemm as mate_gemm
from oracle import moe_oracle as orc

pytestmark = pytest.mark.gpu


def rand_act(m, k, g):
    return orc.fast_fp8_quantize((torch.randn(m, k, generator=g)).to(torch.bfloat16))


def rand_w(n, k, g):
    return orc.quantize_weight_blockwise(torch.randn(n, k, generator=g) * 0.02)


@pytest.mark.parametrize("M", [1, 16, 33, 64, 200, 1000])
@pytest.mark.parametrize("N,K", [(128, 128), (1024, 512), (256, 4096)])
def test_dense_gemm(cuda, M, N, K):
    g = torch.Generator().manual_seed(M * 7 + N + K)
    a, a_s = rand_act(M, K, g)
    b, b_s = rand_w(N, K, g)
    ref = orc.gemm_fp8_nt_groupwise(a, b, a_s, b_s)
    out = mate_gemm.gemm_fp8_nt_groupwise(a.to(cuda), b.to(cuda), a_s.to(cuda), b_s.to(cuda))
    assert_close_bf16(out, ref)
    # most elements round to the same bf16 value
    assert (out.cpu() == ref).float().mean() > 0.95


def test_w8a8_block_fp8_matmul_batched_shape(cuda):
    g = torch.Generator().manual_seed(3)
    a, a_s = rand_act(2 * 48, 512, g)
    b, b_s = rand_w(384, 512, g)
    out = w8a8_block_fp8_matmul(a.view(2, 48, 512).to(cuda), b.to(cuda), a_s.view(2, 48, 4).to(cuda), b_s.to(cuda),
                                [128, 128])
    assert out.shape == (2, 48, 384)
    assert_close_bf16(out.reshape(96, 384), orc.gemm_fp8_nt_groupwise(a, b, a_s, b_s))


@pytest.mark.parametrize("layout", ["sorted_pad", "unsorted_runs", "neg_first", "skewed"])
def test_ragged_gemm(cuda, layout):
    g = torch.Generator().manual_seed(len(layout))
    E, N, K = 8, 256, 512
    if layout == "sorted_pad":
        ids = torch.sort(torch.randint(0, E, (300,), generator=g)).values
        ids = torch.cat([ids, torch.full((84,), -1)])
    elif layout == "unsorted_runs":
        ids = torch.randint(0, E, (40,), generator=g).repeat_interleave(7)
    elif layout == "neg_first":
        ids = torch.cat([torch.full((50,), -1), torch.sort(torch.randint(0, E, (130,), generator=g)).values])
    else:
        ids = torch.cat([torch.full((700,), 3), torch.full((5,), 1), torch.full((300,), 6)])
    ids = ids.int()
    M = ids.numel()
    a, a_s = rand_act(M, K, g)
    w = torch.empty(E, N, K, dtype=torch.float8_e4m3fn)
    w_s = torch.empty(E, N // 128, K // 128)
    for e in range(E):
        w[e], w_s[e] = rand_w(N, K, g)
    sentinel = torch.full((M, N), 7.0, dtype=torch.bfloat16)
    ref = orc.ragged_m_moe_gemm_8bit((a, a_s), (w, w_s), ids, sentinel.clone())
    out = mate_gemm.ragged_m_moe_gemm_8bit((a.to(cuda), a_s.to(cuda)), (w.to(cuda), w_s.to(cuda)), ids.to(cuda),
                                           sentinel.to(cuda))
    torch.cuda.synchronize()
    neg = ids < 0
    assert (out.cpu()[neg] == 7.0).all(), "rows with id -1 must stay untouched"
    assert_close_bf16(out.cpu()[~neg], ref[~neg])


def test_gemm_reports_no_device_timeout(cuda):
    moe.check_device_error()
