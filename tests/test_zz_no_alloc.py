"""msv_ragged_moe_gemm_fp8_noalloc (the ragged FP8 GEMM with its tile list in a static device
array instead of a caller workspace) against msv_ragged_moe_gemm_fp8, both through the C ABI.

Two calls in a row with different row layouts: the second call's tile list is shorter than
the first's, so a stale tail left in the shared array must not leak into its result.  The
file is named to be collected last and needs nothing from the other test files, so it runs
the same alone in a fresh process or after the whole suite.
Tolerance: bf16 max-abs-rel <= 2e-2 and cosine >= 0.9999 (the bar of every GEMM test)."""
import pytest
import torch

import muserve_b200._lib as L
from conftest import assert_close_bf16
from muserve_b200 import moe

pytestmark = pytest.mark.gpu

FP8 = torch.float8_e4m3fn


def _inputs(ids: torch.Tensor, E: int, N: int, K: int, seed: int, dev):
    """Random block-scaled e4m3 operands on ``dev`` for the row->expert map ``ids``."""
    g = torch.Generator(device=dev).manual_seed(seed)
    M = ids.numel()
    a = (torch.randn(M, K, generator=g, device=dev) * 2).to(FP8)
    a_s = torch.rand(M, K // 128, generator=g, device=dev) * 0.01 + 1e-3
    w = (torch.randn(E, N, K, generator=g, device=dev) * 2).to(FP8)
    w_s = torch.rand(E, N // 128, K // 128, generator=g, device=dev) * 0.01 + 1e-3
    return a, a_s, w, w_s, ids.to(device=dev, dtype=torch.int32).contiguous()


def _noalloc(a, a_s, w, w_s, ids, out):
    lib = L.load()
    M, K = a.shape
    E, N, _ = w.shape
    L.check(lib.msv_ragged_moe_gemm_fp8_noalloc(a.data_ptr(), a_s.data_ptr(), M, K, w.data_ptr(), w_s.data_ptr(), E,
                                                N, ids.data_ptr(), out.data_ptr(), L.stream_ptr()),
            "msv_ragged_moe_gemm_fp8_noalloc")
    return out


def test_noalloc_matches_workspace_entry_point_twice(cuda):
    E, N, K = 8, 512, 1024
    g = torch.Generator().manual_seed(5)
    # call 1: many rows, unsorted runs, rows with id -1 at both ends
    ids1 = torch.cat([torch.full((17,), -1), torch.randint(0, E, (60,), generator=g).repeat_interleave(9),
                      torch.full((40,), 2), torch.full((23,), -1)])
    # call 2: fewer rows (a shorter tile list than call 1 left behind), one large expert run
    ids2 = torch.cat([torch.full((150,), 5), torch.full((3,), 0), torch.full((11,), -1), torch.full((20,), 7)])
    for i, ids in enumerate((ids1, ids2)):
        a, a_s, w, w_s, idx = _inputs(ids, E, N, K, seed=100 + i, dev=cuda)
        M = idx.numel()
        ref = moe.ragged_gemm(a, a_s, w, w_s, idx, torch.full((M, N), 7.0, dtype=torch.bfloat16, device=cuda))
        out = _noalloc(a, a_s, w, w_s, idx, torch.full((M, N), 7.0, dtype=torch.bfloat16, device=cuda))
        torch.cuda.synchronize()
        moe.check_device_error()
        neg = (idx < 0).cpu()
        out, ref = out.cpu(), ref.cpu()
        assert (out[neg] == 7.0).all(), f"call {i + 1}: rows with id -1 must stay untouched"
        assert_close_bf16(out[~neg], ref[~neg])


def test_noalloc_rejects_sizes_beyond_the_scratch(cuda):
    # M * N/128 = 8192 * 32 = 262144 tiles > 262128: refused on the host before any launch.
    # The buffers have the claimed sizes all the same.
    M, K, N, E = 8192, 128, 4096, 1
    a = torch.zeros(M, K, dtype=FP8, device=cuda)
    a_s = torch.ones(M, 1, device=cuda)
    w = torch.zeros(E, N, K, dtype=FP8, device=cuda)
    w_s = torch.ones(E, N // 128, 1, device=cuda)
    ids = torch.zeros(M, dtype=torch.int32, device=cuda)
    out = torch.zeros(M, N, dtype=torch.bfloat16, device=cuda)
    lib = L.load()
    rc = lib.msv_ragged_moe_gemm_fp8_noalloc(a.data_ptr(), a_s.data_ptr(), M, K, w.data_ptr(), w_s.data_ptr(), E, N,
                                             ids.data_ptr(), out.data_ptr(), L.stream_ptr())
    assert rc == L.MSV_ERR_INVALID
    msg = lib.msv_last_error().decode()
    assert "262128" in msg and "msv_ragged_moe_gemm_fp8" in msg, msg
    # one row fewer fits
    M2 = 8191
    rc = lib.msv_ragged_moe_gemm_fp8_noalloc(a.data_ptr(), a_s.data_ptr(), M2, K, w.data_ptr(), w_s.data_ptr(), E, N,
                                             ids.data_ptr(), out.data_ptr(), L.stream_ptr())
    L.check(rc, "msv_ragged_moe_gemm_fp8_noalloc at the limit")
    torch.cuda.synchronize()
    moe.check_device_error()
    assert (out[:M2].float() == 0).all()
