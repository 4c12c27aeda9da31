"""The C-ABI library builds, loads without a GPU, exports every entry point declared in
include/muserve_moe.h, and rejects bad arguments with a status code (no GPU touched)."""
import ctypes
import os

import pytest

from conftest import ROOT
import muserve_b200._lib as L

HEADER = os.path.join(ROOT, "include", "muserve_moe.h")


@pytest.fixture(scope="module")
def lib():
    from muserve_b200 import build
    build.build()
    return L.load(require_gpu=False)


def test_exports_every_declared_symbol(lib):
    names = L.header_symbols(HEADER)
    assert len(names) >= 12
    for n in names:
        assert hasattr(lib, n), f"{n} declared in the header but not exported"
    assert set(names) <= set(L._SIGS), "python binding misses a declared entry point"


def test_version_and_error_string(lib):
    assert lib.msv_version() >= 100
    rc = lib.msv_route_topk(None, 0, 1, 512, 10, 1, None, L.MSV_BF16, None, L.MSV_I32, None)
    assert rc == L.MSV_ERR_INVALID
    assert b"msv_route_topk" in lib.msv_last_error()


@pytest.mark.parametrize("call", [
    lambda lib: lib.msv_topk_select(None, 0, 1, 8, 9, None, L.MSV_I64, None, None),
    lambda lib: lib.msv_moe_permute(None, L.MSV_I64, 4, 2, 8, 0, 1, 0, 128, None, None, None, None, None, None),
    lambda lib: lib.msv_fp8_quant_128(None, 0, 4, 100, None, None, 0, None, 0, 0, None),
    lambda lib: lib.msv_ragged_moe_gemm_fp8(None, None, 4, 100, None, None, 2, 128, None, None, None, 0, None),
    lambda lib: lib.msv_gemm_fp8_nt_groupwise(None, None, 4, 128, None, None, 100, None, None, 0, None),
    lambda lib: lib.msv_add_rms_norm_gemma(None, None, None, 4, 4096, 1e-6, None, None),
    lambda lib: lib.msv_moe_forward_tp(None, None, None, None, None, None, None, 0, None, 0, None, None),
    lambda lib: lib.msv_ipc_export(None, None, None),
    lambda lib: lib.msv_ipc_import(None, 0, None),
    lambda lib: lib.msv_add_rms_norm_gemma(None, None, None, 4, 4100, 1e-6, None, None),
    lambda lib: lib.msv_router_from_hidden_bias(None, None, 4, 4096, 512, 10, 1, 1, None, None, 1, None, 2, None,
                                                None, 0, None),
])
def test_bad_arguments_rejected(lib, call):
    assert call(lib) == L.MSV_ERR_INVALID


def test_workspace_sizes(lib):
    s = L.MoeShape(tokens=64, hidden=4096, num_experts=512, top_k=10, inter=1024, shared_inter=1024,
                   placement=0, tp=1, rank=0, add_shared=1, combine_mode=0, weights_dtype=L.MSV_BF16)
    n = lib.msv_moe_forward_workspace_size(ctypes.byref(s))
    rows = 64 * 10 + 64
    assert n > rows * 4096 * 3  # fp8 tokens + bf16 expert outputs at least
    s.hidden = 100  # not a multiple of 128
    assert lib.msv_moe_forward_workspace_size(ctypes.byref(s)) == 0
    s.hidden, s.shared_inter = 4096, 512  # shared intermediate must equal routed
    assert lib.msv_moe_forward_workspace_size(ctypes.byref(s)) == 0
    assert lib.msv_ragged_gemm_workspace_size(1024, 2048) > 0
    # fused TP combine: receive + result areas, 4 bytes per value (two bf16 + a 32-bit flag per word)
    assert lib.msv_tp_shared_bytes(256, 4096) == 2 * 256 * 4096 * 4
    assert lib.msv_tp_shared_bytes(0, 4096) == 0
    assert lib.msv_tp_epoch_bytes() == 1024 * 4
    assert lib.msv_ipc_handle_bytes() == 64
    assert lib.msv_gemm_fp8_workspace_size(64, 1024) > 0


def test_product_path_fails_loudly_without_gpu():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is visible")
    from muserve_b200 import moe
    with pytest.raises(RuntimeError, match="sm_100"):
        moe.route_topk(torch.zeros(2, 8), 2)
