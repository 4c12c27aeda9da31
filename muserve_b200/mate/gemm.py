"""``mate.gemm`` drop-ins backed by the sm_100a grouped GEMM.

The reference calls these two vendor ops (mate 0.2.1, not vendored):
``ragged_m_moe_gemm_8bit`` at ``muserve/model/qwen35_layer_v2.py:613-618`` and ``:638-643``,
``gemm_fp8_nt_groupwise`` at ``:102-106``.
"""
from __future__ import annotations

import torch

from .. import moe


def ragged_m_moe_gemm_8bit(a_pair, w_pair, m_indices: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
    """``out[m] = gemm(a[m], w[m_indices[m]])`` (block scales per row x 128 and per 128 x 128),
    written into the caller's bf16 ``out``; rows with index -1 are left untouched."""
    a, a_scale = a_pair
    w, w_scale = w_pair
    return moe.ragged_gemm(a, a_scale, w, w_scale, m_indices, out)


def gemm_fp8_nt_groupwise(a: torch.Tensor, b: torch.Tensor, a_scale: torch.Tensor, b_scale: torch.Tensor,
                          scale_granularity_mnk=(1, 128, 128), out_dtype=torch.bfloat16) -> torch.Tensor:
    """``a [M,K] e4m3 x b [N,K] e4m3 -> [M,N]`` with per-row x 128 activation scales and 128 x 128
    weight scales."""
    assert tuple(scale_granularity_mnk) == (1, 128, 128), "only (1,128,128) scale granularity"
    assert out_dtype == torch.bfloat16, "only bf16 output"
    return moe.gemm_nt(a, a_scale, b, b_scale)
