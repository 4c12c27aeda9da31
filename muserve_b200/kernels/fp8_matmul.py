"""W8A8 block-wise FP8 GEMM (``muserve/kernels/fp8_matmul.py:172-216``) on sm_100a tensor
cores.  Same arguments and result; only ``block_size == [128, 128]`` and bf16 output."""
from __future__ import annotations

from typing import List

import torch

from .. import moe


def w8a8_block_fp8_matmul(A: torch.Tensor, B: torch.Tensor, As: torch.Tensor, Bs: torch.Tensor,
                          block_size: List[int], output_dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    """``A [..., M, K] e4m3 x B [N, K] e4m3 -> [..., M, N]``; ``As [..., M, K/128]``,
    ``Bs [N/128, K/128]`` fp32 scales."""
    assert len(block_size) == 2
    block_n, block_k = block_size
    assert (block_n, block_k) == (128, 128), "only 128x128 weight blocks"
    assert output_dtype == torch.bfloat16, "only bf16 output"
    assert A.shape[-1] == B.shape[-1], "K dimension mismatch"
    m = A.numel() // A.shape[-1]
    n, k = B.shape
    a2 = A.reshape(m, k).contiguous()
    as2 = As.reshape(m, As.shape[-1]).contiguous()
    c = moe.gemm_nt(a2, as2, B.contiguous(), Bs.contiguous())
    return c.reshape(*A.shape[:-1], n)
