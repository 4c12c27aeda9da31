"""Kernel-layer MoE API, mirroring ``muserve/kernels`` (MoE and FP8 GEMM entries only)."""
from .fp8_matmul import w8a8_block_fp8_matmul  # noqa: F401
