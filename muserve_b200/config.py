"""Shape constants of the reference's MoE layer (``muserve/config.py:5-46``).

The reference binds them at import; here every op reads them at call time and takes
explicit overrides, so one process can run several shapes (tests, benches).
"""
from __future__ import annotations

from dataclasses import dataclass

HIDDEN_SIZE = 4096
NUM_EXPERTS = 512
NUM_EXPERTS_PER_TOK = 10
MOE_INTERMEDIATE = 1024
SHARED_INTERMEDIATE = 1024
TP_SIZE = 1


@dataclass(frozen=True)
class MoEConfig:
    hidden: int = HIDDEN_SIZE
    experts: int = NUM_EXPERTS
    top_k: int = NUM_EXPERTS_PER_TOK
    inter: int = MOE_INTERMEDIATE
    shared_inter: int = SHARED_INTERMEDIATE
    tokens: int = 64


# the benchmark configurations (seeded synthetic data; no checkpoint is used)
C0_CPU_CHECK = MoEConfig(hidden=2048, experts=64, top_k=8, inter=512, shared_inter=512, tokens=32)
C1_DECODE = MoEConfig(tokens=64)
C2_PREFILL = MoEConfig(tokens=8192)
C3_TP_DECODE = MoEConfig(tokens=256)
C4_STACK = MoEConfig(tokens=128)
