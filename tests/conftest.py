import os
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 GPU (B200); run with -m gpu")


def load_golden(name: str) -> dict:
    return torch.load(os.path.join(GOLDEN, f"{name}.pt"), weights_only=False)


def max_abs_rel(a: torch.Tensor, b: torch.Tensor) -> float:
    a, b = a.float().cpu(), b.float().cpu()
    return ((a - b).abs().max() / b.abs().max().clamp(min=1e-30)).item()


def cosine(a: torch.Tensor, b: torch.Tensor) -> float:
    a, b = a.float().cpu().flatten(), b.float().cpu().flatten()
    return torch.nn.functional.cosine_similarity(a, b, dim=0).item()


# the bar for bf16 outputs vs the reference
TOL_MAX_ABS_REL = 2e-2
TOL_COSINE = 0.9999


def assert_close_bf16(out, ref, tol=TOL_MAX_ABS_REL, cos=TOL_COSINE):
    mar, c = max_abs_rel(out, ref), cosine(out, ref)
    assert mar <= tol and c >= cos, f"max_abs_rel={mar:.3e} (<= {tol}) cosine={c:.6f} (>= {cos})"


@pytest.fixture(scope="session")
def cuda():
    assert torch.cuda.is_available(), "GPU test run without a CUDA device"
    import muserve_b200._lib as L
    L.load()
    return torch.device("cuda:0")
