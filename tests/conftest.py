import sys
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parent.parent
GOLDEN = Path(__file__).resolve().parent / "golden"
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

# Tolerances (normwise: max|out - ref| <= tol * max|ref|), from the parity
# requirement on the reference's non-fast Local Attender.
TOL = {torch.float32: 1e-4, torch.bfloat16: 2e-2, torch.float16: 2e-3}


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 CUDA device (run with -m gpu)")
    config.addinivalue_line("markers", "slow: long-running test")


def normwise_err(out: torch.Tensor, ref: torch.Tensor) -> float:
    out = out.detach().to(torch.float64).cpu()
    ref = ref.detach().to(torch.float64).cpu()
    if ref.numel() == 0:
        return 0.0
    scale = ref.abs().max().item()
    return (out - ref).abs().max().item() / max(scale, 1e-30)


def dtype_of(name: str) -> torch.dtype:
    return {"torch.float32": torch.float32, "torch.bfloat16": torch.bfloat16,
            "torch.float16": torch.float16}[name]


@pytest.fixture(scope="session")
def golden_cases():
    return torch.load(GOLDEN / "la_cases.pt", weights_only=False)["cases"]


@pytest.fixture(scope="session")
def golden_config1():
    return torch.load(GOLDEN / "la_config1.pt", weights_only=False)


@pytest.fixture(scope="session")
def cuda_lib():
    """The built C-ABI library; GPU tests require it (no fallback)."""
    from uplift_b200 import _native
    return _native.load(build_if_missing=True)


def pytest_collection_modifyitems(config, items):
    if not torch.cuda.is_available():
        skip = pytest.mark.skip(reason="no CUDA device")
        for item in items:
            if "gpu" in item.keywords:
                item.add_marker(skip)
