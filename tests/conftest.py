"""Shared pytest setup: the `gpu` marker, the repo root on sys.path, and the
per-session CUDA context used by GPU parity tests."""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU and the built libonnxsharp_cuda.so")


def rel_err(got, ref) -> float:
    """The reference's GEMM metric: max |got-ref| / max(1, |ref|) (GemmKernelTests.cs:116-120)."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    if got.size == 0:
        return 0.0
    return float(np.max(np.abs(got - ref) / np.maximum(1.0, np.abs(ref))))


@pytest.fixture(scope="session")
def golden():
    return dict(np.load(GOLDEN / "oracle_small.npz"))


@pytest.fixture(scope="session")
def ctx():
    """One osc_ctx on cuda:0 bound to torch's current stream. Fails (does not
    skip) when the CUDA library cannot be loaded: GPU tests never fall back."""
    import torch

    from onnxsharp_b200.runtime import Context

    if not torch.cuda.is_available():
        pytest.fail("GPU test selected but CUDA is not available")
    c = Context(0)
    c.use_torch_stream()
    yield c
    torch.cuda.synchronize()
    c.close()
