"""Failure detection on the device: a wait inside a kernel that can never
complete must end the kernel with an error the host reads (OSC_ETIMEDOUT from
osc_synchronize), not hang the GPU, and the context must stay usable.

The waits run out on purpose through osc_selfcheck_timeout (a grid barrier
expecting one CTA more than the grid has, an mbarrier nobody arrives on):
nothing faults, traps or loops without bound. After each, the next
DynamicQuantizeMatMul on the same context (whose DynamicQuantizeLinear kernel
uses the same grid barrier and counters) is bit-exact against the oracle."""
from __future__ import annotations

import time

import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu


def _dqmm_bit_exact(ctx, seed):
    import torch

    from onnxsharp_b200.runtime import DqmmWeights, dqmm

    rng = np.random.default_rng(seed)
    a = rng.normal(0, 1, (512, 256)).astype(np.float32)
    w = rng.integers(-127, 128, (256, 384)).astype(np.int8)
    ws = rng.uniform(0.001, 0.02, 384).astype(np.float32)
    b = rng.normal(0, 0.01, 384).astype(np.float32)
    W = DqmmWeights(ctx, torch.from_numpy(w).cuda(), 256, 384, 0)
    acc = torch.empty((512, 384), dtype=torch.int32, device="cuda")
    y = dqmm(ctx, torch.from_numpy(a).cuda(), W, torch.from_numpy(ws).cuda(), torch.from_numpy(b).cuda(), acc_out=acc)
    ctx.synchronize()
    ry, _, racc, _ = oracle.dqmm(a, w, 0, ws, b)
    assert np.array_equal(acc.cpu().numpy(), racc)
    assert np.array_equal(y.cpu().numpy().view(np.uint32), ry.view(np.uint32))


@pytest.mark.parametrize("which", [0, 1], ids=["grid_barrier", "mbarrier"])
def test_starved_wait_reports_timeout_and_context_recovers(ctx, which):
    from onnxsharp_b200 import _lib

    lib = _lib.load()
    _dqmm_bit_exact(ctx, 10 + which)  # healthy before
    t0 = time.monotonic()
    assert lib.osc_selfcheck_timeout(ctx.handle, which) == _lib.OSC_OK
    st = lib.osc_synchronize(ctx.handle, 30000)
    dt = time.monotonic() - t0
    assert st == _lib.OSC_ETIMEDOUT, (st, _lib.last_error())
    assert "bounded internal wait" in _lib.last_error()
    assert 0.5 < dt < 20.0  # the wait gave up after its limit (~1.5 s at full clock)
    # the error word was cleared: the next synchronize is clean
    assert lib.osc_synchronize(ctx.handle, 30000) == _lib.OSC_OK
    _dqmm_bit_exact(ctx, 20 + which)  # the grid barrier counters start from zero again


def test_selfcheck_timeout_rejects_unknown_probe(ctx):
    from onnxsharp_b200 import _lib

    assert _lib.load().osc_selfcheck_timeout(ctx.handle, 7) == _lib.OSC_EINVAL
