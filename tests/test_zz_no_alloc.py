"""osc_gemm_bias_f32_noalloc: the MatMul+bias entry point for callers that
must not allocate device memory while serving (their GPU memory is fixed at
start-up, or a cudaMalloc could stall other work sharing the device). Its
temporaries come from a fixed array inside the library instead of the
context's growable scratch arena. This file is collected last so that a run
stopping at the first failure has already run every other test; it also
passes on its own in a fresh process."""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from conftest import rel_err

pytestmark = pytest.mark.gpu
TOL = 1e-4  # the GEMM tolerance used throughout (GemmKernelTests.cs:116-120)


def _noalloc(ctx, a, w, bias, out):
    from onnxsharp_b200._lib import call, ptr

    call("osc_gemm_bias_f32_noalloc", ctx.handle, ptr(a), int(a.shape[0]), w.k, int(a.stride(0)), w.handle,
         ptr(bias), 0, ptr(out), int(out.stride(0)))


def test_noalloc_matches_the_allocating_entry_point_on_two_calls(ctx):
    import torch

    from onnxsharp_b200.runtime import GemmWeights, gemm_bias

    rng = np.random.default_rng(606)
    k, n = 512, 2048
    b = rng.uniform(-1, 1, (k, n)).astype(np.float32)
    bias = torch.from_numpy(rng.uniform(-1, 1, n).astype(np.float32)).cuda()
    w = GemmWeights(ctx, torch.from_numpy(b).cuda(), k, n)
    # Two calls in a row with different inputs and sizes: the second reuses
    # (and must fully overwrite) the shared array left by the first.
    for m in (2048, 777):
        a = torch.from_numpy(rng.uniform(-1, 1, (m, k)).astype(np.float32)).cuda()
        ref = gemm_bias(ctx, a, w, bias)
        got = torch.full((m, n), float("nan"), device="cuda")
        _noalloc(ctx, a, w, bias, got)
        ctx.synchronize()
        assert rel_err(got.cpu().numpy(), ref.cpu().numpy()) <= TOL


def test_noalloc_rejects_sizes_beyond_the_fixed_scratch(ctx):
    import torch

    from onnxsharp_b200 import OscError
    from onnxsharp_b200.runtime import GemmWeights

    w = GemmWeights(ctx, torch.ones(512, 64, device="cuda"), 512, 64)
    a = torch.ones(2049, 512, device="cuda")  # 2049 * 512 > 1048576
    out = torch.empty(2049, 64, device="cuda")
    with pytest.raises(OscError, match="fixed scratch limit"):
        _noalloc(ctx, a, w, None, out)
