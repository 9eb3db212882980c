"""osc_gemm_bias_f32_noalloc: the MatMul+bias entry point for callers that
must not allocate device memory while serving (their GPU memory is fixed at
start-up, or a cudaMalloc could stall other work sharing the device). Its
temporaries come from a fixed array inside the library instead of the
context's growable scratch arena.

Checked against the CPU oracle (the reference's FMA chain), not against the
allocating entry point, on two calls in a row; that it allocates nothing is
checked twice: in a fresh process where every library allocation is made to
fail (OSC_FAULT=alloc) and by the device's free memory across calls. This file
is collected last so that a run stopping at the first failure has already run
every other test; it also passes on its own in a fresh process."""
from __future__ import annotations

import os
import subprocess
import sys

import numpy as np
import pytest

import oracle
from conftest import ROOT, rel_err

pytestmark = pytest.mark.gpu
TOL = 1e-4  # the GEMM tolerance used throughout (GemmKernelTests.cs:116-120)


def _noalloc(ctx, a, w, bias, out, act=0, lda=None):
    from onnxsharp_b200._lib import call, ptr

    call("osc_gemm_bias_f32_noalloc", ctx.handle, ptr(a), int(a.shape[0]), w.k, int(lda or a.stride(0)), w.handle,
         ptr(bias), int(act), ptr(out), int(out.stride(0)))


def _weights(ctx, rng, k, n):
    import torch

    from onnxsharp_b200.runtime import GemmWeights

    b = rng.uniform(-1, 1, (k, n)).astype(np.float32)
    bias = rng.uniform(-1, 1, n).astype(np.float32)
    return b, bias, GemmWeights(ctx, torch.from_numpy(b).cuda(), k, n), torch.from_numpy(bias).cuda()


def test_noalloc_matches_oracle_on_two_calls(ctx):
    import torch

    rng = np.random.default_rng(606)
    k, n = 512, 2048
    b, bias, w, tbias = _weights(ctx, rng, k, n)
    # Two calls in a row with different inputs and sizes: the second reuses
    # (and must fully overwrite) the shared array left by the first.
    for m in (2048, 777):
        a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
        got = torch.full((m, n), float("nan"), device="cuda")
        _noalloc(ctx, torch.from_numpy(a).cuda(), w, tbias, got)
        ctx.synchronize()
        assert rel_err(got.cpu().numpy(), oracle.gemm(a, b, col_bias=bias)) <= TOL


def test_noalloc_unaligned_output_silu_and_row_pitch(ctx):
    """C at an address off by one float (plain-store epilogue), SiLU fused, and
    A with a row pitch larger than k."""
    import torch

    rng = np.random.default_rng(607)
    m, k, n, lda = 300, 200, 136, 232
    b, bias, w, tbias = _weights(ctx, rng, k, n)
    a_full = rng.uniform(-1, 1, (m, lda)).astype(np.float32)
    ta = torch.from_numpy(a_full).cuda()
    store = torch.full((m * n + 1,), float("nan"), device="cuda")
    c = store[1:].view(m, n)  # 4 bytes past a 256-byte boundary
    _noalloc(ctx, ta[:, :k], w, tbias, c, act=1, lda=lda)
    ctx.synchronize()
    ref = oracle.gemm(np.ascontiguousarray(a_full[:, :k]), b, col_bias=bias, act=1)
    assert rel_err(c.cpu().numpy(), ref) <= TOL


def test_noalloc_rejects_sizes_beyond_the_fixed_scratch(ctx):
    import torch

    from onnxsharp_b200 import OscError
    from onnxsharp_b200.runtime import GemmWeights

    w = GemmWeights(ctx, torch.ones(512, 64, device="cuda"), 512, 64)
    a = torch.ones(2049, 512, device="cuda")  # 2049 * 512 > 1048576
    out = torch.empty(2049, 64, device="cuda")
    with pytest.raises(OscError, match="fixed scratch limit"):
        _noalloc(ctx, a, w, None, out)


def test_noalloc_leaves_device_free_memory_unchanged(ctx):
    import torch

    rng = np.random.default_rng(608)
    m, k, n = 1024, 256, 512
    b, bias, w, tbias = _weights(ctx, rng, k, n)
    a = torch.from_numpy(rng.uniform(-1, 1, (m, k)).astype(np.float32)).cuda()
    out = torch.empty((m, n), device="cuda")
    _noalloc(ctx, a, w, tbias, out)  # first launch loads the kernels' code
    ctx.synchronize()
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    for _ in range(3):
        _noalloc(ctx, a, w, tbias, out)
    ctx.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0


FRESH = r"""
import numpy as np, torch, oracle
from onnxsharp_b200 import OscError
from onnxsharp_b200._lib import call, ptr
from onnxsharp_b200.runtime import Context, GemmWeights, gemm_bias
ctx = Context(0); ctx.use_torch_stream()
rng = np.random.default_rng(609)
m, k, n = 640, 384, 768
a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
b = rng.uniform(-1, 1, (k, n)).astype(np.float32)
bias = rng.uniform(-1, 1, n).astype(np.float32)
w = GemmWeights(ctx, torch.from_numpy(b).cuda(), k, n)
ta, tb = torch.from_numpy(a).cuda(), torch.from_numpy(bias).cuda()
ref = oracle.gemm(a, b, col_bias=bias)
for _ in range(2):
    out = torch.full((m, n), float("nan"), device="cuda")
    call("osc_gemm_bias_f32_noalloc", ctx.handle, ptr(ta), m, k, k, w.handle, ptr(tb), 0, ptr(out), n)
    ctx.synchronize()
    err = float(np.max(np.abs(out.cpu().numpy() - ref) / np.maximum(1.0, np.abs(ref))))
    assert err <= 1e-4, err
try:
    gemm_bias(ctx, ta, w, tb)  # needs the scratch arena: the injected allocation failure must hit it
    raise SystemExit("allocating entry point did not fail")
except OscError as e:
    assert "injected" in str(e), e
print("ok", err)
"""


def test_noalloc_first_call_in_fresh_process_with_allocation_failing():
    """A fresh process whose library allocations all fail (OSC_FAULT=alloc):
    the no-alloc entry point still works from its first call, while the
    allocating one reports the injected failure."""
    env = dict(os.environ, OSC_FAULT="alloc", PYTHONPATH=str(ROOT))
    r = subprocess.run([sys.executable, "-c", FRESH], capture_output=True, text=True, env=env, cwd=ROOT, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert r.stdout.strip().startswith("ok")
