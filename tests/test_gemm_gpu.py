"""MatMul+FusedBias on the B200 tensor cores (3xTF32) against the CPU oracle
(the reference's FMA-chain GEMM), at the reference's tolerance
|d| / max(1, |ref|) <= 1e-4 (GemmKernelTests.cs:116-120)."""
from __future__ import annotations

import json

import numpy as np
import pytest

import oracle
from conftest import GOLDEN, rel_err

pytestmark = pytest.mark.gpu
KAT = json.loads((GOLDEN / "kat.json").read_text())
TOL = KAT["gemm_tolerance"]["vs_naive_double"]


def _run(ctx, a, b, bias=None, act=0, layout=0):
    import torch

    from onnxsharp_b200.runtime import GemmWeights, gemm_bias

    m, k = a.shape
    n = b.shape[1] if layout == 0 else b.shape[0]
    w = GemmWeights(ctx, torch.from_numpy(np.ascontiguousarray(b)).cuda(), k, n, layout)
    out = gemm_bias(ctx, torch.from_numpy(a).cuda(), w, None if bias is None else torch.from_numpy(bias).cuda(), act)
    ctx.synchronize()
    return out.cpu().numpy()


SHAPES = sorted({tuple(s) for key in ("naive_shapes", "column_bias_shapes", "packed_shapes", "scale_bias_shapes")
                 for s in KAT["gemm_tolerance"][key]})


@pytest.mark.parametrize("shape", SHAPES)
def test_gemm_bias_matches_oracle(ctx, shape):
    m, k, n = shape
    rng = np.random.default_rng(m * 31 + k * 7 + n)
    a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
    b = rng.uniform(-1, 1, (k, n)).astype(np.float32)
    bias = rng.uniform(-1, 1, n).astype(np.float32)
    got = _run(ctx, a, b, bias)
    assert rel_err(got, oracle.gemm(a, b, col_bias=bias)) <= TOL


def test_gemm_config1_full_size(ctx):
    """A[2048,512] x B[512,2048] + bias[2048], U(-1,1)."""
    rng = np.random.default_rng(1)
    a = rng.uniform(-1, 1, (2048, 512)).astype(np.float32)
    b = rng.uniform(-1, 1, (512, 2048)).astype(np.float32)
    bias = rng.uniform(-1, 1, 2048).astype(np.float32)
    got = _run(ctx, a, b, bias)
    assert rel_err(got, oracle.gemm(a, b, col_bias=bias)) <= TOL


@pytest.mark.parametrize("m,k,n", [(2000, 300, 2000), (1800, 64, 3600), (4100, 1000, 1920)])
def test_gemm_large_ragged_cta_pairs(ctx, m, k, n):
    """Large GEMMs run on CTA pairs (cluster of 2, tcgen05 cta_group::2, 256 x 256
    pair tiles); ragged M, N and K exercise the partial pair tiles."""
    rng = np.random.default_rng(m + k + n)
    a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
    b = rng.uniform(-1, 1, (k, n)).astype(np.float32)
    bias = rng.uniform(-1, 1, n).astype(np.float32)
    got = _run(ctx, a, b, bias)
    ref = oracle.gemm(a, b, col_bias=bias)
    assert rel_err(got, ref) <= TOL


def test_gemm_golden_fixture(ctx, golden):
    got = _run(ctx, golden["gemm_a"], golden["gemm_b"], golden["gemm_bias"])
    assert rel_err(got, golden["gemm_c"]) <= TOL


def test_gemm_long_k_accumulation(ctx):
    """K = 2304 (256-channel 3x3 conv as a GEMM): chunked TMEM accumulation keeps the error flat."""
    rng = np.random.default_rng(7)
    a = rng.uniform(-1, 1, (300, 2304)).astype(np.float32)
    b = rng.uniform(-1, 1, (2304, 96)).astype(np.float32)
    assert rel_err(_run(ctx, a, b), oracle.gemm(a, b)) <= TOL


def test_gemm_transposed_b_layout(ctx):
    rng = np.random.default_rng(8)
    a = rng.uniform(-1, 1, (77, 100)).astype(np.float32)
    bt = rng.uniform(-1, 1, (130, 100)).astype(np.float32)  # [n, k] (Gemm transB=1)
    got = _run(ctx, a, bt, layout=1)
    assert rel_err(got, oracle.gemm(a, np.ascontiguousarray(bt.T))) <= TOL


def test_gemm_fused_silu(ctx):
    rng = np.random.default_rng(9)
    a = rng.uniform(-1, 1, (130, 64)).astype(np.float32)
    b = rng.uniform(-1, 1, (64, 40)).astype(np.float32)
    bias = rng.uniform(-1, 1, 40).astype(np.float32)
    got = _run(ctx, a, b, bias, act=1)
    assert rel_err(got, oracle.gemm(a, b, col_bias=bias, act=1)) <= TOL


def test_gemm_strided_rows(ctx):
    import torch

    from onnxsharp_b200.runtime import GemmWeights, gemm_bias

    rng = np.random.default_rng(10)
    big = rng.uniform(-1, 1, (64, 80)).astype(np.float32)
    a = big[:, :50]  # lda = 80
    b = rng.uniform(-1, 1, (50, 33)).astype(np.float32)
    w = GemmWeights(ctx, torch.from_numpy(b).cuda(), 50, 33)
    ta = torch.from_numpy(big).cuda()[:, :50]
    out = torch.zeros(64, 40, device="cuda")[:, :33]  # ldc = 40
    gemm_bias(ctx, ta, w, None, 0, out=out, lda=80, ldc=40)
    ctx.synchronize()
    assert rel_err(out.cpu().numpy(), oracle.gemm(np.ascontiguousarray(a), b)) <= TOL


def test_gemm_host_prepack_and_empty_m(ctx):
    import torch

    from onnxsharp_b200.runtime import GemmWeights, gemm_bias

    rng = np.random.default_rng(12)
    b = rng.uniform(-1, 1, (20, 24)).astype(np.float32)
    w = GemmWeights(ctx, b, 20, 24)  # host pointer path
    a = rng.uniform(-1, 1, (3, 20)).astype(np.float32)
    out = gemm_bias(ctx, torch.from_numpy(a).cuda(), w)
    ctx.synchronize()
    assert rel_err(out.cpu().numpy(), oracle.gemm(a, b)) <= TOL
    empty = gemm_bias(ctx, torch.zeros(0, 20, device="cuda"), w)
    assert empty.shape == (0, 24)


def test_gemm_rejects_mismatched_k(ctx):
    import torch

    from onnxsharp_b200 import OscError
    from onnxsharp_b200.runtime import GemmWeights, gemm_bias

    w = GemmWeights(ctx, torch.ones(8, 8, device="cuda"), 8, 8)
    with pytest.raises(OscError):
        gemm_bias(ctx, torch.ones(4, 9, device="cuda"), type("W", (), {"k": 9, "n": 8, "handle": w.handle})())


def test_gemm_split_once_three_weights(ctx):
    """One activation split once (osc_gemm_split_a_f32, strided rows, k not a
    multiple of 4) multiplied by three packed weights, as the Q/K/V
    projections of one input; each product equals the oracle's and the
    one-step entry point's results."""
    import torch

    from onnxsharp_b200 import OscError
    from onnxsharp_b200.runtime import GemmWeights, gemm_bias, gemm_bias_presplit, gemm_split_a

    rng = np.random.default_rng(11)
    m, k, lda = 700, 301, 320
    big = rng.uniform(-1, 1, (m, lda)).astype(np.float32)
    a = np.ascontiguousarray(big[:, :k])
    ta = torch.from_numpy(big).cuda()[:, :k]
    split = gemm_split_a(ctx, ta, k)
    assert split[0].shape == (m, 304)
    for n, act in ((512, 0), (96, 1), (1500, 0)):
        b = rng.uniform(-1, 1, (k, n)).astype(np.float32)
        bias = rng.uniform(-1, 1, n).astype(np.float32)
        w = GemmWeights(ctx, torch.from_numpy(b).cuda(), k, n)
        tb = torch.from_numpy(bias).cuda()
        got = gemm_bias_presplit(ctx, split, w, tb, act)
        one = gemm_bias(ctx, ta, w, tb, act, lda=lda)
        ctx.synchronize()
        assert rel_err(got.cpu().numpy(), oracle.gemm(a, b, col_bias=bias, act=act)) <= TOL
        assert torch.equal(got, one)
    w_small = GemmWeights(ctx, torch.ones(64, 8, device="cuda"), 64, 8)
    with pytest.raises(OscError, match="kp"):
        gemm_bias_presplit(ctx, split, w_small)
