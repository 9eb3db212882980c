"""The unfused int8 operators on the B200: DynamicQuantizeLinear and
MatMulInteger (the graphs that QuantizedMatMul fusion does not catch),
bit-exact against the oracle and the reference's known answers
(QuantOpsTests.cs:40-76, Int8Tests.cs:286-326)."""
from __future__ import annotations

import json

import numpy as np
import pytest

import oracle
from conftest import GOLDEN

pytestmark = pytest.mark.gpu
KAT = json.loads((GOLDEN / "kat.json").read_text())


def T(a):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _dql(ctx, x):
    from onnxsharp_b200.runtime import dynamic_quantize_linear

    y, s, z = dynamic_quantize_linear(ctx, T(x))
    ctx.synchronize()
    return y.cpu().numpy(), float(s.cpu().numpy()[0]), int(z.cpu().numpy()[0])


def _dql_ref(x):
    mn, mx = oracle.minmax(x)
    scale, zp = oracle.dql_params(mn, mx)
    return oracle.quantize_u8(x, scale, zp), scale, zp


def test_dql_known_answer(ctx):
    k = KAT["dynamic_quantize_linear"]
    y, s, z = _dql(ctx, np.array(k["x"], np.float32))
    assert abs(s - k["scale"]) <= k["scale_tol"] and z == k["zero_point"]
    assert y.tolist() == k["q"]


@pytest.mark.parametrize("case", ["normal", "positive", "negative", "zeros", "nan", "odd"])
def test_dql_matches_oracle(ctx, case):
    rng = np.random.default_rng(len(case))
    n = 3 * 1000003 if case == "odd" else 1 << 20
    x = rng.normal(0, 3, n).astype(np.float32)
    if case == "positive":
        x = np.abs(x) + 0.5
    elif case == "negative":
        x = -np.abs(x) - 0.5
    elif case == "zeros":
        x[:] = 0
    elif case == "nan":
        x[rng.integers(0, n, 100)] = np.nan
    y, s, z = _dql(ctx, x)
    ry, rs, rz = _dql_ref(x)
    assert np.float32(s) == np.float32(rs) and z == rz
    assert np.array_equal(y, ry)


def _mmi(ctx, a, a_zp, w, w_zp, lda_pad=0):
    import torch

    from onnxsharp_b200.runtime import DqmmWeights, matmul_integer

    m, k = a.shape
    n = w.shape[1]
    W = DqmmWeights(ctx, T(w), k, n, w_zp)
    ta = T(a)
    if lda_pad:
        big = torch.zeros((m, k + lda_pad), dtype=ta.dtype, device="cuda")
        big[:, :k] = ta
        ta = big[:, :k]
    y = matmul_integer(ctx, ta, a_zp, W)
    ctx.synchronize()
    return y.cpu().numpy()


def test_matmul_integer_known_answer(ctx):
    k = KAT["matmul_integer"]
    y = _mmi(ctx, np.array(k["a"], np.uint8), 0, np.array(k["b"], np.uint8), None)
    assert y.tolist() == k["c"]


@pytest.mark.parametrize("m,k,n,a_signed,w_signed,zp,lda_pad", [
    (37, 100, 50, False, True, "col", 0),       # k not a multiple of 16 (pitched copy), n % 4 != 0
    (130, 256, 300, False, False, "tensor", 0),  # u8 x u8, per-tensor zero point
    (64, 1280, 32, False, True, "col", 0),      # the Int8Tests exactness shape
    (200, 512, 256, True, True, None, 16),       # s8 activations, strided rows read in place
    (1024, 512, 2048, False, True, "col", 0),   # large: persistent tiles, TMA stores
])
def test_matmul_integer_matches_oracle(ctx, m, k, n, a_signed, w_signed, zp, lda_pad):
    rng = np.random.default_rng(m + k + n)
    a = rng.integers(-128, 128, (m, k)).astype(np.int8) if a_signed else rng.integers(0, 256, (m, k)).astype(np.uint8)
    w = rng.integers(-128, 128, (k, n)).astype(np.int8) if w_signed else rng.integers(0, 256, (k, n)).astype(np.uint8)
    if zp == "col":
        w_zp = rng.integers(-20, 21, n).astype(np.int32) if w_signed else rng.integers(100, 156, n).astype(np.int32)
    elif zp == "tensor":
        w_zp = np.int32(128)
    else:
        w_zp = None
    a_zp = -3 if a_signed else 121
    got = _mmi(ctx, a, a_zp, w, w_zp, lda_pad)
    ref = oracle.matmul_integer(a, a_zp, w, 0 if w_zp is None else w_zp)
    assert np.array_equal(got, ref)


def test_matmul_integer_rejects_bad_zero_point(ctx):
    from onnxsharp_b200._lib import OscError

    with pytest.raises(OscError):
        _mmi(ctx, np.zeros((4, 16), np.uint8), 300, np.zeros((16, 8), np.int8), None)
