"""The CPU oracle pinned against the reference's own known-answer vectors and
invariants (tests/golden/kat.json, transcribed from the reference test
sources), plus float64 checks at the reference's tolerances."""
from __future__ import annotations

import json
import math

import numpy as np
import pytest

import oracle
from conftest import GOLDEN, rel_err

KAT = json.loads((GOLDEN / "kat.json").read_text())


def test_dynamic_quantize_linear_kat():
    k = KAT["dynamic_quantize_linear"]
    x = np.array(k["x"], np.float32)
    scale, zp = oracle.dql_params(*oracle.minmax(x))
    assert abs(scale - k["scale"]) <= k["scale_tol"]
    assert zp == k["zero_point"]
    assert oracle.quantize_u8(x, scale, zp).tolist() == k["q"]


def test_quantize_u8_kat_round_half_even_and_saturation():
    k = KAT["quantize_u8"]
    q = oracle.quantize_u8(np.array(k["x"], np.float32), k["scale"], k["zero_point"])
    assert q.tolist() == k["q"]
    s = oracle.quantize_u8(np.array([k["saturate_x"]], np.float32), k["scale"], k["zero_point"])
    assert int(s[0]) == k["saturate_q"]


def test_matmul_integer_kat():
    k = KAT["matmul_integer"]
    c = oracle.matmul_integer(np.array(k["a"], np.uint8), 0, np.array(k["b"], np.uint8), 0)
    assert c.tolist() == k["c"]


def test_minmax_includes_zero_and_skips_nan():
    assert oracle.minmax(np.array([1.0, 2.0, 3.0], np.float32)) == (0.0, 3.0)
    assert oracle.minmax(np.array([-4.0, np.nan, -1.0], np.float32)) == (-4.0, 0.0)


def test_dql_degenerate_scale_is_one():
    assert oracle.dql_params(0.0, 0.0) == (1.0, 0)


def test_f32_substitute_exact_at_long_k():
    """Int8Tests.cs:286-326: widened-int8 F32 accumulation equals the int32 sum."""
    k = KAT["int8_f32_substitute_exact"]
    rng = np.random.default_rng(2026)
    a = rng.integers(0, 256, (k["m"], k["k"])).astype(np.uint8)
    w = (rng.integers(0, 256, (k["k"], k["n"])) - 128).astype(np.int8)
    wz = rng.integers(k["w_zero_range"][0], k["w_zero_range"][1], k["n"]).astype(np.int32)
    exact = oracle.matmul_integer(a, k["a_zero"], w, wz)
    af = (a.astype(np.float32) - k["a_zero"])
    wf = (w.astype(np.float32) - wz[None, :].astype(np.float32))
    got = oracle.gemm(af, wf)
    assert np.array_equal(got.astype(np.int64), exact.astype(np.int64))


@pytest.mark.parametrize("shape", KAT["gemm_tolerance"]["naive_shapes"])
def test_gemm_matches_naive_double(shape):
    m, k, n = shape
    rng = np.random.default_rng(m * 31 + k * 7 + n)
    a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
    b = rng.uniform(-1, 1, (k, n)).astype(np.float32)
    ref = a.astype(np.float64) @ b.astype(np.float64)
    assert rel_err(oracle.gemm(a, b), ref) <= KAT["gemm_tolerance"]["vs_naive_double"]


@pytest.mark.parametrize("shape", KAT["gemm_tolerance"]["column_bias_shapes"])
def test_gemm_column_bias(shape):
    m, k, n = shape
    rng = np.random.default_rng(m + k * 13 + n * 7)
    a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
    b = rng.uniform(-1, 1, (k, n)).astype(np.float32)
    bias = rng.uniform(-1, 1, n).astype(np.float32)
    ref = a.astype(np.float64) @ b.astype(np.float64) + bias
    assert rel_err(oracle.gemm(a, b, col_bias=bias), ref) <= 1e-4


@pytest.mark.parametrize("shape", KAT["gemm_tolerance"]["scale_bias_shapes"])
def test_gemm_scale_bias_epilogue(shape):
    """GemmKernelTests.cs:57-104: fused scale+bias within 1e-5 of plain*scale+bias."""
    m, k, n = shape
    rng = np.random.default_rng(m * 13 + k * 29 + n * 11)
    a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
    b = rng.uniform(-1, 1, (k, n)).astype(np.float32)
    scale = (0.0001 + rng.uniform(0, 1, n) * 0.01).astype(np.float32)
    bias = rng.uniform(-1, 1, n).astype(np.float32)
    plain = oracle.gemm(a, b)
    fused = oracle.gemm(a, b, col_bias=bias, col_scale=scale)
    expected = plain.astype(np.float64) * scale + bias
    assert rel_err(fused, expected) <= KAT["gemm_tolerance"]["kernel_vs_kernel"]


def test_gemm_thread_count_invariant():
    rng = np.random.default_rng(5)
    a = rng.uniform(-1, 1, (97, 130)).astype(np.float32)
    b = rng.uniform(-1, 1, (130, 75)).astype(np.float32)
    assert np.array_equal(oracle.gemm(a, b, threads=1), oracle.gemm(a, b, threads=4))


def test_exp_polynomial_accuracy_and_clamp():
    xs = np.linspace(-80, 80, 2001, dtype=np.float32)
    got = np.array([oracle.exp(float(x)) for x in xs])
    ref = np.exp(xs.astype(np.float64))
    assert np.max(np.abs(got - ref) / ref) < 5e-7
    assert oracle.exp(-1000.0) == pytest.approx(math.exp(-87.3), rel=1e-6)  # clamp to -87.3
    assert math.isinf(oracle.exp(88.5))  # n rounds to 128: 2^128 overflows, as in VectorMath.Exp


def test_silu_matches_definition():
    xs = np.linspace(-20, 20, 401, dtype=np.float32)
    got = oracle.unary(xs, 1)
    ref = xs.astype(np.float64) / (1 + np.exp(-xs.astype(np.float64)))
    assert np.max(np.abs(got - ref) / np.maximum(1, np.abs(ref))) < 1e-6


def test_dqmm_exact_integer_accumulator_and_quantized_values():
    rng = np.random.default_rng(3)
    a = rng.normal(0, 1, (29, 96)).astype(np.float32)
    w = rng.integers(-127, 128, (96, 40)).astype(np.int8)
    ws = rng.uniform(0.001, 0.02, 40).astype(np.float32)
    bias = rng.normal(0, 0.01, 40).astype(np.float32)
    y, q, acc, (s, z) = oracle.dqmm(a, w, 0, ws, bias)
    mn, mx = oracle.minmax(a)
    assert (s, z) == oracle.dql_params(mn, mx)
    assert np.array_equal(q, oracle.quantize_u8(a, s, z))
    exact = oracle.matmul_integer(q, z, w, 0)
    assert np.array_equal(acc, exact)
    ref = exact.astype(np.float64) * (np.float64(s) * ws.astype(np.float64)) + bias
    assert rel_err(y, ref) <= 1e-5


def test_conv_matches_float64_direct():
    rng = np.random.default_rng(11)
    x = rng.uniform(0, 1, (2, 6, 9, 10)).astype(np.float32)
    w = rng.normal(0, 0.3, (8, 3, 3, 3)).astype(np.float32)
    b = rng.normal(0, 0.01, 8).astype(np.float32)
    y = oracle.conv2d(x, w, b, stride=(2, 1), pads=(1, 0, 1, 2), group=2)
    # float64 direct convolution
    xp = np.pad(x.astype(np.float64), ((0, 0), (0, 0), (1, 1), (0, 2)))
    N, C, H, W = x.shape
    OH, OW = y.shape[2:]
    ref = np.zeros(y.shape)
    for g in range(2):
        for o in range(4):
            oc = g * 4 + o
            for ic in range(3):
                for ky in range(3):
                    for kx in range(3):
                        patch = xp[:, g * 3 + ic, ky:ky + 2 * OH:2, kx:kx + OW]
                        ref[:, oc] += w[oc, ic, ky, kx] * patch[:, :OH, :OW]
            ref[:, oc] += b[oc]
    assert rel_err(y, ref) < 1e-5


def _conv64(x, w, b, s, p):
    """float64 direct convolution, group 1, square stride s and padding p."""
    N, C, H, W = x.shape
    M, _, k, _ = w.shape
    xp = np.pad(x.astype(np.float64), ((0, 0), (0, 0), (p, p), (p, p)))
    OH, OW = (H + 2 * p - k) // s + 1, (W + 2 * p - k) // s + 1
    ref = np.zeros((N, M, OH, OW)) + b.astype(np.float64)[None, :, None, None]
    for ky in range(k):
        for kx in range(k):
            patch = xp[:, :, ky:ky + s * (OH - 1) + 1:s, kx:kx + s * (OW - 1) + 1:s]
            ref += np.einsum("nchw,mc->nmhw", patch, w[:, :, ky, kx].astype(np.float64))
    return ref


@pytest.mark.parametrize("C,M,H,W,k,s,p", [
    (40, 24, 20, 20, 1, 1, 0),    # 1x1: the blocked GEMM straight on the image
    (16, 20, 20, 44, 3, 1, 1),    # narrow rows: whole-image columns times the GEMM
    (12, 18, 9, 80, 3, 2, 1),     # 40-wide output rows (stride 2): whole-image columns
    (8, 14, 6, 128, 3, 1, 1),     # 128-wide rows: the row-at-a-time path
    (5, 7, 5, 64, 5, 1, 2),       # 64-wide rows, 5x5
])
def test_conv_paths_match_float64(C, M, H, W, k, s, p):
    """Every group-1 conv route of the oracle (1x1 GEMM, whole-image columns,
    row at a time) against a float64 convolution."""
    rng = np.random.default_rng(C * 100 + W)
    x = rng.uniform(-1, 1, (2, C, H, W)).astype(np.float32)
    w = rng.normal(0, 0.3, (M, C, k, k)).astype(np.float32)
    b = rng.normal(0, 0.1, M).astype(np.float32)
    y = oracle.conv2d(x, w, b, stride=(s, s), pads=(p, p, p, p))
    assert rel_err(y, _conv64(x, w, b, s, p)) < 1e-5


def _attn_ref(q, k, v, heads, scale):
    B, T, Cw = q.shape
    D = Cw // heads
    qh = q.reshape(B, T, heads, D).transpose(0, 2, 1, 3).astype(np.float64)
    kh = k.reshape(B, T, heads, D).transpose(0, 2, 1, 3).astype(np.float64)
    vh = v.reshape(B, T, heads, D).transpose(0, 2, 1, 3).astype(np.float64)
    s = (qh * scale) @ kh.transpose(0, 1, 3, 2)
    s = np.exp(s - s.max(-1, keepdims=True))
    p = s / s.sum(-1, keepdims=True)
    return (p @ vh).transpose(0, 2, 1, 3).reshape(B, T, Cw)


@pytest.mark.parametrize("T", [40, 128])
def test_attention_matches_float64(T):
    rng = np.random.default_rng(T)
    q, k, v = (rng.normal(0, 1, (2, T, 64)).astype(np.float32) for _ in range(3))
    got = oracle.attention(q, k, v, heads=4, scale=0.25)
    assert np.max(np.abs(got - _attn_ref(q, k, v, 4, 0.25))) < 1e-5


def test_dfl_matches_float64():
    rng = np.random.default_rng(1)
    x = rng.normal(0, 2, (1, 64, 77)).astype(np.float32)
    got = oracle.dfl(x)
    xr = x.reshape(1, 4, 16, 77).astype(np.float64)
    p = np.exp(xr - xr.max(2, keepdims=True))
    p /= p.sum(2, keepdims=True)
    ref = (p * np.arange(16)[None, None, :, None]).sum(2)
    assert np.max(np.abs(got - ref)) < 1e-5


def test_layernorm_matches_float64():
    rng = np.random.default_rng(2)
    x = rng.normal(0, 1, (7, 37)).astype(np.float32)
    g = rng.normal(1, 0.1, 37).astype(np.float32)
    b = rng.normal(0, 0.1, 37).astype(np.float32)
    got = oracle.layernorm(x, g, b)
    xd = x.astype(np.float64)
    ref = (xd - xd.mean(-1, keepdims=True)) / np.sqrt(xd.var(-1, keepdims=True) + 1e-5) * g + b
    assert np.max(np.abs(got - ref)) < 1e-5


def test_golden_fixture_is_reproducible(golden):
    """The committed oracle outputs still match the oracle (catches silent oracle drift)."""
    g = golden
    assert np.array_equal(oracle.gemm(g["gemm_a"], g["gemm_b"], col_bias=g["gemm_bias"], threads=1), g["gemm_c"])
    y, q, acc, (s, z) = oracle.dqmm(g["dqmm_a"], g["dqmm_w"], 0, g["dqmm_wscale"], g["dqmm_bias"], threads=1)
    assert np.array_equal(y, g["dqmm_y"]) and np.array_equal(q, g["dqmm_q"]) and np.array_equal(acc, g["dqmm_acc"])
    assert np.array_equal(oracle.conv2d(g["conv_x"], g["conv_w"], g["conv_b"], pads=(1, 1, 1, 1), act=1, threads=1),
                          g["conv_y"])
    assert np.array_equal(oracle.attention(g["attn_q"], g["attn_k"], g["attn_v"], heads=2, scale=0.25, threads=1),
                          g["attn_o"])
    assert np.array_equal(oracle.dfl(g["dfl_x"], 16, threads=1), g["dfl_y"])
    assert np.array_equal(oracle.layernorm(g["ln_x"], g["ln_g"], g["ln_b"], 1e-5, threads=1), g["ln_y"])
