"""DynamicQuantizeMatMul on the B200 integer tensor cores against the oracle:
bit-exact quantised values, int32 accumulators, scale/zero point and FP32
outputs (the reference's own rounding, QuantizedMatMulOps.cs:115-201)."""
from __future__ import annotations

import json

import numpy as np
import pytest

import oracle
from conftest import GOLDEN

pytestmark = pytest.mark.gpu
KAT = json.loads((GOLDEN / "kat.json").read_text())


def _run(ctx, a, w, w_zp, w_scale, bias, minmax_override=None):
    import torch

    from onnxsharp_b200.runtime import DqmmWeights, dqmm

    m, k = a.shape
    n = w.shape[1]
    W = DqmmWeights(ctx, torch.from_numpy(w).cuda(), k, n, w_zp)
    ta = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    q = torch.empty((m, k), dtype=torch.uint8, device="cuda")
    acc = torch.empty((m, n), dtype=torch.int32, device="cuda")
    params = torch.empty(2, dtype=torch.float32, device="cuda")
    y = dqmm(ctx, ta, W, torch.from_numpy(np.atleast_1d(w_scale).astype(np.float32)).cuda(),
             None if bias is None else torch.from_numpy(bias).cuda(), minmax_override=minmax_override, q_out=q,
             acc_out=acc, params_out=params)
    ctx.synchronize()
    return y.cpu().numpy(), q.cpu().numpy(), acc.cpu().numpy(), params.cpu().numpy()


def _check(got, ref):
    y, q, acc, params = got
    ry, rq, racc, (rs, rz) = ref
    assert params[0] == np.float32(rs) and int(params[1]) == rz
    assert np.array_equal(q, rq)
    assert np.array_equal(acc, racc)
    assert np.array_equal(y.view(np.uint32), ry.view(np.uint32)), "y not bit-identical"


def _config3(seed=3):
    rng = np.random.default_rng(seed)
    a = rng.normal(0, 1, (4096, 512)).astype(np.float32)
    w = rng.integers(-127, 128, (512, 2048)).astype(np.int8)
    ws = rng.uniform(0.001, 0.02, 2048).astype(np.float32)
    b = rng.normal(0, 0.01, 2048).astype(np.float32)
    return a, w, ws, b


def test_dqmm_config3_bit_exact(ctx):
    """A[4096,512] N(0,1), W int8 U[-127,127], per-column scales, bias."""
    a, w, ws, b = _config3()
    _check(_run(ctx, a, w, 0, ws, b), oracle.dqmm(a, w, 0, ws, b))


def test_dqmm_without_debug_outputs_same_y(ctx):
    """The serving call (no q / acc / params outputs) gives the same y bits."""
    import torch

    from onnxsharp_b200.runtime import DqmmWeights, dqmm

    a, w, ws, b = _config3(4)
    y_dbg = _run(ctx, a, w, 0, ws, b)[0]
    W = DqmmWeights(ctx, torch.from_numpy(w).cuda(), 512, 2048, 0)
    y = dqmm(ctx, torch.from_numpy(a).cuda(), W, torch.from_numpy(ws).cuda(), torch.from_numpy(b).cuda())
    ctx.synchronize()
    assert np.array_equal(y.cpu().numpy().view(np.uint32), y_dbg.view(np.uint32))


def test_dqmm_golden_fixture_ragged(ctx, golden):
    g = golden
    got = _run(ctx, g["dqmm_a"], g["dqmm_w"], 0, g["dqmm_wscale"], g["dqmm_bias"])
    y, q, acc, params = got
    assert np.array_equal(q, g["dqmm_q"]) and np.array_equal(acc, g["dqmm_acc"])
    assert params[0] == g["dqmm_params"][0] and params[1] == g["dqmm_params"][1]
    assert np.array_equal(y.view(np.uint32), g["dqmm_y"].view(np.uint32))


def test_dqmm_dql_kat(ctx):
    """QuantOpsTests.cs:40-50 through the fused op: scale 3/255, zp 85, q [0,85,170,255]."""
    kat = KAT["dynamic_quantize_linear"]
    a = np.array([kat["x"]], np.float32)
    w = np.ones((4, 16), np.int8)
    y, q, acc, params = _run(ctx, a, w, 0, np.float32(1.0), None)
    assert abs(params[0] - kat["scale"]) <= kat["scale_tol"] and int(params[1]) == kat["zero_point"]
    assert q[0].tolist() == kat["q"]
    assert acc[0, 0] == sum(v - kat["zero_point"] for v in kat["q"])


@pytest.mark.parametrize("m,k,n,signed,zp", [
    (37, 64, 50, True, None),          # tails in both directions
    (100, 256, 300, False, "col"),     # uint8 weights, per-column zero points
    (5, 1280, 32, True, "tensor"),     # long k (Int8Tests F32-substitute shape), per-tensor zero point
    (130, 100, 17, False, "tensor"),   # k not a multiple of 128, n < 16 tail
])
def test_dqmm_weight_kinds(ctx, m, k, n, signed, zp):
    rng = np.random.default_rng(m + k + n)
    a = rng.normal(0, 2, (m, k)).astype(np.float32)
    if signed:
        w = rng.integers(-128, 128, (k, n)).astype(np.int8)
    else:
        w = rng.integers(0, 256, (k, n)).astype(np.uint8)
    zps = None if zp is None else (rng.integers(100, 156, n).astype(np.int32) if zp == "col" else np.int32(128 if not signed else 3))
    ws = rng.uniform(0.001, 0.02, n).astype(np.float32)
    b = rng.normal(0, 0.01, n).astype(np.float32)
    _check(_run(ctx, a, w, zps, ws, b), oracle.dqmm(a, w, 0 if zps is None else zps, ws, b))


def test_dqmm_scalar_scale_no_bias_all_positive(ctx):
    rng = np.random.default_rng(21)
    a = rng.uniform(0.5, 3.0, (64, 96)).astype(np.float32)  # min clamps to 0 -> zp 0
    w = rng.integers(-127, 128, (96, 48)).astype(np.int8)
    _check(_run(ctx, a, w, 0, np.float32(0.01), None), oracle.dqmm(a, w, 0, np.float32(0.01), None))


def test_dqmm_all_zero_input_scale_one(ctx):
    a = np.zeros((8, 32), np.float32)
    w = np.ones((32, 16), np.int8)
    y, q, acc, params = _run(ctx, a, w, 0, np.float32(0.5), None)
    assert params.tolist() == [1.0, 0.0] and not q.any() and not acc.any() and not y.any()


def test_dqmm_nan_row_propagates_only_to_its_row(ctx):
    rng = np.random.default_rng(22)
    a = rng.normal(0, 1, (20, 64)).astype(np.float32)
    a[3, 10] = np.nan
    w = rng.integers(-127, 128, (64, 32)).astype(np.int8)
    ws = rng.uniform(0.001, 0.02, 32).astype(np.float32)
    y, q, acc, params = _run(ctx, a, w, 0, ws, None)
    ry, _, _, (rs, rz) = oracle.dqmm(np.delete(a, 3, axis=0), w, 0, ws, None)
    assert np.isnan(y[3]).all()
    assert params[0] == rs and int(params[1]) == rz  # NaN skipped by MinMax
    assert not np.isnan(np.delete(y, 3, axis=0)).any()


def test_dqmm_row_shards_with_global_range_match_whole(ctx):
    """The multi-GPU recipe: shards quantise with the all-reduced range and
    reproduce the single-tensor result bit-exactly (before the epilogue row
    grouping, which is per call: compare q and acc, and y on grouped-aligned
    shards)."""
    import torch

    from onnxsharp_b200.runtime import minmax

    a, w, ws, b = _config3(5)
    whole = _run(ctx, a, w, 0, ws, b)
    mm = minmax(ctx, torch.from_numpy(a).cuda())
    ctx.synchronize()
    parts = [_run(ctx, a[i:i + 1024], w, 0, ws, b, minmax_override=mm) for i in range(0, 4096, 1024)]
    assert np.array_equal(np.concatenate([p[1] for p in parts]), whole[1])
    assert np.array_equal(np.concatenate([p[2] for p in parts]), whole[2])
    y = np.concatenate([p[0] for p in parts])
    # 1024-row shards: the 12/6/4 row grouping leaves 1024 = 12*85 + 4 -> all rows fused, as in the whole tensor
    assert np.array_equal(y.view(np.uint32), whole[0].view(np.uint32))


def test_dqmm_row_shards_bit_exact_with_global_range(ctx):
    """osc_dqmm_shard_f32 on one GPU: A split into uneven row shards, each
    quantised with the whole tensor's range and classified by its rows' index
    in the whole tensor, reproduces q, the int32 accumulators and y of the
    unsharded oracle bit for bit (the reference's FMA / mul+add epilogue
    boundary at the 12/6/4-row groups falls inside a shard here)."""
    import torch

    from onnxsharp_b200.runtime import DqmmWeights, dqmm, minmax

    rng = np.random.default_rng(61)
    m, k, n = 1027, 256, 384  # whole-matrix groups cover rows < 1026; row 1026 is a leftover row
    a = rng.normal(0, 1, (m, k)).astype(np.float32)
    w = rng.integers(-127, 128, (k, n)).astype(np.int8)
    ws = rng.uniform(0.001, 0.02, n).astype(np.float32)
    b = rng.normal(0, 0.01, n).astype(np.float32)
    ry, rq, racc, _ = oracle.dqmm(a, w, 0, ws, b)
    W = DqmmWeights(ctx, torch.from_numpy(w).cuda(), k, n, 0)
    ta = torch.from_numpy(a).cuda()
    mm = minmax(ctx, ta)
    tws, tb = torch.from_numpy(ws).cuda(), torch.from_numpy(b).cuda()
    for lo, hi in [(0, 515), (515, 1025), (1025, 1027)]:
        q = torch.empty((hi - lo, k), dtype=torch.uint8, device="cuda")
        acc = torch.empty((hi - lo, n), dtype=torch.int32, device="cuda")
        y = dqmm(ctx, ta[lo:hi], W, tws, tb, minmax_override=mm, q_out=q, acc_out=acc, row0=lo, rows_total=m)
        ctx.synchronize()
        assert np.array_equal(q.cpu().numpy(), rq[lo:hi])
        assert np.array_equal(acc.cpu().numpy(), racc[lo:hi])
        assert np.array_equal(y.cpu().numpy().view(np.uint32), ry[lo:hi].view(np.uint32)), (lo, hi)
