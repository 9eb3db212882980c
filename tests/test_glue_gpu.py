"""Glue operators on the B200 against the oracle / exact numpy: direct conv
(first layer, depthwise), conv views + fused residual, MaxPool, nearest
Resize, broadcasting binary ops, unary activations, Softmax, DflSoftmax,
LayerNorm, the PSA attention and the fused YOLO decode."""
from __future__ import annotations

import numpy as np
import pytest

import oracle
from conftest import rel_err

pytestmark = pytest.mark.gpu


def T(a):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("C,M,k,s,group", [(3, 16, 3, 2, 1), (64, 64, 3, 1, 64), (80, 80, 3, 1, 80), (8, 16, 5, 2, 2)])
def test_conv_direct(ctx, C, M, k, s, group):
    import torch

    from onnxsharp_b200 import ops

    rng = np.random.default_rng(C + M + k)
    x = rng.uniform(0, 1, (2, C, 33, 30)).astype(np.float32)
    w = (rng.normal(0, 1, (M, C // group, k, k)) * np.sqrt(2 / (C // group * k * k))).astype(np.float32)
    b = rng.normal(0, 0.01, M).astype(np.float32)
    p = k // 2
    oh, ow = ops.out_size(33, k, s, p, p), ops.out_size(30, k, s, p, p)
    y = torch.empty(2, M, oh, ow, device="cuda")
    ops.conv2d_direct(ctx, T(x), T(w), T(b), y, s, p, 1, group, 1)
    ctx.synchronize()
    ref = oracle.conv2d(x, w, b, (s, s), (p, p, p, p), (1, 1), group, 1)
    assert rel_err(y.cpu().numpy(), ref) <= 1e-5


@pytest.mark.parametrize("C,k,s,H,W", [(16, 3, 2, 33, 30), (6, 5, 1, 150, 41), (4, 3, 1, 20, 700), (8, 7, 1, 70, 70)])
def test_conv_depthwise_geometries(ctx, C, k, s, H, W):
    """Depthwise bands: stride 2, 5x5 / 7x7, images taller than one 64-row band,
    rows wide enough to shrink the band to fit 48 KB of shared memory."""
    import torch

    from onnxsharp_b200 import ops

    rng = np.random.default_rng(C * k + H)
    x = rng.uniform(-1, 1, (2, C, H, W)).astype(np.float32)
    w = (rng.normal(0, 1, (C, 1, k, k)) * np.sqrt(2 / (k * k))).astype(np.float32)
    b = rng.normal(0, 0.01, C).astype(np.float32)
    p = k // 2
    oh, ow = ops.out_size(H, k, s, p, p), ops.out_size(W, k, s, p, p)
    y = torch.empty(2, C, oh, ow, device="cuda")
    ops.conv2d_direct(ctx, T(x), T(w), T(b), y, s, p, 1, C, 1)
    ctx.synchronize()
    ref = oracle.conv2d(x, w, b, (s, s), (p, p, p, p), (1, 1), C, 1)
    assert rel_err(y.cpu().numpy(), ref) <= 1e-5


@pytest.mark.parametrize("C,H,W,act,resid", [(80, 80, 80, 1, False), (7, 9, 100, 0, True), (128, 20, 20, 17, True),
                                                (5, 17, 99, 1, True)])
def test_conv_depthwise3_register_window(ctx, C, H, W, act, resid):
    """Depthwise 3x3 stride 1 (the register-window kernels; four columns per
    thread when W % 4 == 0, one otherwise): channel-slice views on input and
    output, partial row strips, fused residual, fast activation."""
    import torch

    from onnxsharp_b200 import ops

    rng = np.random.default_rng(C + H + W)
    x = rng.uniform(-1, 1, (3, C + 2, H, W)).astype(np.float32)
    w = (rng.normal(0, 1, (C, 1, 3, 3)) * np.sqrt(2 / 9)).astype(np.float32)
    b = rng.normal(0, 0.01, C).astype(np.float32)
    res = rng.normal(0, 1, (3, C, H, W)).astype(np.float32) if resid else None
    out_big = torch.zeros(3, C + 4, H, W, device="cuda")
    ops.conv2d_direct(ctx, T(x)[:, 2:], T(w), T(b), out_big[:, 4:], 1, 1, 1, C, act,
                      T(res) if resid else None)
    ctx.synchronize()
    ref = oracle.conv2d(np.ascontiguousarray(x[:, 2:]), w, b, (1, 1), (1, 1, 1, 1), (1, 1), C, act & 15)
    if resid:
        ref = res + ref
    got = out_big.cpu().numpy()
    assert rel_err(got[:, 4:], ref) <= (2e-6 if act & 16 else 1e-5)
    assert not got[:, :4].any()


@pytest.mark.parametrize(
    "C,M,k,s,H,W,resid",
    [
        (3, 16, 3, 2, 65, 64, False),   # stem: one partial channel chunk, odd rows
        (16, 8, 3, 1, 33, 30, False),   # 8 output channels, width not a multiple of 4
        (16, 32, 3, 2, 40, 40, False),  # stride 2, two full channel chunks
        (12, 80, 1, 1, 20, 24, False),  # 1x1, partial output-channel block
        (32, 16, 3, 1, 24, 36, True),   # fused residual
        (5, 24, 1, 2, 17, 19, False),   # 1x1 stride 2, ragged everything
    ],
)
def test_conv_tile_bit_exact(ctx, C, M, k, s, H, W, resid):
    """The register-blocked CUDA-core conv keeps the im2col FMA order per
    output (acc = bias, then (ic, ky, kx) ascending), so it reproduces the
    oracle's bits; channel-slice views on input and output."""
    import torch

    from onnxsharp_b200 import ops

    rng = np.random.default_rng(C * 7 + M + k + s)
    x = rng.uniform(0, 1, (2, C + 3, H, W)).astype(np.float32)
    w = (rng.normal(0, 1, (M, C, k, k)) * np.sqrt(2 / (C * k * k))).astype(np.float32)
    b = rng.normal(0, 0.01, M).astype(np.float32)
    p = k // 2
    oh, ow = ops.out_size(H, k, s, p, p), ops.out_size(W, k, s, p, p)
    res = rng.normal(0, 1, (2, M, oh, ow)).astype(np.float32) if resid else None
    out_big = torch.zeros(2, M + 4, oh, ow, device="cuda")
    dx = T(x)
    ops.conv2d_direct(ctx, dx[:, 2:2 + C], T(w), T(b), out_big[:, 4:], s, p, 1, 1, 1,
                      T(res) if resid else None)
    ctx.synchronize()
    ref = oracle.conv2d(np.ascontiguousarray(x[:, 2:2 + C]), w, b, (s, s), (p, p, p, p), (1, 1), 1, 1)
    if resid:
        ref = res + ref
    got = out_big.cpu().numpy()
    assert np.array_equal(got[:, 4:], ref)
    assert not got[:, :4].any()


@pytest.mark.parametrize("C,M,k,s,act", [(16, 32, 3, 2, 1), (32, 32, 1, 1, 1), (8, 16, 3, 1, 3)])
def test_conv_tile_fast_activation(ctx, C, M, k, s, act):
    """OSC_ACT_FAST: the same sums with the hardware-instruction SiLU/Sigmoid,
    within 2e-6 of the oracle's exact activation in |d| / max(1, |ref|)."""
    import torch

    from onnxsharp_b200 import _lib, ops

    rng = np.random.default_rng(C + M + k)
    x = rng.uniform(-2, 2, (2, C, 40, 40)).astype(np.float32)
    w = (rng.normal(0, 1, (M, C, k, k)) * np.sqrt(2 / (C * k * k))).astype(np.float32)
    b = rng.normal(0, 0.01, M).astype(np.float32)
    p = k // 2
    oh = ops.out_size(40, k, s, p, p)
    y = torch.empty(2, M, oh, oh, device="cuda")
    ops.conv2d_direct(ctx, T(x), T(w), T(b), y, s, p, 1, 1, act | _lib.ACT_FAST)
    ctx.synchronize()
    ref = oracle.conv2d(x, w, b, (s, s), (p, p, p, p), (1, 1), 1, act)
    assert rel_err(y.cpu().numpy(), ref) <= 2e-6


def test_conv_ex_views_and_residual(ctx):
    """Input and output are channel slices of larger buffers; y = res + SiLU(conv(x) + b)."""
    import torch

    from onnxsharp_b200 import ops
    from onnxsharp_b200.runtime import ConvWeights

    rng = np.random.default_rng(3)
    big_x = rng.uniform(0, 1, (2, 96, 20, 24)).astype(np.float32)
    w = (rng.normal(0, 0.1, (32, 48, 3, 3))).astype(np.float32)
    b = rng.normal(0, 0.01, 32).astype(np.float32)
    res = rng.normal(0, 1, (2, 32, 20, 24)).astype(np.float32)
    out_big = torch.zeros(2, 80, 20, 24, device="cuda")
    dx = T(big_x)
    ops.conv2d_ex(ctx, dx[:, 40:88], ConvWeights(ctx, T(w), w.shape), T(b), out_big[:, 16:48], 1, 1, 1, 1,
                  T(res))
    ctx.synchronize()
    ref = res + oracle.conv2d(np.ascontiguousarray(big_x[:, 40:88]), w, b, pads=(1, 1, 1, 1), act=1)
    got = out_big.cpu().numpy()
    assert rel_err(got[:, 16:48], ref) <= 1e-4
    assert not got[:, :16].any() and not got[:, 48:].any()  # nothing outside the slice


def test_maxpool_and_resize(ctx):
    import torch

    from onnxsharp_b200 import ops
    from oracle import yolo_ref

    rng = np.random.default_rng(4)
    x = rng.normal(0, 1, (2, 16, 20, 20)).astype(np.float32)
    y = torch.empty(2, 16, 20, 20, device="cuda")
    ops.maxpool2d(ctx, T(x), y, 5, 1, 2)
    z = torch.empty(2, 16, 40, 40, device="cuda")
    ops.resize_nearest(ctx, T(x), z, 2)
    ctx.synchronize()
    assert np.array_equal(y.cpu().numpy(), yolo_ref._maxpool(x, 5, 1, 2))
    assert np.array_equal(z.cpu().numpy(), np.repeat(np.repeat(x, 2, 2), 2, 3))


@pytest.mark.parametrize("shape,k,s,p", [((2, 5, 33, 47), 3, 2, 1), ((1, 3, 700, 9), 5, 1, 2), ((3, 2, 8, 8), 2, 2, 0),
                                         ((40, 7, 20, 20), 5, 1, 2), ((1, 2, 10, 300), 3, 1, 1), ((2, 3, 30, 30), 4, 2, 1)])
def test_maxpool_geometries(ctx, shape, k, s, p):
    """Odd sizes, stride 2, tall planes, planes packed several to a CTA (and a
    partial last CTA), rows wider than 256 and a 4x4 window (the generic
    kernel), and a channel slice of a wider buffer on both sides (SPPF's layout)."""
    import torch

    from onnxsharp_b200 import ops
    from oracle import yolo_ref

    rng = np.random.default_rng(sum(shape))
    n, c, h, w = shape
    big = rng.normal(0, 1, (n, c + 3, h, w)).astype(np.float32)
    x = np.ascontiguousarray(big[:, 1:1 + c])
    oh, ow = (h + 2 * p - k) // s + 1, (w + 2 * p - k) // s + 1
    out = torch.zeros(n, c + 2, oh, ow, device="cuda")
    ops.maxpool2d(ctx, T(big)[:, 1:1 + c], out[:, 2:], k, s, p)
    ctx.synchronize()
    got = out.cpu().numpy()
    assert np.array_equal(got[:, 2:], yolo_ref._maxpool(x, k, s, p))
    assert not got[:, :2].any()


@pytest.mark.parametrize("shape,scale,slice_out", [((2, 4, 7, 9), 2, False), ((1, 3, 5, 6), 3, False),
                                                   ((2, 6, 40, 40), 2, True), ((1, 2, 300, 302), 2, False)])
def test_resize_nearest_geometries(ctx, shape, scale, slice_out):
    """Odd widths and scale 3 take the scalar kernel; even widths the 2x one,
    also into a channel slice of a concatenation buffer."""
    import torch

    from onnxsharp_b200 import ops

    rng = np.random.default_rng(sum(shape) + scale)
    x = rng.normal(0, 1, shape).astype(np.float32)
    n, c, h, w = shape
    extra = 4 if slice_out else 0
    out = torch.zeros(n, c + extra, h * scale, w * scale, device="cuda")
    ops.resize_nearest(ctx, T(x), out[:, extra:], scale)
    ctx.synchronize()
    got = out.cpu().numpy()
    assert np.array_equal(got[:, extra:], np.repeat(np.repeat(x, scale, 2), scale, 3))
    assert not got[:, :extra].any()


@pytest.mark.parametrize("op,fn", [(0, np.add), (1, np.subtract), (2, np.multiply), (3, np.divide)])
def test_binary_broadcast(ctx, op, fn):
    import torch

    from onnxsharp_b200 import ops

    rng = np.random.default_rng(op)
    a = rng.normal(0, 1, (2, 3, 4, 5)).astype(np.float32)
    b = rng.uniform(0.5, 2, (3, 1, 5)).astype(np.float32)
    y = torch.empty(2, 3, 4, 5, device="cuda")
    ops.binary(ctx, op, T(a), T(b), y)
    ctx.synchronize()
    assert np.array_equal(y.cpu().numpy(), fn(a, b).astype(np.float32))


@pytest.mark.parametrize("act", [1, 2, 3])
def test_unary_bit_exact(ctx, act):
    import torch

    from onnxsharp_b200 import ops

    x = np.linspace(-30, 30, 10007, dtype=np.float32)
    y = torch.empty(10007, device="cuda")
    ops.unary(ctx, T(x), y, act)
    ctx.synchronize()
    assert np.array_equal(y.cpu().numpy(), oracle.unary(x, act))  # VectorMath restated bit-for-bit


@pytest.mark.parametrize("len_", [400, 16, 13, 1])
def test_softmax_rows(ctx, len_):
    import torch

    from onnxsharp_b200 import ops

    x = np.random.default_rng(len_).normal(0, 3, (37, len_)).astype(np.float32)
    y = torch.empty(37, len_, device="cuda")
    ops.softmax(ctx, T(x), y)
    ctx.synchronize()
    assert np.max(np.abs(y.cpu().numpy() - oracle.softmax(x))) <= 1e-7


def test_dfl(ctx, golden):
    import torch

    from onnxsharp_b200 import ops

    x = golden["dfl_x"]
    y = torch.empty(x.shape[0], 4, x.shape[2], device="cuda")
    ops.dfl(ctx, T(x), y)
    ctx.synchronize()
    assert np.max(np.abs(y.cpu().numpy() - golden["dfl_y"])) <= 1e-6


def test_layernorm(ctx, golden):
    import torch

    from onnxsharp_b200 import ops

    y = torch.empty(golden["ln_x"].shape, device="cuda")
    ops.layernorm(ctx, T(golden["ln_x"]), T(golden["ln_g"]), T(golden["ln_b"]), 1e-5, y)
    ctx.synchronize()
    assert np.max(np.abs(y.cpu().numpy() - golden["ln_y"])) <= 1e-6


@pytest.mark.parametrize("B,heads,kd,hd,h,w,extra", [
    (2, 2, 32, 64, 20, 20, 0),    # YOLO11n's C2PSA at 640x640: fused kernel, 16-query blocks
    (32, 2, 32, 64, 20, 20, 8),   # fused, 64-query blocks, qkv a channel slice
    (1, 2, 32, 64, 13, 11, 0),    # fused, T = 143: softmax tail, padded P / V rows
    (1, 1, 32, 64, 23, 22, 0),    # fused, T = 506 (the largest row the softmax registers hold is 512)
    (3, 1, 16, 32, 7, 9, 0),      # other head shape (T = 63): tensor-core path, padded K, unaligned rows
    (1, 4, 32, 64, 40, 40, 24),   # T = 1600: tensor-core path, qkv a channel slice of a wider buffer
])
def test_psa_attention(ctx, B, heads, kd, hd, h, w, extra):
    """PSA attention (one fused kernel for YOLO11's head shape, the tensor-core
    composed path otherwise) against the oracle's MatMul -> Mul -> Softmax ->
    MatMul chain at the FP32 tolerance |d| / max(1, |ref|) <= 1e-4."""
    import torch

    from onnxsharp_b200 import ops
    from oracle import yolo_ref

    c = heads * (2 * kd + hd)
    big = np.random.default_rng(9 + h).normal(0, 1, (B, c + extra, h, w)).astype(np.float32)
    qkv = np.ascontiguousarray(big[:, extra:])
    out = torch.empty(B, heads * hd, h, w, device="cuda")
    ops.psa_attention(ctx, T(big)[:, extra:], out, heads, kd, hd, kd ** -0.5)
    ctx.synchronize()
    ref = yolo_ref._psa(qkv, heads, kd, hd, kd ** -0.5, 0)
    assert rel_err(out.cpu().numpy(), ref) <= 1e-4


def test_yolo_decode(ctx):
    import torch

    from onnxsharp_b200 import ops
    from oracle import yolo_ref

    rng = np.random.default_rng(10)
    boxes = [rng.normal(0, 2, (2, 64, n, n)).astype(np.float32) for n in (80, 40, 20)]
    cls = [rng.normal(0, 2, (2, 80, n, n)).astype(np.float32) for n in (80, 40, 20)]
    out = torch.empty(2, 84, 8400, device="cuda")
    ops.yolo_decode(ctx, [T(b) for b in boxes], [T(c) for c in cls], (8, 16, 32), out)
    ctx.synchronize()
    ref = yolo_ref._decode(boxes, cls, (8, 16, 32), 0)
    got = out.cpu().numpy()
    assert np.max(np.abs(got[:, :4] - ref[:, :4])) <= 1e-4
    assert np.array_equal(got[:, 4:], ref[:, 4:])
