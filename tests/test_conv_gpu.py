"""Conv(+bias, +fused SiLU) on the B200 tensor cores (implicit GEMM, 3xTF32)
against the CPU oracle's restatement of the reference im2col conv
(Kernels/ConvKernels.cs:262-462), tolerance |d| / max(1, |ref|) <= 1e-4."""
from __future__ import annotations

import numpy as np
import pytest

import oracle
from conftest import rel_err

pytestmark = pytest.mark.gpu
TOL = 1e-4


def _conv(ctx, x, w, b=None, stride=(1, 1), pads=(0, 0, 0, 0), dil=(1, 1), act=0):
    import torch

    from onnxsharp_b200.runtime import ConvWeights, conv2d

    cw = ConvWeights(ctx, torch.from_numpy(w).cuda(), w.shape)
    y = conv2d(ctx, torch.from_numpy(x).cuda(), cw, None if b is None else torch.from_numpy(b).cuda(), stride, pads,
               dil, 1, act)
    ctx.synchronize()
    return y.cpu().numpy()


def _case(seed, N, C, H, W, M, k, std=None):
    rng = np.random.default_rng(seed)
    x = rng.uniform(0, 1, (N, C, H, W)).astype(np.float32)
    fan = C * k * k
    w = (rng.normal(0, 1, (M, C, k, k)) * (std or np.sqrt(2.0 / fan))).astype(np.float32)
    b = rng.normal(0, 0.01, M).astype(np.float32)
    return x, w, b


def test_conv_golden_fixture(ctx, golden):
    g = golden
    y = _conv(ctx, g["conv_x"], g["conv_w"], g["conv_b"], pads=(1, 1, 1, 1), act=1)
    assert rel_err(y, g["conv_y"]) <= TOL


def test_conv_config2_batch1_full_spatial(ctx):
    """BASELINE config 2 at B=1: [1,64,160,160] -> [1,128,160,160], 3x3 s1 p1, SiLU."""
    x, w, b = _case(2, 1, 64, 160, 160, 128, 3)
    y = _conv(ctx, x, w, b, pads=(1, 1, 1, 1), act=1)
    assert rel_err(y, oracle.conv2d(x, w, b, pads=(1, 1, 1, 1), act=1)) <= TOL


def test_conv_config2_batch16_all_images(ctx):
    """BASELINE config 2 at B=16: every image checked against the oracle."""
    x, w, b = _case(3, 16, 64, 160, 160, 128, 3)
    y = _conv(ctx, x, w, b, pads=(1, 1, 1, 1), act=1)
    ref = oracle.conv2d(x, w, b, pads=(1, 1, 1, 1), act=1)
    for i in range(16):
        assert rel_err(y[i], ref[i]) <= TOL, f"image {i}"


@pytest.mark.parametrize(
    "N,C,H,W,M,k,stride,pads,dil,act",
    [
        (2, 3, 33, 35, 16, 3, 2, (1, 1, 1, 1), 1, 1),      # stem-like: C=3, stride 2
        (1, 16, 40, 40, 32, 3, 2, (1, 1, 1, 1), 1, 1),     # stride 2
        (2, 48, 20, 20, 200, 1, 1, (0, 0, 0, 0), 1, 0),    # 1x1, M > 128 and not a multiple
        (1, 32, 21, 19, 64, 3, 1, (1, 0, 2, 1), 1, 2),     # asymmetric pads, ReLU
        (1, 32, 24, 24, 32, 3, 1, (2, 2, 2, 2), 2, 3),     # dilation 2, Sigmoid
        (3, 64, 9, 7, 96, 5, 1, (2, 2, 2, 2), 1, 1),       # 5x5, tiny spatial
        (1, 256, 20, 20, 256, 3, 1, (1, 1, 1, 1), 1, 1),   # K = 2304
        (1, 8, 17, 17, 8, 7, 3, (3, 3, 3, 3), 1, 0),       # stride 3, 7x7
        (1, 64, 160, 160, 64, 3, 2, (1, 1, 1, 1), 1, 1),   # <= 64 channels, few tiles: pixel-major at 80x80
        (2, 48, 83, 97, 40, 3, 1, (1, 1, 1, 1), 1, 1),     # pixel-major, ragged image, 40 channels
        (1, 256, 20, 20, 64, 3, 1, (1, 1, 1, 1), 1, 1),    # 4 pixel tiles of 72 k-blocks: K split in 18 slices
        (1, 128, 40, 40, 128, 3, 2, (1, 1, 1, 1), 1, 1),   # under one channel-major wave: pixel tiles, 9 K slices
        (2, 96, 13, 11, 200, 3, 1, (1, 1, 1, 1), 1, 3),    # split K, 2 channel tiles (200 = 128 + 72), ragged
    ],
)
def test_conv_geometries(ctx, N, C, H, W, M, k, stride, pads, dil, act):
    x, w, b = _case(N * 1000 + C + k, N, C, H, W, M, k)
    y = _conv(ctx, x, w, b, (stride, stride), pads, (dil, dil), act)
    ref = oracle.conv2d(x, w, b, (stride, stride), pads, (dil, dil), 1, act)
    assert y.shape == ref.shape
    assert rel_err(y, ref) <= TOL


def test_conv_without_bias(ctx):
    x, w, _ = _case(9, 1, 32, 12, 12, 32, 3)
    y = _conv(ctx, x, w, None, pads=(1, 1, 1, 1))
    assert rel_err(y, oracle.conv2d(x, w, None, pads=(1, 1, 1, 1))) <= TOL


def test_conv_rejects_bad_output_size_and_groups(ctx):
    import torch

    from onnxsharp_b200 import OscError
    from onnxsharp_b200 import _lib
    from onnxsharp_b200.runtime import ConvWeights

    x = torch.zeros(1, 8, 10, 10, device="cuda")
    cw = ConvWeights(ctx, torch.zeros(8, 8, 3, 3, device="cuda"), (8, 8, 3, 3))
    y = torch.zeros(1, 8, 10, 10, device="cuda")
    with pytest.raises(OscError):  # pad 0 gives 8x8, not 10x10
        _lib.call("osc_conv2d_bias_act_f32", ctx.handle, x.data_ptr(), 1, 8, 10, 10, cw.handle, 1, 1, 0, 0, 0, 0, 1,
                  1, 1, None, 0, y.data_ptr(), 10, 10)
    with pytest.raises(OscError):  # grouped conv is a different entry point
        _lib.call("osc_conv2d_bias_act_f32", ctx.handle, x.data_ptr(), 1, 8, 10, 10, cw.handle, 1, 1, 1, 1, 1, 1, 1,
                  1, 2, None, 0, y.data_ptr(), 10, 10)


@pytest.mark.parametrize(
    "N,C,H,W,M,act",
    [
        (3, 96, 40, 40, 128, 1),    # 12.5 pixel tiles per image
        (1, 32, 160, 160, 32, 1),   # narrow: MMA N = 32
        (2, 80, 80, 80, 80, 1),     # MMA N = 80, K padded to 96
        (1, 512, 20, 20, 256, 0),   # K = 512: 16 k-blocks in 8 TMEM chunks, 2 channel tiles
        (2, 7, 6, 6, 5, 3),         # C = 7, M = 5 (N rounded to 16), Sigmoid
        (1, 16, 5, 5, 16, 1),       # 25-pixel planes: not 16-byte aligned, implicit-GEMM fallback
        (1, 256, 20, 20, 64, 1),    # 64-channel tile: 8 k-blocks around the 4-stage ring
        (2, 64, 12, 12, 48, 0),     # 64-channel tile, 48 channels: the last epilogue warp group idle
    ],
)
def test_conv_pointwise(ctx, N, C, H, W, M, act):
    """1x1 convs read NCHW directly (A operand MN-major, hi/lo split in shared memory)."""
    x, w, b = _case(N * 7 + C + M, N, C, H, W, M, 1)
    y = _conv(ctx, x, w, b, act=act)
    assert rel_err(y, oracle.conv2d(x, w, b, act=act)) <= TOL


def test_conv_pointwise_views_and_residual(ctx):
    """The C3k2 / C2PSA pattern: input a channel slice (Split), output a slice of
    a Concat buffer, residual Add fused: y = res + SiLU(conv1x1(x) + b)."""
    import torch

    from onnxsharp_b200 import ops
    from onnxsharp_b200.runtime import ConvWeights

    rng = np.random.default_rng(31)
    big_x = rng.uniform(0, 1, (3, 200, 20, 20)).astype(np.float32)
    w = (rng.normal(0, 1, (64, 128, 1, 1)) * np.sqrt(2.0 / 128)).astype(np.float32)
    b = rng.normal(0, 0.01, 64).astype(np.float32)
    res = rng.normal(0, 1, (3, 64, 20, 20)).astype(np.float32)
    out_big = torch.zeros(3, 192, 20, 20, device="cuda")
    ops.conv2d_ex(ctx, torch.from_numpy(big_x).cuda()[:, 36:164], ConvWeights(ctx, torch.from_numpy(w).cuda(), w.shape),
                  torch.from_numpy(b).cuda(), out_big[:, 64:128], 1, 0, 1, 1, torch.from_numpy(res).cuda())
    ctx.synchronize()
    ref = res + oracle.conv2d(np.ascontiguousarray(big_x[:, 36:164]), w, b, act=1)
    got = out_big.cpu().numpy()
    assert rel_err(got[:, 64:128], ref) <= TOL
    assert not got[:, :64].any() and not got[:, 128:].any()


@pytest.mark.parametrize("k,C,M", [(3, 256, 64), (1, 512, 128)])
def test_conv_split_k_views_and_residual(ctx, k, C, M):
    """Split-K (few output tiles, long K) through the view / residual path: the
    K slices' partial sums are added by the reduce kernel, which then applies
    bias, SiLU and the residual into a channel slice of a wider output."""
    import torch

    from onnxsharp_b200 import ops
    from onnxsharp_b200.runtime import ConvWeights

    rng = np.random.default_rng(37 + k)
    x = rng.uniform(0, 1, (1, C, 20, 20)).astype(np.float32)
    w = (rng.normal(0, 1, (M, C, k, k)) * np.sqrt(2.0 / (C * k * k))).astype(np.float32)
    b = rng.normal(0, 0.01, M).astype(np.float32)
    res = rng.normal(0, 1, (1, M, 20, 20)).astype(np.float32)
    out_big = torch.zeros(1, M + 64, 20, 20, device="cuda")
    ops.conv2d_ex(ctx, torch.from_numpy(x).cuda(), ConvWeights(ctx, torch.from_numpy(w).cuda(), w.shape),
                  torch.from_numpy(b).cuda(), out_big[:, 32:32 + M], 1, k // 2, 1, 1, torch.from_numpy(res).cuda())
    ctx.synchronize()
    ref = res + oracle.conv2d(x, w, b, pads=(k // 2,) * 4, act=1)
    got = out_big.cpu().numpy()
    assert rel_err(got[:, 32:32 + M], ref) <= TOL
    assert not got[:, :32].any() and not got[:, 32 + M:].any()


@pytest.mark.parametrize("N,C,H,M,stride", [(36, 32, 40, 64, 1), (36, 64, 40, 32, 1), (36, 32, 40, 48, 1),
                                            (36, 32, 80, 64, 2)])
def test_conv_channel_major_narrow_layers(ctx, N, C, H, M, stride):
    """Layers of at most 64 output channels on the channel-major kernel (many
    256-pixel tiles): 64-row weight boxes stacked [W hi; W lo] into one
    128-row operand, 2 MMAs per K step, the epilogue adding D rows r and
    r + 64; 48 and 32 channels leave zero rows in both halves. The launch is
    checked to be the channel-major kernel."""
    x, w, b = _case(50 + M + stride, N, C, H, H, M, 3)
    ctx.profile_reset()
    ctx.profile(True)
    y = _conv(ctx, x, w, b, stride=(stride, stride), pads=(1, 1, 1, 1), act=1)
    ctx.profile(False)
    assert ctx.profile_read("k_conv_tf32x3")[1] == 1
    assert rel_err(y, oracle.conv2d(x, w, b, stride=(stride, stride), pads=(1, 1, 1, 1), act=1)) <= TOL
