"""The native static-plan executor (osc_plan_build / osc_plan_run): any graph
of fused nodes over channel slices of NCHW buffers, lifetime-coloured into one
device arena, replayed as one CUDA graph per (input, output) pair.

1. The YOLO11n-shaped IR lowered to a native plan gives the same bits as the
   Python-driven plan (yolo.Net): same kernels, same routing, same order.
2. A small graph that is not YOLO (conv into a Concat slice, MaxPool,
   depthwise conv with a residual, Resize into the other Concat slice, 1x1
   conv, MatMul+bias, Softmax) against the oracle's composition.
3. The config-4 attention block as a plan (three MatMul+bias projections,
   FusedAttention, the output projection) against the oracle."""
from __future__ import annotations

import numpy as np
import pytest

import oracle
from conftest import rel_err

pytestmark = pytest.mark.gpu


def test_native_yolo_plan_matches_python_plan(ctx):
    import torch

    from onnxsharp_b200 import plan as P
    from onnxsharp_b200 import yolo

    g = yolo.build_yolo11n()
    params = yolo.init_params(g, 51)
    images = np.random.default_rng(51).uniform(0, 1, (2, 3, 640, 640)).astype(np.float32)
    net = yolo.Net(ctx, g, params, 2)
    net.input_view().copy_(torch.from_numpy(images))
    want = net.forward(use_graph=True).cpu().numpy()
    pl = P.build_yolo_plan(ctx, g, net.dev_params, net.packed, 2)
    assert 0 < pl.arena_bytes() <= net.arena_bytes
    x = torch.from_numpy(images).cuda()
    out = torch.full((2, 84, 8400), float("nan"), device="cuda")
    for _ in range(2):  # eager + capture, then a replay of the cached graph
        pl.run(x, out)
        ctx.synchronize()
        assert np.array_equal(out.cpu().numpy().view(np.uint32), want.view(np.uint32))
    x2 = torch.from_numpy(images[::-1].copy()).cuda()  # a new input pointer: a second cached graph
    out2 = torch.empty_like(out)
    pl.run(x2, out2)
    ctx.synchronize()
    assert np.array_equal(out2.cpu().numpy(), want[::-1])
    pl.close()
    net.close()


def _conv_w(rng, m, c, k):
    return (rng.standard_normal((m, c, k, k)) * np.sqrt(2.0 / (c * k * k))).astype(np.float32)


def test_native_plan_generic_graph_matches_oracle(ctx):
    import torch

    from onnxsharp_b200 import ACT_NONE, ACT_SILU
    from onnxsharp_b200 import plan as P
    from onnxsharp_b200.runtime import ConvWeights, GemmWeights

    rng = np.random.default_rng(52)
    B = 2
    x = rng.uniform(0, 1, (B, 16, 32, 32)).astype(np.float32)
    w1, b1 = _conv_w(rng, 64, 16, 3), rng.normal(0, 0.01, 64).astype(np.float32)
    wd, bd = _conv_w(rng, 64, 1, 3), rng.normal(0, 0.01, 64).astype(np.float32)
    w2, b2 = _conv_w(rng, 32, 128, 1), rng.normal(0, 0.01, 32).astype(np.float32)
    wm, bm = rng.uniform(-0.2, 0.2, (32, 48)).astype(np.float32), rng.uniform(-1, 1, 48).astype(np.float32)
    T = lambda a: torch.from_numpy(a).cuda()  # noqa: E731
    cw1, cw2 = ConvWeights(ctx, T(w1), w1.shape), ConvWeights(ctx, T(w2), w2.shape)
    gw = GemmWeights(ctx, T(wm), 32, 48)
    dev = dict(b1=T(b1), wd=T(wd), bd=T(bd), b2=T(b2), bm=T(bm))
    # buffers: 0 input, 1 cat [128,32,32], 2 pool [64,16,16], 3 dw [64,16,16], 4 e [32,32,32], 5 f [32,32,48],
    # 6 g [32,32,48]
    bufs = [(16, 32, 32), (128, 32, 32), (64, 16, 16), (64, 16, 16), (32, 32, 32), (32, 32, 48), (32, 32, 48)]
    nodes = [
        P.node(P.OP_CONV, [(0, 0, 16)], [(1, 0, 64)], [1, 1, 1, ACT_SILU, 3, 1], weights=cw1.handle, bias=dev["b1"]),
        P.node(P.OP_MAXPOOL, [(1, 0, 64)], [(2, 0, 64)], [2, 2, 0]),
        P.node(P.OP_CONV_DIRECT, [(2, 0, 64), (2, 0, 64)], [(3, 0, 64)], [1, 1, 1, ACT_SILU, 3, 64],
               weights=dev["wd"], bias=dev["bd"]),
        P.node(P.OP_RESIZE_NEAREST, [(3, 0, 64)], [(1, 64, 64)], [2]),
        P.node(P.OP_CONV, [(1, 0, 128)], [(4, 0, 32)], [1, 0, 1, ACT_NONE, 1, 1], weights=cw2.handle,
               bias=dev["b2"]),
        P.node(P.OP_MATMUL_BIAS, [(4, 0, 32)], [(5, 0, 32)], [0, 0, 0, ACT_NONE], weights=gw.handle, bias=dev["bm"]),
        P.node(P.OP_SOFTMAX, [(5, 0, 32)], [(6, 0, 32)]),
    ]
    pl = P.Plan(ctx, B, bufs, 0, nodes, keep=[cw1, cw2, gw, dev])
    tx = T(x)
    pl.run(tx, None)
    pl.run(tx, None)
    ctx.synchronize()
    got = _read(pl, 6, tx, (B, 32, 32, 48))
    # oracle composition
    a = oracle.conv2d(x, w1, b1, pads=(1, 1, 1, 1), act=1)
    p = a.reshape(B, 64, 16, 2, 16, 2).max(axis=(3, 5))
    d = (oracle.conv2d(p, wd, bd, pads=(1, 1, 1, 1), group=64, act=1) + p).astype(np.float32)
    cat = np.concatenate([a, np.repeat(np.repeat(d, 2, axis=2), 2, axis=3)], 1)
    e = oracle.conv2d(cat, w2, b2)
    f = oracle.gemm(e.reshape(-1, 32), wm, col_bias=bm)
    want = oracle.softmax(f).reshape(B, 32, 32, 48)
    assert rel_err(got.cpu().numpy(), want) <= 1e-4
    pl.close()


class _DevicePointer:
    """A float32 device buffer at a raw address (the CUDA array interface torch reads)."""

    def __init__(self, address: int, n: int):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": "<f4", "data": (address, False), "version": 3}


def _read(pl, buf, inp, shape):
    """A copy of one of the plan's arena buffers as a host array."""
    import torch

    n = int(np.prod(shape))
    return torch.as_tensor(_DevicePointer(pl.buffer_ptr(buf, inp), n), device="cuda").clone().view(shape)


def test_native_plan_attention_block_matches_oracle(ctx):
    import torch

    from onnxsharp_b200 import plan as P
    from onnxsharp_b200.runtime import GemmWeights

    rng = np.random.default_rng(53)
    B, T_, Cw, H = 4, 128, 256, 4
    x = rng.normal(0, 1, (B, T_, Cw)).astype(np.float32)
    lim = np.sqrt(6.0 / (2 * Cw))
    ws = [rng.uniform(-lim, lim, (Cw, Cw)).astype(np.float32) for _ in range(4)]
    gws = [GemmWeights(ctx, torch.from_numpy(w).cuda(), Cw, Cw) for w in ws]
    zero = torch.zeros(Cw, device="cuda")
    # buffers [T, 1, C] per sequence: 0 x, 1 q, 2 k, 3 v, 4 attn, 5 y
    bufs = [(T_, 1, Cw)] * 6
    nodes = [P.node(P.OP_MATMUL_BIAS, [(0, 0, T_)], [(1 + i, 0, T_)], weights=gws[i].handle, bias=zero)
             for i in range(3)]
    nodes.append(P.node(P.OP_ATTENTION, [(1, 0, T_), (2, 0, T_), (3, 0, T_)], [(4, 0, T_)], [H], [0.125]))
    nodes.append(P.node(P.OP_MATMUL_BIAS, [(4, 0, T_)], [(5, 0, T_)], weights=gws[3].handle, bias=zero))
    pl = P.Plan(ctx, B, bufs, 0, nodes, keep=[gws, zero])
    tx = torch.from_numpy(x).cuda()
    pl.run(tx, None)
    ctx.synchronize()
    y = _read(pl, 5, tx, (B, T_, Cw))
    q, k, v = (oracle.gemm(x.reshape(-1, Cw), w).reshape(B, T_, Cw) for w in ws[:3])
    o = oracle.attention(q, k, v, H, 0.125)
    want = oracle.gemm(o.reshape(-1, Cw), ws[3]).reshape(B, T_, Cw)
    assert rel_err(y.cpu().numpy(), want) <= 1e-4
    pl.close()
