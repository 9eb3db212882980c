"""FusedAttention on the B200 (one head per SM for T <= 128; a composed
tensor-core path for longer sequences and other head sizes) against the oracle's restatement of
AttentionLayer (ComputeBlocks for T > 64, ComputeRows otherwise). Tolerance:
max |d| <= 1e-5 absolute (the reference's attention golden, AttentionTests.cs)
and |d| / max(1, |ref|) <= 1e-4."""
from __future__ import annotations

import numpy as np
import pytest

import oracle
from conftest import rel_err

pytestmark = pytest.mark.gpu


def _attn(ctx, q, k, v, heads, scale, mask=None, out_head_space=False):
    import torch

    from onnxsharp_b200.runtime import attention

    t = lambda a: None if a is None else torch.from_numpy(np.ascontiguousarray(a)).cuda()
    out = attention(ctx, t(q), t(k), t(v), heads, scale, t(mask), out_head_space)
    ctx.synchronize()
    return out.cpu().numpy()


def _qkv(seed, B, T, C):
    rng = np.random.default_rng(seed)
    return [rng.normal(0, 1, (B, T, C)).astype(np.float32) for _ in range(3)]


def _check(got, ref):
    assert got.shape == ref.shape
    assert np.max(np.abs(got - ref)) <= 1e-5
    assert rel_err(got, ref) <= 1e-4


def test_attention_config4_core(ctx):
    """BASELINE config 4 core: B=64, T=128, H=8, D=64, scale 1/sqrt(64)."""
    q, k, v = _qkv(4, 64, 128, 512)
    _check(_attn(ctx, q, k, v, 8, 0.125), oracle.attention(q, k, v, heads=8, scale=0.125))


def test_attention_golden_fixture(ctx, golden):
    g = golden
    _check(_attn(ctx, g["attn_q"], g["attn_k"], g["attn_v"], 2, 0.25), g["attn_o"])


@pytest.mark.parametrize("B,T,H,D", [(2, 40, 4, 64), (3, 127, 2, 64), (1, 1, 1, 64), (2, 64, 8, 32), (1, 100, 3, 32),
                                     (40, 77, 8, 32), (37, 128, 8, 64)])  # several heads per persistent CTA
def test_attention_shapes(ctx, B, T, H, D):
    q, k, v = _qkv(B * 131 + T, B, T, H * D)
    s = 1.0 / np.sqrt(D)
    _check(_attn(ctx, q, k, v, H, s), oracle.attention(q, k, v, heads=H, scale=s))


@pytest.mark.parametrize("full", [False, True], ids=["row_mask", "full_mask"])
def test_attention_mask(ctx, full):
    B, T, H, D = 40, 93, 8, 64  # 320 heads: each CTA walks several, T not a multiple of 8
    rows = T if full else 1
    q, k, v = _qkv(rows, B, T, H * D)
    rng = np.random.default_rng(99)
    mask = np.where(rng.uniform(size=(B, 1, rows, T)) < 0.2, -1e4, 0.0).astype(np.float32)
    _check(_attn(ctx, q, k, v, H, 0.125, mask), oracle.attention(q, k, v, heads=H, scale=0.125, mask=mask))


def test_attention_output_head_space(ctx):
    q, k, v = _qkv(5, 2, 70, 128)
    _check(_attn(ctx, q, k, v, 2, 0.125, out_head_space=True),
           oracle.attention(q, k, v, heads=2, scale=0.125, out_head_space=1))


def test_attention_block_with_projections(ctx):
    """Config-4 block at B=8: Q/K/V projections (MatMul+bias), FusedAttention, output projection."""
    import torch

    from onnxsharp_b200.runtime import GemmWeights, attention, gemm_bias

    rng = np.random.default_rng(44)
    B, T, C, H = 8, 128, 512, 8
    x = rng.normal(0, 1, (B * T, C)).astype(np.float32)
    lim = np.sqrt(6.0 / (C + C))
    ws = [rng.uniform(-lim, lim, (C, C)).astype(np.float32) for _ in range(4)]
    bias = np.zeros(C, np.float32)
    dx = torch.from_numpy(x).cuda()
    db = torch.from_numpy(bias).cuda()
    gw = [GemmWeights(ctx, torch.from_numpy(w).cuda(), C, C) for w in ws]
    qd, kd, vd = (gemm_bias(ctx, dx, w, db).view(B, T, C) for w in gw[:3])
    od = attention(ctx, qd, kd, vd, H, 0.125)
    yd = gemm_bias(ctx, od.view(B * T, C), gw[3], db)
    ctx.synchronize()
    q, k, v = (oracle.gemm(x, w, col_bias=bias).reshape(B, T, C) for w in ws[:3])
    o = oracle.attention(q, k, v, heads=H, scale=0.125)
    y = oracle.gemm(o.reshape(B * T, C), ws[3], col_bias=bias)
    assert rel_err(yd.cpu().numpy(), y) <= 1e-4


def test_attention_rejects_bad_mask_rows(ctx):
    """A mask must be [B, 1, 1|T, T] (AttentionOps.cs:249-351)."""
    import torch

    from onnxsharp_b200 import OscError
    from onnxsharp_b200.runtime import attention

    z = torch.zeros(1, 129, 64, device="cuda")
    m = torch.zeros(1, 1, 7, 129, device="cuda")
    with pytest.raises(OscError):
        attention(ctx, z, z, z, 1, 0.125, m)


@pytest.mark.parametrize("B,T,H,D,mask_rows,head_space", [
    (2, 200, 2, 64, 0, False),     # beyond one 128-key tile
    (1, 1000, 4, 32, 1, True),     # long sequence, [B,1,1,T] key mask, head-space output
    (1, 300, 3, 48, 300, False),   # head size outside {32, 64}, full [B,1,T,T] mask
    (2, 64, 2, 16, 0, False),      # short sequence, small head (composed path by head size)
    (1, 4096, 1, 64, 0, False),    # the fusion limit (GraphFusion admits T <= 4096)
])
def test_attention_long_sequences(ctx, B, T, H, D, mask_rows, head_space):
    """T > 128 and other head sizes take the composed path (tensor-core QK^T and
    e.V, the reference's lazy softmax with its 8-lane sum order in between)."""
    q, k, v = _qkv(T + D, B, T, H * D)
    mask = None
    if mask_rows:
        rng = np.random.default_rng(T)
        mask = np.where(rng.uniform(0, 1, (B, 1, mask_rows, T)) < 0.2, -1e4, 0.0).astype(np.float32)
    s = 1.0 / np.sqrt(D)
    _check(_attn(ctx, q, k, v, H, s, mask, head_space),
           oracle.attention(q, k, v, heads=H, scale=s, mask=mask, out_head_space=int(head_space)))
