"""MatMul beyond the constant-weight path, on the B200 (3xTF32), against the
oracle's FMA-chain GEMM at the reference's tolerance |d| / max(1, |ref|) <= 1e-4
(GemmKernelTests.cs:116-120):
- batched / transposed-view MatMul with a non-constant B (attention QK^T and
  P.V outside FusedAttention; DnnOps.cs:2945-3094 and the gemm_view strides);
- ONNX Gemm with transA / transB, alpha, beta and C broadcasting
  (AttnOps.cs:31-128)."""
from __future__ import annotations

import numpy as np
import pytest

import oracle
from conftest import rel_err

pytestmark = pytest.mark.gpu


def T(x):
    import torch

    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def _ref_batched(a, b, bias=None):
    *batch, m, k = a.shape
    n = b.shape[-1]
    a2 = np.broadcast_to(a, tuple(np.broadcast_shapes(a.shape[:-2], b.shape[:-2])) + (m, k)).reshape(-1, m, k)
    b2 = np.broadcast_to(b, tuple(np.broadcast_shapes(a.shape[:-2], b.shape[:-2])) + (k, n)).reshape(-1, k, n)
    out = np.stack([oracle.gemm(np.ascontiguousarray(x), np.ascontiguousarray(y), col_bias=bias)
                    for x, y in zip(a2, b2)])
    return out.reshape(tuple(np.broadcast_shapes(a.shape[:-2], b.shape[:-2])) + (m, n))


def test_attention_scores_and_values_through_transposed_views(ctx):
    """S = Q K^T with K^T a stride view of K [B,H,T,D]; O = P V; T = 400 as in C2PSA."""
    from onnxsharp_b200.runtime import matmul_batched

    rng = np.random.default_rng(1)
    q = rng.normal(0, 1, (2, 2, 400, 32)).astype(np.float32)
    k = rng.normal(0, 1, (2, 2, 400, 32)).astype(np.float32)
    v = rng.normal(0, 1, (2, 2, 400, 64)).astype(np.float32)
    tk = T(k)
    s = matmul_batched(ctx, T(q), tk.transpose(-1, -2))
    ctx.synchronize()
    ref_s = _ref_batched(q, np.swapaxes(k, -1, -2))
    assert rel_err(s.cpu().numpy(), ref_s) <= 1e-4
    p = np.exp(ref_s - ref_s.max(-1, keepdims=True)).astype(np.float32)
    o = matmul_batched(ctx, T(p), T(v))
    ctx.synchronize()
    assert rel_err(o.cpu().numpy(), _ref_batched(p, v)) <= 1e-4


@pytest.mark.parametrize("a_shape,b_shape,bias", [
    ((3, 37, 50), (50, 70), True),        # B shared across batches (stride 0)
    ((4, 5, 33, 20), (4, 5, 20, 9), False),  # two batch dims, ragged everything
    ((1, 300, 256), (256, 256), True),    # the DETR-style [300,1,256] projection folded to one batch
])
def test_batched_matmul_shapes(ctx, a_shape, b_shape, bias):
    from onnxsharp_b200.runtime import matmul_batched

    rng = np.random.default_rng(sum(a_shape) + sum(b_shape))
    a = rng.uniform(-1, 1, a_shape).astype(np.float32)
    b = rng.uniform(-1, 1, b_shape).astype(np.float32)
    cb = rng.uniform(-1, 1, b_shape[-1]).astype(np.float32) if bias else None
    got = matmul_batched(ctx, T(a), T(b), None if cb is None else T(cb))
    ctx.synchronize()
    assert rel_err(got.cpu().numpy(), _ref_batched(a, b, cb)) <= 1e-4


def _gemm_ref(a, b, alpha, beta, c):
    d = oracle.gemm(np.ascontiguousarray(a), np.ascontiguousarray(b))
    out = (np.float32(alpha) * d).astype(np.float32) if alpha != 1.0 else d
    if c is not None and beta != 0.0:
        m, n = out.shape
        cf = c.reshape(-1)
        if cf.size >= m * n:
            cb = cf[: m * n].reshape(m, n)
        elif cf.size == 1:
            cb = np.full((m, n), cf[0], np.float32)
        else:
            cb = np.broadcast_to(cf[np.arange(n) % cf.size], (m, n))
        out = (out + (np.float32(beta) * cb).astype(np.float32)).astype(np.float32)
    return out


@pytest.mark.parametrize("trans_a,trans_b,packed,alpha,beta,c_kind", [
    (False, False, True, 1.0, 1.0, "row"),
    (True, False, False, 0.5, 2.0, "full"),
    (False, True, False, 1.0, -1.0, "scalar"),
    (True, True, True, 2.0, 0.0, "full"),
    (False, False, False, 1.0, 1.0, None),
])
def test_onnx_gemm(ctx, trans_a, trans_b, packed, alpha, beta, c_kind):
    from onnxsharp_b200.runtime import GemmWeights, gemm_onnx

    rng = np.random.default_rng(int(trans_a) * 4 + int(trans_b) * 2 + int(packed))
    m, k, n = 150, 96, 200
    a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
    b = rng.uniform(-1, 1, (k, n)).astype(np.float32)
    c = {"row": rng.uniform(-1, 1, n), "full": rng.uniform(-1, 1, (m, n)), "scalar": rng.uniform(-1, 1, 1),
         None: None}[c_kind]
    c = None if c is None else c.astype(np.float32)
    a_in = a.T.copy() if trans_a else a
    b_in = b.T.copy() if trans_b else b
    w = GemmWeights(ctx, T(b_in), k, n, 1 if trans_b else 0) if packed else None
    got = gemm_onnx(ctx, T(a_in), trans_a, w=w, b=None if packed else T(b_in), trans_b=trans_b, alpha=alpha, beta=beta,
                    c=None if c is None else T(c))
    ctx.synchronize()
    assert rel_err(got.cpu().numpy(), _gemm_ref(a, b, alpha, beta, c)) <= 1e-4
