"""ctypes binding of the CPU oracle (oracle.c).

TEST INFRASTRUCTURE ONLY: the checker used by tests/, __graft_entry__.smoke()
and bench.py's CPU-baseline / reference arms. The product (onnxsharp_b200)
never imports this package.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "liboracle.so"

_f = C.POINTER(C.c_float)
_i32 = C.POINTER(C.c_int32)
_u8 = C.POINTER(C.c_uint8)
_vp = C.c_void_p
_int = C.c_int
_long = C.c_long
_flt = C.c_float

_SIGS = {
    "orc_exp": (_flt, [_flt]),
    "orc_sigmoid": (_flt, [_flt]),
    "orc_silu": (_flt, [_flt]),
    "orc_unary": (None, [_vp, _vp, _long, _int, _int]),
    "orc_gemm_f32": (None, [_vp, _int, _vp, _int, _int, _int, _int, _vp, _vp, _vp, _int, _int, _vp, _int, _int]),
    "orc_minmax": (None, [_vp, _long, _f, _f]),
    "orc_dql_params": (None, [_flt, _flt, _f, C.POINTER(_int)]),
    "orc_quantize_u8": (None, [_vp, _long, _flt, _int, _vp, _int]),
    "orc_dqmm": (None, [_vp, _int, _int, _vp, _int, _vp, _int, _vp, _int, _vp, _int, _int, _vp, _vp, _vp, _vp, _int]),
    "orc_letterbox": (None, [_vp, _int, _int, _int, _int, _int, _int, _int, _vp, _vp]),
    "orc_matmul_integer": (None, [_vp, _int, _int, _int, _int, _vp, _int, _vp, _int, _int, _vp, _int]),
    "orc_conv2d": (None, [_vp, _int, _int, _int, _int, _vp, _int, _int, _int, _int, _int, _int, _int, _int, _int,
                          _int, _vp, _int, _vp, _int, _int, _int]),
    "orc_attention": (None, [_vp, _vp, _vp, _vp, _int, _int, _int, _int, _int, _flt, _int, _int, _int, _vp, _int]),
    "orc_dfl": (None, [_vp, _int, _int, _int, _int, _vp, _int]),
    "orc_softmax_rows": (None, [_vp, _vp, _long, _int, _int]),
    "orc_layernorm": (None, [_vp, _int, _int, _vp, _vp, _flt, _vp, _int]),
}

_lib = None


def build() -> Path:
    """Compile liboracle.so with the committed Makefile (no-op when current)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not LIB.exists() or LIB.stat().st_mtime < (HERE / "oracle.c").stat().st_mtime:
            build()
        l = C.CDLL(str(LIB))
        for name, (res, args) in _SIGS.items():
            fn = getattr(l, name)
            fn.restype = res
            fn.argtypes = args
        _lib = l
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data


def _c(a, dtype=np.float32):
    return None if a is None else np.ascontiguousarray(a, dtype=dtype)


THREADS = int(os.environ.get("ONNXSHARP_THREADS", "0"))


def exp(x: float) -> float:
    return lib().orc_exp(float(x))


def unary(x, act: int, threads: int = THREADS):
    x = _c(x)
    y = np.empty_like(x)
    lib().orc_unary(_p(x), _p(y), x.size, act, threads)
    return y


def gemm(a, b, row_bias=None, col_bias=None, col_scale=None, act: int = 0, mr12: int = 1, threads: int = THREADS):
    """C = A[m,k] @ B[k,n] with the reference's FMA-chain semantics."""
    a, b = _c(a), _c(b)
    m, k = a.shape
    n = b.shape[1]
    rb, cb, cs = _c(row_bias), _c(col_bias), _c(col_scale)
    c = np.empty((m, n), np.float32)
    lib().orc_gemm_f32(_p(a), k, _p(b), n, m, k, n, _p(rb), _p(cb), _p(cs), mr12, act, _p(c), n, threads)
    return c


def minmax(x):
    x = _c(x)
    mn, mx = C.c_float(), C.c_float()
    lib().orc_minmax(_p(x), x.size, C.byref(mn), C.byref(mx))
    return mn.value, mx.value


def dql_params(mn: float, mx: float):
    s, z = C.c_float(), C.c_int()
    lib().orc_dql_params(mn, mx, C.byref(s), C.byref(z))
    return s.value, z.value


def quantize_u8(x, scale: float, zp: int, threads: int = THREADS):
    x = _c(x)
    q = np.empty(x.shape, np.uint8)
    lib().orc_quantize_u8(_p(x), x.size, scale, zp, _p(q), threads)
    return q


def dqmm(a, w, w_zp, w_scale, bias=None, mr12: int = 1, threads: int = THREADS):
    """DynamicQuantizeMatMul: returns (y, q_u8, acc_s32, (scale, zp))."""
    a = _c(a)
    m, k = a.shape
    w = np.ascontiguousarray(w)
    signed = 1 if w.dtype == np.int8 else 0
    n = w.shape[1]
    zp = np.ascontiguousarray(np.atleast_1d(w_zp), dtype=np.int32)
    sc = np.ascontiguousarray(np.atleast_1d(w_scale), dtype=np.float32)
    b = _c(bias)
    y = np.empty((m, n), np.float32)
    q = np.empty((m, k), np.uint8)
    acc = np.empty((m, n), np.int32)
    params = np.empty(2, np.float32)
    lib().orc_dqmm(_p(a), m, k, _p(w), signed, _p(zp), zp.size, _p(sc), sc.size, _p(b), n, mr12, _p(y), _p(q), _p(acc),
                   _p(params), threads)
    return y, q, acc, (float(params[0]), int(params[1]))


def matmul_integer(a, a_zp: int, w, w_zp, threads: int = THREADS):
    """MatMulInteger: s32 sum_t (a - a_zp)(w - w_zp[j]); a and w are uint8 or int8 arrays."""
    a = np.ascontiguousarray(a)
    assert a.dtype in (np.uint8, np.int8)
    w = np.ascontiguousarray(w)
    signed = 1 if w.dtype == np.int8 else 0
    zp = np.ascontiguousarray(np.atleast_1d(w_zp), dtype=np.int32)
    m, k = a.shape
    n = w.shape[1]
    acc = np.empty((m, n), np.int32)
    lib().orc_matmul_integer(_p(a), 1 if a.dtype == np.int8 else 0, m, k, a_zp, _p(w), signed, _p(zp), zp.size, n,
                             _p(acc), threads)
    return acc


def conv_out(size: int, k: int, s: int, p0: int, p1: int, d: int) -> int:
    """Ops/DnnOps.cs:53-66 (SpatialOut, floor mode)."""
    return (size + p0 + p1 - ((k - 1) * d + 1)) // s + 1


def conv2d(x, w, bias=None, stride=(1, 1), pads=(0, 0, 0, 0), dil=(1, 1), group=1, act=0, threads: int = THREADS,
           out=None):
    """NCHW conv; pads = (top, left, bottom, right). `out`: an optional
    C-contiguous float32 [N, M, OH, OW] array to write into."""
    x, w = _c(x), _c(w)
    N, Cc, H, W = x.shape
    M, _, kh, kw = w.shape
    OH = conv_out(H, kh, stride[0], pads[0], pads[2], dil[0])
    OW = conv_out(W, kw, stride[1], pads[1], pads[3], dil[1])
    if out is not None and (out.shape != (N, M, OH, OW) or out.dtype != np.float32 or not out.flags.c_contiguous):
        raise ValueError("conv2d: out must be a C-contiguous float32 array of the output shape")
    y = np.empty((N, M, OH, OW), np.float32) if out is None else out
    b = _c(bias)
    lib().orc_conv2d(_p(x), N, Cc, H, W, _p(w), M, kh, kw, stride[0], stride[1], pads[0], pads[1], dil[0], dil[1], group,
                     _p(b), act, _p(y), OH, OW, threads)
    return y


def attention(q, k, v, heads: int, scale: float, mask=None, out_head_space: int = 0, heads_form: int = 1,
              block_min_seq: int = 64, threads: int = THREADS):
    q, k, v = _c(q), _c(k), _c(v)
    if heads_form:
        B, T, Cw = q.shape
        H, D = heads, Cw // heads
    else:
        B, H, T, D = q.shape
    out = np.empty((B, H, T, D) if out_head_space else (B, T, H * D), np.float32)
    m = _c(mask)
    mask_rows = 0 if m is None else m.shape[2]
    lib().orc_attention(_p(q), _p(k), _p(v), _p(m), mask_rows, B, T, H, D, scale, heads_form, out_head_space,
                        block_min_seq, _p(out), threads)
    return out


def softmax(x, threads: int = THREADS):
    """Softmax over the last axis (VectorMath.SoftmaxRow per row)."""
    x = _c(x)
    y = np.empty_like(x)
    lib().orc_softmax_rows(_p(x), _p(y), x.size // x.shape[-1], x.shape[-1], threads)
    return y


def dfl(x, bins: int = 16, threads: int = THREADS):
    """x: [B, 4*bins, N] -> [B, 4, N]."""
    x = _c(x)
    B, CB, N = x.shape
    sides = CB // bins
    out = np.empty((B, sides, N), np.float32)
    lib().orc_dfl(_p(x), B, sides, bins, N, _p(out), threads)
    return out


def layernorm(x, gamma=None, beta=None, eps: float = 1e-5, axis: int = -1, threads: int = THREADS):
    x = _c(x)
    axis = axis % x.ndim
    outer = int(np.prod(x.shape[:axis])) if axis else 1
    inner = int(np.prod(x.shape[axis:]))
    y = np.empty_like(x)
    lib().orc_layernorm(_p(x), outer, inner, _p(_c(gamma)), _p(_c(beta)), eps, _p(y), threads)
    return y


def letterbox(pixels, bgr: bool = False, target=(640, 640), row_stride: int = 0):
    """ImagePreprocessor.Letterbox of an [H, W, 3|4] uint8 image: ([3, th, tw] float32, (rw, rh, ox, oy))."""
    px = np.ascontiguousarray(pixels, dtype=np.uint8)
    h, w, bpp = px.shape
    tw, th = target
    dst = np.empty((3, th, tw), np.float32)
    pl = np.zeros(4, np.int32)
    lib().orc_letterbox(_p(px), w, h, row_stride or w * bpp, bpp, 1 if bgr else 0, tw, th, _p(dst), _p(pl))
    return dst, tuple(int(v) for v in pl)
