"""Host-side handles over the C ABI: the per-GPU context and packed weights.

Mirrors the reference's split between a one-time weight prepack
(Layer.PrepackWeights, src/OnnxSharp/Core/LayerInfo.cs:75-218, with packed
panels cached by tensor identity, Ops/DnnOps.cs:2823-2832) and a per-inference
Forward. Tensors are torch tensors on the context's device; torch is used for
device memory and streams only, every computation runs in libonnxsharp_cuda.
"""
from __future__ import annotations

import ctypes as C
import weakref

from . import _lib
from ._lib import call, ptr


class Context:
    """One GPU: a stream, a device error word and a scratch arena (osc_ctx)."""

    def __init__(self, device: int = 0, stream: int | None = None):
        _lib.load()
        h = C.c_void_p()
        call("osc_create", int(device), C.byref(h))
        self.handle = h
        self.device = int(device)
        self._finalizer = weakref.finalize(self, _lib.load().osc_destroy, h)
        if stream is not None:
            self.set_stream(stream)

    def set_stream(self, stream: int | None) -> None:
        call("osc_set_stream", self.handle, stream)

    def get_stream(self) -> int | None:
        return _lib.load().osc_get_stream(self.handle)

    def use_torch_stream(self) -> None:
        import torch

        self.set_stream(torch.cuda.current_stream(self.device).cuda_stream)

    def synchronize(self, timeout_ms: int = 60000) -> None:
        call("osc_synchronize", self.handle, int(timeout_ms))

    def reserve_scratch(self, nbytes: int) -> None:
        call("osc_reserve_scratch", self.handle, int(nbytes))

    # -- per-kernel event timing (osc_profile_*) and launch accounting
    def profile(self, on: bool = True) -> None:
        call("osc_profile_enable", self.handle, 1 if on else 0)

    def profile_read(self, prefix: str = "") -> tuple[float, int]:
        """(total milliseconds, launches) of recorded kernels whose name starts with prefix."""
        ms = C.c_double()
        n = C.c_int()
        call("osc_profile_read", self.handle, prefix.encode(), C.byref(ms), C.byref(n))
        return ms.value, n.value

    def profile_reset(self) -> None:
        call("osc_profile_reset", self.handle)

    def launch_count(self) -> int:
        return int(_lib.load().osc_launch_count(self.handle))

    def memcpy_htod(self, dst, src, nbytes: int) -> None:
        call("osc_memcpy_htod", self.handle, ptr(dst), ptr(src), int(nbytes))

    def memcpy_dtoh(self, dst, src, nbytes: int) -> None:
        call("osc_memcpy_dtoh", self.handle, ptr(dst), ptr(src), int(nbytes))

    def capture(self, fn) -> "CapturedGraph":
        """Record the launches fn() makes on this context's stream into a CUDA
        graph (osc_graph_begin / osc_graph_end). fn runs once eagerly first so
        that scratch sizes and kernel attributes are settled outside the
        capture. The stream must not be the legacy default stream."""
        fn()
        self.synchronize()
        call("osc_graph_begin", self.handle)
        h = C.c_void_p()
        try:
            fn()
        finally:
            call("osc_graph_end", self.handle, C.byref(h))
        return CapturedGraph(self, h)

    def close(self) -> None:
        self._finalizer()


class GroupContext(Context):
    """A context owned by a Group (osc_group_ctx): usable like any Context,
    destroyed with its group."""

    def __init__(self, handle, device: int, group: "Group"):  # noqa: D107 - no osc_create
        self.handle = handle
        self.device = int(device)
        self._group = group
        self._finalizer = weakref.finalize(self, lambda: None)


class Group:
    """Several GPUs of one node driven from this process (osc_group_*): a
    context per GPU and an NCCL communicator clique among them."""

    def __init__(self, devices):
        _lib.load()
        self.devices = [int(d) for d in devices]
        arr = (C.c_int * len(self.devices))(*self.devices)
        h = C.c_void_p()
        call("osc_group_create", len(self.devices), arr, C.byref(h))
        self.handle = h
        self._finalizer = weakref.finalize(self, _lib.load().osc_group_destroy, h)
        self.ctxs = []
        for r, d in enumerate(self.devices):
            c = C.c_void_p()
            call("osc_group_ctx", self.handle, r, C.byref(c))
            self.ctxs.append(GroupContext(c, d, self))

    def __len__(self):
        return len(self.devices)

    @staticmethod
    def _ptrs(xs):
        return (C.c_void_p * len(xs))(*[ptr(x) for x in xs])

    def all_gather(self, send, recv, nbytes: int) -> None:
        call("osc_group_allgather", self.handle, self._ptrs(send), self._ptrs(recv), int(nbytes))

    def allreduce_minmax(self, minmax) -> None:
        call("osc_group_allreduce_minmax", self.handle, self._ptrs(minmax))

    def run_sharded(self, graphs, shard_out, gathered_out, shard_bytes: int) -> None:
        hs = [getattr(x, "handle", x) for x in graphs]  # CapturedGraph or a raw osc_graph handle
        g = (C.c_void_p * len(hs))(*[h.value if isinstance(h, C.c_void_p) else h for h in hs])
        call("osc_group_run_sharded", self.handle, g, self._ptrs(shard_out), self._ptrs(gathered_out),
             int(shard_bytes))

    def synchronize(self, timeout_ms: int = 60000) -> None:
        call("osc_group_synchronize", self.handle, int(timeout_ms))

    def close(self) -> None:
        self._finalizer()


class CapturedGraph:
    """An instantiated CUDA graph of library launches (osc_graph_launch replays it on the context's stream)."""

    def __init__(self, ctx: Context, handle):
        self.ctx, self.handle = ctx, handle
        self._finalizer = weakref.finalize(self, _lib.load().osc_graph_free, handle)

    def launch(self) -> None:
        call("osc_graph_launch", self.ctx.handle, self.handle)

    def close(self) -> None:
        self._finalizer()


class GemmWeights:
    """Constant B of a MatMul/Gemm, prepacked once into the 3xTF32 operand form."""

    def __init__(self, ctx: Context, b, k: int, n: int, layout: int = 0):
        h = C.c_void_p()
        name = "osc_gemm_prepack_f32" if _is_device(b) else "osc_gemm_prepack_f32_host"
        call(name, ctx.handle, ptr(b), int(k), int(n), int(layout), C.byref(h))
        self.handle = h
        self.k, self.n = int(k), int(n)
        self._finalizer = weakref.finalize(self, _lib.load().osc_gemm_weights_free, h)


class ConvWeights:
    """Constant W [M, C, kh, kw] of a Conv, prepacked once (tap-major K, 3xTF32 split)."""

    def __init__(self, ctx: Context, w, shape):
        M, Cc, kh, kw = (int(v) for v in shape)
        h = C.c_void_p()
        call("osc_conv_prepack_f32", ctx.handle, ptr(w), M, Cc, kh, kw, 0 if _is_device(w) else 1, C.byref(h))
        self.handle = h
        self.shape = (M, Cc, kh, kw)
        self._finalizer = weakref.finalize(self, _lib.load().osc_conv_weights_free, h)


def conv_out(size: int, k: int, s: int, p0: int, p1: int, d: int) -> int:
    """ONNX Conv output size, floor mode (Ops/DnnOps.cs:53-66)."""
    return (size + p0 + p1 - ((k - 1) * d + 1)) // s + 1


def conv2d(ctx: Context, x, w: ConvWeights, bias=None, stride=(1, 1), pads=(0, 0, 0, 0), dil=(1, 1), group: int = 1,
           act: int = _lib.ACT_NONE, out=None):
    """y = act(conv(x, W) + bias); x NCHW FP32 on the device; pads = (top, left, bottom, right)."""
    import torch

    N, Cc, H, W = x.shape
    M, _, kh, kw = w.shape
    OH = conv_out(H, kh, stride[0], pads[0], pads[2], dil[0])
    OW = conv_out(W, kw, stride[1], pads[1], pads[3], dil[1])
    if out is None:
        out = torch.empty((N, M, OH, OW), dtype=torch.float32, device=x.device)
    call("osc_conv2d_bias_act_f32", ctx.handle, ptr(x), N, Cc, H, W, w.handle, stride[0], stride[1], pads[0], pads[1],
         pads[2], pads[3], dil[0], dil[1], group, ptr(bias), int(act), ptr(out), OH, OW)
    return out


class DqmmWeights:
    """Constant int8/uint8 W [k, n] of a DynamicQuantizeMatMul with its zero points."""

    def __init__(self, ctx: Context, w, k: int, n: int, zero_points=None):
        import numpy as np

        is_signed = 1 if str(getattr(w, "dtype", "")).endswith("int8") and "uint8" not in str(w.dtype) else 0
        zp = None if zero_points is None else np.ascontiguousarray(np.atleast_1d(zero_points), dtype=np.int32)
        h = C.c_void_p()
        call("osc_dqmm_prepack", ctx.handle, ptr(w), int(k), int(n), is_signed, None if zp is None else zp.ctypes.data,
             0 if zp is None else zp.size, 0 if _is_device(w) else 1, C.byref(h))
        self.handle = h
        self.k, self.n, self.signed = int(k), int(n), bool(is_signed)
        self._finalizer = weakref.finalize(self, _lib.load().osc_dqmm_weights_free, h)


def dqmm(ctx: Context, a, w: DqmmWeights, w_scale, bias=None, out=None, minmax_override=None, q_out=None,
         acc_out=None, params_out=None, row0: int | None = None, rows_total: int | None = None):
    """DynamicQuantizeMatMul: y = (quant_u8(A) - zp) @ (W - wzp) * (a_scale * w_scale) + bias.
    With row0 / rows_total, A is the row shard [row0, row0 + m) of a tensor of rows_total rows
    and minmax_override its global range (osc_dqmm_shard_f32)."""
    import torch

    m = a.shape[0]
    if out is None:
        out = torch.empty((m, w.n), dtype=torch.float32, device=a.device)
    if row0 is not None:
        call("osc_dqmm_shard_f32", ctx.handle, ptr(a), int(m), w.k, int(a.stride(0)), w.handle, ptr(w_scale),
             int(w_scale.numel()), ptr(bias), ptr(out), ptr(minmax_override), int(row0), int(rows_total), ptr(q_out),
             ptr(acc_out), ptr(params_out))
        return out
    call("osc_dqmm_f32", ctx.handle, ptr(a), int(m), w.k, int(a.stride(0)), w.handle, ptr(w_scale),
         int(w_scale.numel()), ptr(bias), ptr(out), ptr(minmax_override), ptr(q_out), ptr(acc_out), ptr(params_out))
    return out


def matmul_batched(ctx: Context, a, b, col_bias=None, out=None):
    """Batched MatMul over torch views a [..., m, k] and b [..., k, n] (any strides, up to two batch
    dimensions, size-1 or stride-0 batch dims broadcast); returns the dense [..., m, n] product."""
    import torch

    *ab, m, k = a.shape
    *bb, k2, n = b.shape
    if k2 != k:
        raise ValueError(f"matmul_batched: K mismatch {tuple(a.shape)} x {tuple(b.shape)}")
    nb = max(len(ab), len(bb))
    if nb > 2:
        raise ValueError("matmul_batched: at most two batch dimensions")
    ab, bb = [1] * (nb - len(ab)) + list(ab), [1] * (nb - len(bb)) + list(bb)
    batch = [max(x, y) for x, y in zip(ab, bb)]
    a_st = [0] * (nb - (a.dim() - 2)) + list(a.stride()[:-2])
    b_st = [0] * (nb - (b.dim() - 2)) + list(b.stride()[:-2])
    a_st = [0 if ab[i] == 1 else a_st[i] for i in range(nb)]
    b_st = [0 if bb[i] == 1 else b_st[i] for i in range(nb)]
    outer, inner = ([1, 1] + batch)[-2:]
    ao, ai = ([0, 0] + a_st)[-2:]
    bo, bi = ([0, 0] + b_st)[-2:]
    if out is None:
        out = torch.empty(batch + [m, n], dtype=torch.float32, device=a.device)
    call("osc_matmul_batched_f32", ctx.handle, outer, inner, m, k, n, ptr(a), ao, ai, a.stride(-2), a.stride(-1),
         ptr(b), bo, bi, b.stride(-2), b.stride(-1), ptr(col_bias), ptr(out))
    return out


def gemm_onnx(ctx: Context, a, trans_a: bool, w=None, b=None, trans_b: bool = False, alpha: float = 1.0,
              beta: float = 1.0, c=None, out=None):
    """ONNX Gemm: alpha * A' B' + beta * C; B' from GemmWeights `w` or a device tensor `b`."""
    import torch

    m, k = (a.shape[1], a.shape[0]) if trans_a else (a.shape[0], a.shape[1])
    n = w.n if w is not None else (b.shape[0] if trans_b else b.shape[1])
    if out is None:
        out = torch.empty((m, n), dtype=torch.float32, device=a.device)
    call("osc_gemm_onnx_f32", ctx.handle, ptr(a), int(trans_a), int(m), int(k), None if w is None else w.handle,
         ptr(b), int(trans_b), int(n), float(alpha), float(beta), ptr(c), 0 if c is None else int(c.numel()), ptr(out))
    return out


def dynamic_quantize_linear(ctx: Context, x, y=None, y_scale=None, y_zero_point=None):
    """DynamicQuantizeLinear: (y u8 like x, y_scale f32 [1], y_zero_point u8 [1]) on the device."""
    import torch

    if y is None:
        y = torch.empty(x.shape, dtype=torch.uint8, device=x.device)
    if y_scale is None:
        y_scale = torch.empty(1, dtype=torch.float32, device=x.device)
    if y_zero_point is None:
        y_zero_point = torch.empty(1, dtype=torch.uint8, device=x.device)
    call("osc_dynamic_quantize_linear_f32", ctx.handle, ptr(x), int(x.numel()), ptr(y), ptr(y_scale),
         ptr(y_zero_point))
    return y, y_scale, y_zero_point


def matmul_integer(ctx: Context, a, a_zero_point: int, w: "DqmmWeights", out=None):
    """MatMulInteger: s32 [m, n] = (a - a_zero_point) @ (W - w_zp); a is a uint8 or int8 [m, k] device tensor."""
    import torch

    m = a.shape[0]
    if out is None:
        out = torch.empty((m, w.n), dtype=torch.int32, device=a.device)
    signed = 1 if a.dtype == torch.int8 else 0
    call("osc_matmul_integer_i8", ctx.handle, ptr(a), signed, int(m), w.k, int(a.stride(0)), int(a_zero_point),
         w.handle, ptr(out))
    return out


def minmax(ctx: Context, x, out=None):
    """{min(x, 0), max(x, 0)} over all elements of x (NaN skipped), as a 2-float device tensor."""
    import torch

    if out is None:
        out = torch.empty(2, dtype=torch.float32, device=x.device)
    call("osc_minmax_f32", ctx.handle, ptr(x), int(x.numel()), ptr(out))
    return out


def attention(ctx: Context, q, k, v, heads: int, scale: float, mask=None, out_head_space: bool = False, out=None):
    """FusedAttention, heads form: q/k/v [B, T, H*D] on the device."""
    import torch

    B, T, width = q.shape
    D = width // heads
    if out is None:
        shape = (B, heads, T, D) if out_head_space else (B, T, width)
        out = torch.empty(shape, dtype=torch.float32, device=q.device)
    mask_rows = 0 if mask is None else int(mask.shape[2])
    call("osc_attention_f32", ctx.handle, ptr(q), ptr(k), ptr(v), ptr(mask), mask_rows, int(B), int(T), int(heads),
         int(D), float(scale), 1 if out_head_space else 0, ptr(out))
    return out


def _is_device(x) -> bool:
    return bool(getattr(x, "is_cuda", False))


def gemm_split_a(ctx: Context, a, k: int, out=None):
    """The K-major TF32 hi/lo split of A [m, k] (FP32 on the device) that the
    MatMul kernels read, as a (hi, lo) pair of [m, kp] tensors (kp = k rounded
    up to 4): split once, then gemm_bias_presplit by several weights."""
    import torch

    m, kp = int(a.shape[0]), (int(k) + 3) // 4 * 4
    if out is None:
        out = (torch.empty((m, kp), dtype=torch.float32, device=a.device),
               torch.empty((m, kp), dtype=torch.float32, device=a.device))
    call("osc_gemm_split_a_f32", ctx.handle, ptr(a), m, int(k), int(a.stride(0)), kp, ptr(out[0]), ptr(out[1]))
    return out


def gemm_bias_presplit(ctx: Context, split, w: GemmWeights, bias=None, act: int = _lib.ACT_NONE, out=None,
                       ldc: int = 0):
    """C = A @ B + bias, then `act`, from A's split (gemm_split_a)."""
    import torch

    hi, lo = split
    m, kp = int(hi.shape[0]), int(hi.shape[1])
    if out is None:
        out = torch.empty((m, w.n), dtype=torch.float32, device=hi.device)
    call("osc_gemm_bias_presplit_f32", ctx.handle, ptr(hi), ptr(lo), m, kp, w.handle, ptr(bias), int(act), ptr(out),
         int(ldc or out.stride(0)))
    return out


def gemm_bias(ctx: Context, a, w: GemmWeights, bias=None, act: int = _lib.ACT_NONE, out=None, lda: int = 0,
              ldc: int = 0):
    """C = A @ B + bias (FusedBias), then `act`; A is [m, k] FP32 on the device."""
    import torch

    m, k = a.shape[0], w.k
    if out is None:
        out = torch.empty((m, w.n), dtype=torch.float32, device=a.device)
    call("osc_gemm_bias_f32", ctx.handle, ptr(a), int(m), int(k), int(lda or a.stride(0)), w.handle, ptr(bias),
         int(act), ptr(out), int(ldc or out.stride(0)))
    return out
