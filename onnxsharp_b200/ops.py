"""Python wrappers of the graph-glue entry points of libonnxsharp_cuda.

Tensors are torch CUDA tensors in NCHW. A 4-D argument may be a channel
slice of a larger buffer (``buf[:, c0:c1]``): its ``data_ptr()`` points at the
first channel of image 0 and ``stride(0)`` is the image stride the C ABI takes
as ``*_nstride``; the inner three dimensions must be dense.
"""
from __future__ import annotations

import ctypes as C

from . import _lib
from ._lib import call, ptr

OP_ADD, OP_SUB, OP_MUL, OP_DIV = 0, 1, 2, 3


def _nchw(t):
    n, c, h, w = t.shape
    if t.stride(3) != 1 or t.stride(2) != w or t.stride(1) != h * w:
        raise ValueError("inner dimensions of an NCHW view must be dense")
    return n, c, h, w, t.stride(0)


def out_size(size: int, k: int, s: int, p0: int, p1: int, d: int = 1) -> int:
    return (size + p0 + p1 - ((k - 1) * d + 1)) // s + 1


def conv2d_ex(ctx, x, w, bias, y, stride=1, pad=0, dil=1, act=_lib.ACT_NONE, residual=None):
    """y = residual + act(conv(x, W) + bias) on the tensor cores (group 1; W is a runtime.ConvWeights)."""
    n, c, h, wd, xs = _nchw(x)
    _, m, oh, ow, ys = _nchw(y)
    rs = 0 if residual is None else _nchw(residual)[4]
    call("osc_conv2d_ex_f32", ctx.handle, ptr(x), xs, n, c, h, wd, w.handle, stride, stride, pad, pad, pad, pad, dil,
         dil, ptr(bias), int(act), ptr(residual), rs, ptr(y), ys, oh, ow)
    return y


def conv2d_direct(ctx, x, w, bias, y, stride=1, pad=0, dil=1, group=1, act=_lib.ACT_NONE, residual=None):
    """Direct conv on CUDA cores (depthwise / first layer); w is the raw [M, C/g, kh, kw] device tensor."""
    n, c, h, wd, xs = _nchw(x)
    _, m, oh, ow, ys = _nchw(y)
    rs = 0 if residual is None else _nchw(residual)[4]
    kh, kw = int(w.shape[2]), int(w.shape[3])
    call("osc_conv2d_direct_f32", ctx.handle, ptr(x), xs, n, c, h, wd, ptr(w), m, kh, kw, stride, stride, pad, pad,
         pad, pad, dil, dil, group, ptr(bias), int(act), ptr(residual), rs, ptr(y), ys, oh, ow)
    return y


def maxpool2d(ctx, x, y, k, stride, pad):
    n, c, h, w, xs = _nchw(x)
    _, _, oh, ow, ys = _nchw(y)
    call("osc_maxpool2d_f32", ctx.handle, ptr(x), xs, n, c, h, w, k, k, stride, stride, pad, pad, pad, pad, ptr(y), ys,
         oh, ow)
    return y


def resize_nearest(ctx, x, y, scale=2):
    n, c, h, w, xs = _nchw(x)
    ys = _nchw(y)[4]
    call("osc_resize_nearest_f32", ctx.handle, ptr(x), xs, n, c, h, w, scale, scale, ptr(y), ys)
    return y


def binary(ctx, op, a, b, y):
    """y = a (op) b with numpy broadcasting (dense tensors, rank <= 4)."""
    ash = (C.c_longlong * max(1, a.dim()))(*a.shape)
    bsh = (C.c_longlong * max(1, b.dim()))(*b.shape)
    call("osc_binary_f32", ctx.handle, int(op), ptr(a), ash, a.dim(), ptr(b), bsh, b.dim(), ptr(y))
    return y


def unary(ctx, x, y, act):
    call("osc_unary_f32", ctx.handle, ptr(x), ptr(y), x.numel(), int(act))
    return y


def softmax(ctx, x, y):
    """Softmax over the last axis."""
    call("osc_softmax_f32", ctx.handle, ptr(x), ptr(y), x.numel() // x.shape[-1], int(x.shape[-1]))
    return y


def dfl(ctx, x, out, bins=16):
    b, cb, n = x.shape
    call("osc_dfl_f32", ctx.handle, ptr(x), b, cb // bins, bins, n, ptr(out))
    return out


def layernorm(ctx, x, gamma, beta, eps, y, inner=None):
    inner = int(inner or x.shape[-1])
    call("osc_layernorm_f32", ctx.handle, ptr(x), x.numel() // inner, inner, ptr(gamma), ptr(beta), float(eps), ptr(y))
    return y


def psa_attention(ctx, qkv, out, heads, kd, hd, scale):
    """qkv [B, heads*(2kd+hd), H, W] (view) -> out [B, heads*hd, H, W] (view)."""
    n, _, h, w, qs = _nchw(qkv)
    os_ = _nchw(out)[4]
    call("osc_psa_attention_f32", ctx.handle, ptr(qkv), qs, n, heads, kd, hd, h * w, float(scale), ptr(out), os_)
    return out


def yolo_decode(ctx, boxes, classes, strides, out):
    """boxes[i] [B, 64, h, w], classes[i] [B, nc, h, w] (views) -> out [B, 4+nc, A]."""
    B = int(boxes[0].shape[0])
    nc = int(classes[0].shape[1])
    bp = (C.c_void_p * 3)(*[ptr(t) for t in boxes])
    cp = (C.c_void_p * 3)(*[ptr(t) for t in classes])
    bs = (C.c_longlong * 3)(*[t.stride(0) for t in boxes])
    cs = (C.c_longlong * 3)(*[t.stride(0) for t in classes])
    hs = (C.c_int * 3)(*[int(t.shape[2]) for t in boxes])
    ws = (C.c_int * 3)(*[int(t.shape[3]) for t in boxes])
    st = (C.c_float * 3)(*[float(s) for s in strides])
    call("osc_yolo_decode_f32", ctx.handle, B, nc, bp, bs, cp, cs, hs, ws, st, ptr(out))
    return out


def letterbox(ctx, pixels, dst, bgr: bool = False):
    """Letterbox an [H, W, 3|4] uint8 device image into dst [3, th, tw] (a slice of the batch
    input); returns the placement (resized_w, resized_h, offset_x, offset_y)."""
    h, w, bpp = pixels.shape
    _, th, tw = dst.shape
    pl = (C.c_int * 4)()
    call("osc_letterbox_u8", ctx.handle, ptr(pixels), w, h, int(pixels.stride(0)), bpp, int(bgr), tw, th, ptr(dst), pl)
    return tuple(pl)


def letterbox_batch(ctx, frames, dst, bgr: bool = False):
    """Letterbox a [B, H, W, 3|4] uint8 device batch of frames into dst [B, 3, th, tw] (or channel-
    complete views of it) in one launch; returns the placement shared by every frame."""
    B, h, w, bpp = frames.shape
    _, _, th, tw = dst.shape
    pl = (C.c_int * 4)()
    call("osc_letterbox_batch_u8", ctx.handle, ptr(frames), B, int(frames.stride(0)), w, h, int(frames.stride(1)),
         bpp, int(bgr), tw, th, ptr(dst), int(dst.stride(0)), pl)
    return tuple(pl)


def yolo_detect_into(ctx, output, dets, counts, conf: float = 0.25, iou: float = 0.45, max_candidates: int = 30000,
                     class_agnostic: bool = False, transforms=None):
    """osc_yolo_detect_f32 into caller buffers dets [B, max_det, 6] and counts [B] (int32)."""
    B, fields, anchors = output.shape
    call("osc_yolo_detect_f32", ctx.handle, ptr(output), B, fields, anchors, float(conf), float(iou),
         int(dets.shape[1]), max_candidates, int(class_agnostic), ptr(transforms), ptr(dets), ptr(counts))


def yolo_detect(ctx, output, conf: float = 0.25, iou: float = 0.45, max_det: int = 300, max_candidates: int = 30000,
                class_agnostic: bool = False, transforms=None):
    """Detections of a [B, 4 + nc, A] output: (dets [B, max_det, 6] (class, score, x, y, w, h), counts [B])."""
    import torch

    B, fields, anchors = output.shape
    dets = torch.zeros((B, max_det, 6), dtype=torch.float32, device=output.device)
    counts = torch.zeros(B, dtype=torch.int32, device=output.device)
    call("osc_yolo_detect_f32", ctx.handle, ptr(output), B, fields, anchors, float(conf), float(iou), max_det,
         max_candidates, int(class_agnostic), ptr(transforms), ptr(dets), ptr(counts))
    return dets, counts
