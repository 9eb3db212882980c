"""CPU oracle executor of the YOLO11n-shaped plan (onnxsharp_b200.yolo.Graph)
and the reference's detection post-processing.

TEST INFRASTRUCTURE ONLY: runs the same IR node by node with the oracle's
restatements of the reference's CPU kernels (conv im2col order + VectorMath
SiLU, MaxPool, nearest Resize, the PSA MatMul/Softmax chain, DflSoftmax and
the exported dist2bbox op order) to check the CUDA executor; never imported by
the product.

Post-processing restates YoloDecoder.Decode (src/OnnxSharp/Vision/YoloDecoder.cs:68-188,
channels-first raw head: best class score >= confidence, cx/cy/w/h -> x/y/w/h)
and DetectionNms.Suppress (src/OnnxSharp/Vision/Detection.cs:62-107: score
order, per-class suppression when IoU > threshold, Detection.IoU :31-50).
The reference sorts with an unstable sort; here ties keep anchor order.
"""
from __future__ import annotations

import numpy as np

import oracle


def _maxpool(x, k, s, p):
    n, c, h, w = x.shape
    oh, ow = (h + 2 * p - k) // s + 1, (w + 2 * p - k) // s + 1
    xp = np.full((n, c, h + 2 * p, w + 2 * p), -np.inf, np.float32)
    xp[:, :, p:p + h, p:p + w] = x
    out = np.full((n, c, oh, ow), -np.inf, np.float32)
    for ky in range(k):
        for kx in range(k):
            out = np.maximum(out, xp[:, :, ky:ky + s * oh:s, kx:kx + s * ow:s])
    return out


def _psa(qkv, heads, kd, hd, scale, threads):
    n, _, h, w = qkv.shape
    t = h * w
    out = np.empty((n, heads * hd, h, w), np.float32)
    per = 2 * kd + hd
    for b in range(n):
        for hh in range(heads):
            blk = qkv[b, hh * per:(hh + 1) * per].reshape(per, t)
            q, k, v = blk[:kd], blk[kd:2 * kd], blk[2 * kd:]
            s = oracle.gemm(np.ascontiguousarray(q.T), np.ascontiguousarray(k), threads=threads)  # MatMul
            s = (s * np.float32(scale)).astype(np.float32)                                        # Mul
            p = oracle.softmax(s, threads=threads)                                                # Softmax
            o = oracle.gemm(np.ascontiguousarray(v), np.ascontiguousarray(p.T), threads=threads)  # MatMul v @ P^T
            out[b, hh * hd:(hh + 1) * hd] = o.reshape(hd, h, w)
    return out


def _decode(boxes, classes, strides, threads):
    n = boxes[0].shape[0]
    box = np.concatenate([b.reshape(n, 64, -1) for b in boxes], axis=2)       # Concat_3 / Split (box part)
    cls = np.concatenate([c.reshape(n, c.shape[1], -1) for c in classes], axis=2)
    dist = oracle.dfl(box, 16, threads=threads)                                # DflSoftmax -> [n, 4, A]
    ax, ay, st = [], [], []
    for b, s in zip(boxes, strides):
        h, w = b.shape[2:]
        yy, xx = np.meshgrid(np.arange(h, dtype=np.float32) + np.float32(0.5),
                             np.arange(w, dtype=np.float32) + np.float32(0.5), indexing="ij")
        ax.append(xx.ravel())
        ay.append(yy.ravel())
        st.append(np.full(h * w, s, np.float32))
    anc = np.stack([np.concatenate(ax), np.concatenate(ay)])[None]            # [1, 2, A]
    stride = np.concatenate(st)[None, None]
    lt, rb = dist[:, :2], dist[:, 2:]                                          # Slice, Slice_1
    x1y1 = (anc - lt).astype(np.float32)                                       # Sub
    x2y2 = (anc + rb).astype(np.float32)                                       # Add_1
    c_xy = ((x1y1 + x2y2).astype(np.float32) / np.float32(2)).astype(np.float32)  # Add_2, Div_1
    wh = (x2y2 - x1y1).astype(np.float32)                                      # Sub_1
    dbox = (np.concatenate([c_xy, wh], 1) * stride).astype(np.float32)         # Concat_4, Mul_2
    return np.concatenate([dbox, oracle.unary(cls, 3, threads=threads)], 1)   # Sigmoid, Concat


_BUFS: dict = {}


def run(g, params: dict, images: np.ndarray, threads: int = 0) -> np.ndarray:
    """Run the plan on [B, 3, H, W] images; returns [B, 4 + nc, A]."""
    n = images.shape[0]
    # the activation buffers, allocated once per (graph, batch) like the
    # reference's arena; every element is written by its producer before use
    key = (id(g), n)
    if key not in _BUFS:
        _BUFS.clear()
        _BUFS[key] = {name: np.empty((n, c, h, w), np.float32) for name, (c, h, w) in g.buffers.items()}
    bufs = _BUFS[key]
    bufs[g.input][...] = images

    def view(r):
        return bufs[r.buf][:, r.c0:r.c0 + r.c]

    out = None
    for node in g.nodes:
        a = node.attrs
        if node.op == "conv":
            x = np.ascontiguousarray(view(node.ins[0]))
            k, s, p = a["k"], a["s"], a["p"]
            dst = view(node.outs[0])
            direct = dst.flags.c_contiguous and not a["residual"]   # a channel slice of one image is contiguous
            y = oracle.conv2d(x, params[node.name + ".w"], params[node.name + ".b"], (s, s), (p, p, p, p), (1, 1),
                              a["group"], a["act"], threads=threads, out=dst if direct else None)
            if a["residual"]:
                np.add(view(node.ins[1]), y, out=y)   # Add(x, act(conv)), float32
            if not direct:
                dst[...] = y
        elif node.op == "maxpool":
            view(node.outs[0])[...] = _maxpool(view(node.ins[0]), a["k"], a["s"], a["p"])
        elif node.op == "upsample":
            sc = a["scale"]
            view(node.outs[0])[...] = np.repeat(np.repeat(view(node.ins[0]), sc, axis=2), sc, axis=3)
        elif node.op == "psa":
            view(node.outs[0])[...] = _psa(np.ascontiguousarray(view(node.ins[0])), a["heads"], a["kd"], a["hd"],
                                           a["scale"], threads)
        elif node.op == "decode":
            k = len(node.ins) // 2
            out = _decode([np.ascontiguousarray(view(r)) for r in node.ins[:k]],
                          [np.ascontiguousarray(view(r)) for r in node.ins[k:]], a["strides"], threads)
        else:  # pragma: no cover
            raise ValueError(node.op)
    return out


def iou(a, b) -> float:
    """Detection.IoU (Detection.cs:31-50) on (x, y, w, h) float32 boxes."""
    f = np.float32
    x1 = max(f(a[0]), f(b[0]))
    y1 = max(f(a[1]), f(b[1]))
    x2 = min(f(a[0] + a[2]), f(b[0] + b[2]))
    y2 = min(f(a[1] + a[3]), f(b[1] + b[3]))
    iw, ih = f(x2 - x1), f(y2 - y1)
    if iw <= 0 or ih <= 0:
        return 0.0
    inter = f(iw * ih)
    union = f(f(f(a[2] * a[3]) + f(b[2] * b[3])) - inter)
    return 0.0 if union <= 0 else float(f(inter / union))


def detect(output: np.ndarray, conf: float = 0.25, iou_thr: float = 0.45, max_det: int = 300,
           max_candidates: int = 30000, class_agnostic: bool = False) -> list[tuple]:
    """YoloDecoder.Decode + DetectionNms.Suppress for one image's [4 + nc, A] output.
    Returns (class, score, x, y, w, h, anchor) tuples in NMS order."""
    f = np.float32
    nc = output.shape[0] - 4
    scores = output[4:]
    cls = np.argmax(scores, axis=0)  # first maximum, as the strict '>' scan
    best = scores[cls, np.arange(output.shape[1])]
    cands = []
    for a in np.nonzero(np.isfinite(best) & (best >= f(conf)))[0]:
        x, y, w, h = (f(v) for v in output[:4, a])
        if not all(np.isfinite([x, y, w, h])):
            continue
        x = f(x - f(w * f(0.5)))
        y = f(y - f(h * f(0.5)))
        if w <= 0 or h <= 0:
            continue
        cands.append((int(cls[a]), float(best[a]), float(x), float(y), float(w), float(h), int(a)))
    cands.sort(key=lambda d: (-d[1], d[6]))
    cands = cands[:max_candidates]
    kept = []
    for c in cands:
        if any((class_agnostic or k[0] == c[0]) and iou(k[2:6], c[2:6]) > iou_thr for k in kept):
            continue
        kept.append(c)
        if len(kept) >= max_det:
            break
    _ = nc
    return kept


def to_source(kept, placement, src_w: int, src_h: int) -> list[tuple]:
    """YoloDecoder.Decode's last step (YoloDecoder.cs:170-186): letterbox boxes back to the
    source image (Letterbox.ToSourceX/Y, ImagePreprocessor.cs:16-18), clamped, zero-area dropped."""
    f = np.float32
    rw, rh, ox, oy = placement
    sx, sy = f(f(rw) / f(src_w)), f(f(rh) / f(src_h))
    out = []
    for cls, score, x, y, w, h, a in kept:
        def clamp(v, hi):
            return f(min(max(v, f(0)), f(hi)))
        x1 = clamp(f(f(f(x) - f(ox)) / sx), src_w)
        y1 = clamp(f(f(f(y) - f(oy)) / sy), src_h)
        x2 = clamp(f(f(f(f(x) + f(w)) - f(ox)) / sx), src_w)
        y2 = clamp(f(f(f(f(y) + f(h)) - f(oy)) / sy), src_h)
        if x2 <= x1 or y2 <= y1:
            continue
        out.append((cls, score, float(x1), float(y1), float(f(x2 - x1)), float(f(y2 - y1)), a))
    return out
