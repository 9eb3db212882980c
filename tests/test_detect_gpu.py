"""The steps either side of the YOLO forward on the B200: letterbox
pre-processing (bit-identical to ImagePreprocessor.Letterbox) and the detect
tail (YoloDecoder.Decode + DetectionNms.SuppressSorted): identical detection
lists to the oracle, in letterbox and in source coordinates."""
from __future__ import annotations

import numpy as np
import pytest

import oracle
from oracle import yolo_ref

pytestmark = pytest.mark.gpu


def T(a):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("h,w,bpp,bgr,pad", [
    (480, 640, 3, False, 0),    # 4:3 frame: bars top and bottom
    (720, 1280, 3, True, 0),    # BGR 16:9
    (500, 300, 4, False, 8),    # RGBA, portrait, padded rows
    (640, 640, 3, False, 0),    # already square: identity placement
    (37, 1001, 3, True, 0),     # extreme aspect ratio
])
def test_letterbox_bit_exact(ctx, h, w, bpp, bgr, pad):
    import torch

    from onnxsharp_b200 import ops

    rng = np.random.default_rng(h * w)
    img = rng.integers(0, 256, (h, w, bpp)).astype(np.uint8)
    ref, ref_pl = oracle.letterbox(img, bgr=bgr)
    dev = torch.zeros((h, w * bpp + pad), dtype=torch.uint8, device="cuda")
    dev[:, : w * bpp] = T(img.reshape(h, w * bpp))
    pix = dev[:, : w * bpp].view(h, w, bpp)
    dst = torch.empty((2, 3, 640, 640), device="cuda")
    pl = ops.letterbox(ctx, pix, dst[1], bgr=bgr)
    ctx.synchronize()
    assert pl == ref_pl
    assert np.array_equal(dst[1].cpu().numpy().view(np.uint32), ref.view(np.uint32))


def _synthetic_output(rng, anchors=8400, nc=80):
    """A plausible detect-head output: boxes spread over the 640 x 640 canvas,
    class scores in (0, 1) with a few confident anchors and clusters of
    overlapping boxes (so NMS has work)."""
    out = np.zeros((4 + nc, anchors), np.float32)
    centres = rng.uniform(40, 600, (60, 2))
    pick = rng.integers(0, 60, anchors)
    out[0] = centres[pick, 0] + rng.normal(0, 6, anchors)
    out[1] = centres[pick, 1] + rng.normal(0, 6, anchors)
    out[2] = rng.uniform(10, 120, anchors)
    out[3] = rng.uniform(10, 120, anchors)
    scores = rng.uniform(0, 0.3, (nc, anchors)).astype(np.float32)
    hot = rng.integers(0, anchors, 2000)
    scores[rng.integers(0, nc, 2000), hot] = rng.uniform(0.3, 1.0, 2000)
    out[4:] = scores
    return out.astype(np.float32)


@pytest.mark.parametrize("with_transform", [False, True])
def test_detect_matches_oracle(ctx, with_transform):
    from onnxsharp_b200 import ops

    rng = np.random.default_rng(7 + with_transform)
    outs = np.stack([_synthetic_output(rng) for _ in range(3)])
    placements = [(640, 480, 0, 80, 640, 480), (360, 640, 140, 0, 720, 1280), (640, 640, 0, 0, 640, 640)]
    tf = np.array(placements, np.float32) if with_transform else None
    dets, counts = ops.yolo_detect(ctx, T(outs), conf=0.25, iou=0.45, max_det=300,
                                   transforms=None if tf is None else T(tf))
    ctx.synchronize()
    dets, counts = dets.cpu().numpy(), counts.cpu().numpy()
    for i in range(3):
        kept = yolo_ref.detect(outs[i], conf=0.25, iou_thr=0.45, max_det=300)
        if with_transform:
            rw, rh, ox, oy, sw, sh = placements[i]
            kept = yolo_ref.to_source(kept, (rw, rh, ox, oy), sw, sh)
        assert counts[i] == len(kept) > 0
        got = dets[i, : counts[i]]
        assert got[:, 0].astype(int).tolist() == [k[0] for k in kept]
        ref = np.array([k[1:6] for k in kept], np.float32)
        assert np.array_equal(got[:, 1:].view(np.uint32), ref.view(np.uint32))


def test_detect_caps_and_empty(ctx):
    """max_det caps the kept list; an image with no confident anchor gives no detection."""
    from onnxsharp_b200 import ops

    rng = np.random.default_rng(11)
    outs = np.stack([_synthetic_output(rng), _synthetic_output(rng)])
    outs[1, 4:] = 0.1
    dets, counts = ops.yolo_detect(ctx, T(outs), conf=0.25, iou=0.45, max_det=5)
    ctx.synchronize()
    counts = counts.cpu().numpy()
    ref = yolo_ref.detect(outs[0], conf=0.25, iou_thr=0.45, max_det=5)
    assert counts.tolist() == [len(ref), 0] and len(ref) == 5
    assert dets.cpu().numpy()[0, :5, 0].astype(int).tolist() == [k[0] for k in ref]


@pytest.mark.parametrize("case", ["dense_capped", "dense_uncapped", "agnostic"])
def test_detect_dense_candidates_match_oracle(ctx, case):
    """Every anchor a candidate (as with random-init weights, scores in a narrow
    band): the block-parallel greedy NMS walks several 1024-candidate chunks
    and must keep exactly the boxes of the one-at-a-time loop, in order."""
    from onnxsharp_b200 import ops

    rng = np.random.default_rng(31)
    out = _synthetic_output(rng)
    out[4:] = rng.uniform(0.2, 0.6, out[4:].shape).astype(np.float32)
    out[2:4] = rng.uniform(4, 40, (2, out.shape[1])).astype(np.float32)  # small boxes: many survive
    max_det = {"dense_capped": 300, "dense_uncapped": 1024, "agnostic": 300}[case]
    agn = case == "agnostic"
    dets, counts = ops.yolo_detect(ctx, T(out[None]), conf=0.25, iou=0.45, max_det=max_det, class_agnostic=agn)
    ctx.synchronize()
    kept = yolo_ref.detect(out, conf=0.25, iou_thr=0.45, max_det=max_det, class_agnostic=agn)
    n = int(counts.cpu().numpy()[0])
    assert n == len(kept) > 0
    got = dets.cpu().numpy()[0, :n]
    assert got[:, 0].astype(int).tolist() == [k[0] for k in kept]
    ref = np.array([k[1:6] for k in kept], np.float32)
    assert np.array_equal(got[:, 1:].view(np.uint32), ref.view(np.uint32))
