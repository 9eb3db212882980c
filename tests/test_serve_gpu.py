"""Frames in, detections out (onnxsharp_b200.serve.DetectPipeline): the
batched letterbox matches the per-frame one bit for bit, and every pipelined
batch's detections equal the same steps run one by one (letterbox each frame,
forward, decode + NMS mapped back to the source frame), including when the
pipeline's slots are reused. The per-step kernels themselves are checked
against the oracle in test_detect_gpu.py and test_yolo_batches_gpu.py."""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_letterbox_batch_equals_per_frame(ctx):
    import torch

    from onnxsharp_b200 import ops

    rng = np.random.default_rng(12)
    frames = torch.from_numpy(rng.integers(0, 256, (3, 480, 800, 3), dtype=np.uint8)).cuda()
    dst = torch.full((3, 3, 640, 640), float("nan"), device="cuda")
    pl = ops.letterbox_batch(ctx, frames, dst, bgr=True)
    one = torch.empty((3, 640, 640), device="cuda")
    for i in range(3):
        assert ops.letterbox(ctx, frames[i], one, bgr=True) == pl
        ctx.synchronize()
        assert torch.equal(dst[i].view(torch.int32), one.view(torch.int32)), f"frame {i}"


def test_detect_pipeline_matches_stepwise(ctx):
    import torch

    from onnxsharp_b200 import ops, yolo
    from onnxsharp_b200.serve import DetectPipeline

    g = yolo.build_yolo11n()
    params = yolo.init_params(g, 21)
    B, hw = 2, (360, 640)
    rng = np.random.default_rng(13)
    batches = [rng.integers(0, 256, (B,) + hw + (3,), dtype=np.uint8) for _ in range(3)]

    # step by step on a separate plan
    ref_net = yolo.Net(ctx, g, params, B)
    want = []
    for fr in batches:
        dev = torch.from_numpy(fr).cuda()
        for i in range(B):
            pl = ops.letterbox(ctx, dev[i], ref_net.input_view()[i], bgr=True)
        out = ref_net.forward(use_graph=False)
        tr = torch.tensor([[pl[0], pl[1], pl[2], pl[3], hw[1], hw[0]]] * B, dtype=torch.float32, device="cuda")
        dets, counts = ops.yolo_detect(ctx, out, conf=0.25, iou=0.45, max_det=300, transforms=tr)
        ctx.synchronize()
        want.append([dets[i, : counts[i]].cpu().numpy() for i in range(B)])
    ref_net.close()

    net = yolo.Net(ctx, g, params, B)
    pipe = DetectPipeline(net, frame_hw=hw, bgr=True, depth=2)
    results = []
    for fr in batches + batches[:1]:  # the 4th batch reuses slot 1's buffers after slot 0's
        f, r = pipe.host_buffers()
        f.copy_(torch.from_numpy(fr))
        pipe.submit(f, r)
        results.append((f, r))
    pipe.synchronize()
    for k, (_, r) in enumerate(results):
        got = pipe.unpack(r.numpy())
        ref = want[k % 3]
        assert len(got) == B
        for i in range(B):
            assert got[i].shape == ref[i].shape and got[i].shape[0] > 0, (k, i)
            assert np.array_equal(got[i].view(np.uint32), ref[i].view(np.uint32)), (k, i)
    net.close()
