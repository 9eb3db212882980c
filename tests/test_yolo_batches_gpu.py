"""The YOLO11n-shaped plan at BASELINE config 5's batch sizes (B = 1, 8, 64)
against the CPU oracle running the same IR with the reference's kernels, and
the detections after the reference's decode + NMS at its DetectorOptions
defaults (confidence 0.25, IoU 0.45, Vision/YoloDecoder.cs:25-28).

The plan is specialised per batch size (one arena and one CUDA graph per B),
so each B is its own code path. Images checked: all at B = 1 and 8; 0, 31 and
63 at B = 64 (the oracle takes a fraction of a second per image).

Detections are compared decision by decision, with flags for near-threshold
and near-tie cases (tests/detcmp.py); the flag counts are printed per image."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import rel_err
from detcmp import compare_detections

pytestmark = pytest.mark.gpu


def _plan(ctx, g, params, images):
    import torch

    from onnxsharp_b200 import yolo

    net = yolo.Net(ctx, g, params, images.shape[0])
    net.input_view().copy_(torch.from_numpy(images))
    out = net.forward(use_graph=True).cpu().numpy()
    ctx.synchronize()
    net.close()
    return out


@pytest.fixture(scope="module")
def model():
    from onnxsharp_b200 import yolo

    g = yolo.build_yolo11n()
    return g, yolo.init_params(g, 11)


@pytest.mark.parametrize("batch,checked", [(1, (0,)), (8, tuple(range(8))), (64, (0, 31, 63))],
                         ids=["B1", "B8", "B64"])
def test_yolo_batch_matches_oracle_and_detections(ctx, model, batch, checked):
    from oracle import yolo_ref

    g, params = model
    images = np.random.default_rng(100 + batch).uniform(0, 1, (batch, 3, 640, 640)).astype(np.float32)
    out = _plan(ctx, g, params, images)
    assert out.shape == (batch, 84, 8400)
    assert np.all(np.isfinite(out))
    ref = yolo_ref.run(g, params, np.ascontiguousarray(images[list(checked)]))
    for j, i in enumerate(checked):
        assert rel_err(out[i, :4], ref[j, :4]) <= 1e-4, f"image {i}: boxes"
        assert np.max(np.abs(out[i, 4:] - ref[j, 4:])) <= 1e-4, f"image {i}: class scores"
        rep, bad = compare_detections(out[i], ref[j])
        print(f"B={batch} image {i}: {rep}")
        assert not bad, (i, bad[:5], rep)
