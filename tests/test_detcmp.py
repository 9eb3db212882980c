"""The detection comparator (tests/detcmp.py) itself, on CPU: it accepts an
output that differs from the oracle's by rounding-level noise (reporting the
ties it meets) and rejects outputs with a planted error in a box or a score."""
from __future__ import annotations

import numpy as np
import pytest

from detcmp import compare_detections


@pytest.fixture(scope="module")
def ref():
    from oracle import yolo_ref
    from onnxsharp_b200 import yolo

    g = yolo.build_yolo11n()
    images = np.random.default_rng(3).uniform(0, 1, (1, 3, 640, 640)).astype(np.float32)
    return yolo_ref.run(g, yolo.init_params(g, 11), images)[0]


def test_identical_outputs_agree(ref):
    rep, bad = compare_detections(ref, ref)
    assert not bad and rep["identical"] and rep["kept"] == 300


def test_rounding_noise_is_flagged_not_failed(ref):
    rng = np.random.default_rng(0)
    noisy = ref.copy()
    noisy[4:] += rng.uniform(-1.2e-7, 1.2e-7, noisy[4:].shape).astype(np.float32)
    noisy[:4] *= (1 + rng.uniform(-2e-6, 2e-6, noisy[:4].shape)).astype(np.float32)
    rep, bad = compare_detections(noisy, ref)
    assert not bad, bad[:5]


def test_planted_box_error_is_caught(ref):
    from detcmp import _candidates

    bad_out = ref.copy()
    _, best, _, _ = _candidates(ref)
    top = np.argsort(-best)[:50]
    bad_out[2:4, top] *= 1.5  # widen the 50 best boxes: suppression decisions change
    _, bad = compare_detections(bad_out, ref)
    assert bad


def test_planted_score_error_is_caught(ref):
    bad_out = ref.copy()
    bad_out[4:, :100] += 1e-3  # far beyond the tie tolerance: the order changes
    _, bad = compare_detections(bad_out, ref)
    assert bad
