"""Host-side logic of the YOLO11n-shaped plan: graph structure against the
reference's shape table counts, FLOPs, and the device arena's lifetime
colouring (BufferAllocator.Assign semantics, mirroring the reference's
BufferAllocatorTests)."""
from __future__ import annotations

import itertools

import numpy as np

from onnxsharp_b200 import arena, yolo


def test_graph_matches_reference_op_counts():
    g = yolo.build_yolo11n()
    ops = yolo.count_ops(g)
    # tests/data/yolo11n.shapes.tsv: 88 Conv (incl. the DFL 1x1, fused here into
    # decode; the 128-ch PSA pe conv runs as 2 per-head depthwise convs), 3 MaxPool, 2 Resize.
    assert ops == {"conv": 88, "maxpool": 3, "upsample": 2, "psa": 1, "decode": 1}
    assert abs(yolo.flops_per_image(g) - 6.54e9) < 0.01e9


def test_graph_levels_and_output():
    g = yolo.build_yolo11n()
    assert g.buffers["m16"] == (64, 80, 80) and g.buffers["m19"] == (128, 40, 40) and g.buffers["m22"] == (256, 20, 20)
    assert sum((640 // s) ** 2 for s in g.strides) == 8400
    a = yolo.anchors(g)
    assert a.shape == (8400, 3) and a[0].tolist() == [0.5, 0.5, 8.0] and a[-1].tolist() == [19.5, 19.5, 32.0]


def test_params_he_normal():
    g = yolo.build_yolo11n()
    p = yolo.init_params(g, 1)
    w = p["model.8.cv2.w"]
    assert w.shape == (256, 384, 1, 1)
    assert abs(w.std() - np.sqrt(2 / 384)) < 0.01


def test_arena_strict_reuse_and_inplace():
    L = arena.Lifetime
    lts = [L(0, 1, 100), L(1, 2, 100), L(2, 3, 100), L(3, 4, 300)]
    slot, n = arena.assign_slots(lts)
    assert slot[0] != slot[1]          # overlapping at op 1
    assert slot[2] == slot[0]          # 0 is dead before op 2
    assert slot[3] == slot[1]          # strict '<': slot of buffer 2 (read at op 3) is not reused at op 3
    slot2, _ = arena.assign_slots(lts, inplace={1: 0})
    assert slot2[1] == slot2[0]
    offs, total = arena.plan_offsets(lts)
    assert total == 256 + 512 and all(o % 256 == 0 for o in offs)


def test_yolo_arena_never_overlaps_live_buffers():
    g = yolo.build_yolo11n()
    names, first, last = yolo.buffer_lifetimes(g)
    assert g.input not in names  # the input lives in the plan's slots, not the arena
    assert all(first[n] >= 0 and last[n] >= first[n] for n in names)
    sizes = {n: 4 * int(np.prod(g.buffers[n])) for n in names}
    lts = [arena.Lifetime(first[n], last[n], sizes[n]) for n in names]
    offs, total = arena.plan_offsets(lts)
    assert total < sum(sizes.values()) // 2  # colouring reuses memory
    for (i, a), (j, b) in itertools.combinations(enumerate(names), 2):
        if offs[i] < 0 or offs[j] < 0:
            continue
        live = not (max(last[a], first[a]) < first[b] or max(last[b], first[b]) < first[a])
        overlap = offs[i] < offs[j] + sizes[b] and offs[j] < offs[i] + sizes[a]
        assert not (live and overlap), (a, b)
