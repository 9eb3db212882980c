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


# ---------------------------------------------------------------- node-by-node shape check
TSV = __import__("conftest").GOLDEN / "yolo11n.shapes.tsv"


def _tsv_tensors():
    """(node index, op type, tensor name, shape without the batch dim) of every TENSOR row."""
    rows = []
    for line in TSV.read_text().splitlines():
        idx, kind, op, name, _batch, shape = line.split("\t")
        if kind == "TENSOR":
            dims = tuple(int(v) for v in shape.split(","))
            assert dims[0] == 1, line  # the table is recorded at batch 1
            rows.append((int(idx), op, name.lstrip("/"), dims[1:]))
    return rows


def _ir_shape(g, name, op):
    """The shape our IR gives the exported tensor `name` (per image), or raises KeyError.

    Convs keep their names: the exported module path minus the trailing
    conv/Conv and minus every segment the next one extends ("m" before "m.0",
    "ffn" before "ffn.0", "cv3.0" before "cv3.0.0"); activations, residual Adds, Splits and Concats
    are fused into convs or are channel slices of buffers, so their shapes are
    those of the conv output / slice / buffer that stands for them; the C2PSA
    attention and Detect-tail internals follow from the psa / decode nodes'
    attributes."""
    convs = {n.name: n for n in g.nodes if n.op == "conv"}
    psa = next(n for n in g.nodes if n.op == "psa")
    dec = next(n for n in g.nodes if n.op == "decode")
    A = sum((640 // s) ** 2 for s in g.strides)
    nc = dec.attrs["nc"]
    heads, kd, hd = psa.attrs["heads"], psa.attrs["kd"], psa.attrs["hd"]
    ph, pw = g.hw(psa.ins[0])
    T = ph * pw

    def out(n):
        r = n.outs[0]
        return (r.c,) + g.hw(r)

    def conv_shape(path):
        seg = path.split("/")
        if seg[-1] == "conv":
            seg = seg[:-1]
        key = ".".join(s for s, nxt in zip(seg, seg[1:] + [""]) if not nxt.startswith(s + "."))
        if key in convs:
            return out(convs[key]), convs[key]
        parts = [convs[k] for k in convs if k.startswith(key + ".")]  # per-head slices of one conv
        if not parts:
            raise KeyError(name)
        refs = sorted((p.outs[0] for p in parts), key=lambda r: r.c0)
        assert all(r.buf == refs[0].buf for r in refs)
        assert all(a.c0 + a.c == b.c0 for a, b in zip(refs, refs[1:]))
        return (sum(r.c for r in refs),) + g.hw(refs[0]), parts[0]

    path, leaf = name.rsplit("/", 1) if "/" in name else ("", name)
    seg = path.split("/") if path else []
    top = seg[0] if seg else ""
    scale = {"": 0, "_1": 1, "_2": 2}
    if name == "output0":
        return (4 + nc, A)
    if op == "Conv":
        if seg[:2] == ["model.23", "dfl"]:
            return (1, 4, A)
        return conv_shape(path)[0]
    if op in ("Sigmoid", "Mul") and seg and seg[-1] == "act":
        return conv_shape("/".join(seg[:-1]))[0]
    if top == "model.23":
        if seg[1:] == ["dfl"]:
            return {"Reshape_output_0": (4, 16, A), "Transpose_output_0": (16, 4, A), "Softmax_output_0": (16, 4, A),
                    "Reshape_1_output_0": (4, A)}[leaf]
        stem = leaf[: leaf.index("_output")]
        if op in ("Concat", "Reshape") and stem.split("_")[0] in ("Concat", "Reshape") and stem[len(op):] in scale:
            s = g.strides[scale[stem[len(op):]]]
            hw = (640 // s, 640 // s)
            return (64 + nc,) + (hw if op == "Concat" else (hw[0] * hw[1],))
        return {"Concat_3": (64 + nc, A), "Concat_4": (4, A), "Mul_2": (4, A), "Sigmoid": (nc, A),
                "Slice": (2, A), "Slice_1": (2, A), "Sub": (2, A), "Sub_1": (2, A), "Add_1": (2, A), "Add_2": (2, A),
                "Div_1": (2, A)}.get(stem) or {"Split_output_0": (64, A), "Split_output_1": (nc, A)}[leaf]
    if seg[-2:] == ["m.0", "attn"] and top == "model.10":
        stem = leaf[: leaf.index("_output")]
        return {"Reshape": (heads, 2 * kd + hd, T), "Transpose": (heads, T, kd), "MatMul": (heads, T, T),
                "Mul": (heads, T, T), "Softmax": (heads, T, T), "Transpose_1": (heads, T, T),
                "MatMul_1": (heads, hd, T), "Reshape_1": (heads * hd, ph, pw), "Reshape_2": (heads * hd, ph, pw),
                "Add": out(psa)}.get(stem) or {"Split_output_0": (heads, kd, T), "Split_output_1": (heads, kd, T),
                                              "Split_output_2": (heads, hd, T)}[leaf]
    if op == "Split" and len(seg) == 1:
        c, h, w = out(convs[top + ".cv1"])
        return (c // 2, h, w)
    if op == "Add":
        if top == "model.10" and leaf.startswith("Add_output"):             # attn.proj + x
            shape, node = conv_shape("model.10/m/m.0/attn/proj")
        elif top == "model.10" and leaf.startswith("Add_1"):                # ffn + x
            shape, node = conv_shape("model.10/m/m.0/ffn/ffn.1")
        elif leaf.startswith("Add_output") and seg[-1].startswith("m."):   # bottleneck shortcut
            shape, node = conv_shape(path + "/cv2")
        else:
            raise KeyError(name)
        assert node.attrs["residual"], f"{name}: the Add is not fused into {node.name}"
        return shape
    if op == "Concat":
        if len(seg) == 1 and top.split(".")[1] in ("12", "15", "18", "21"):  # neck Concat modules
            return g.buffers["cat" + top.split(".")[1]]
        return g.buffers[".".join(s for s in seg if s != "m") + ".cat"]
    if op == "MaxPool":
        suffix = {"m": 0, "m_1": 1, "m_2": 2}[seg[-1]]
        return out(next(n for n in g.nodes if n.name == f"{top}.m{suffix}"))
    if op == "Resize":
        return out(next(n for n in g.nodes if n.name == top))
    raise KeyError(name)


def test_graph_matches_reference_shape_table_node_by_node():
    """Every tensor of the reference's tests/data/yolo11n.shapes.tsv (the exported
    YOLO11n at batch 1) has the same shape in the plan's IR, and every conv of
    the IR stands for an exported Conv."""
    g = yolo.build_yolo11n()
    rows = _tsv_tensors()
    assert len(rows) == 332
    bad, seen_convs = [], set()
    for idx, op, name, shape in rows:
        try:
            got = tuple(_ir_shape(g, name, op))
        except KeyError:
            bad.append((idx, name, "unmapped"))
            continue
        if got != shape:
            bad.append((idx, name, f"IR {got} != table {shape}"))
        if op == "Conv":
            seen_convs.add(name)
    assert not bad, bad[:10]
    assert len(seen_convs) == 88
    ir_convs = [n.name for n in g.nodes if n.op == "conv"]
    # the exported graph's 88 Convs = our 87 conv names (the 128-channel PSA
    # position encoding runs as 2 per-head depthwise convs) + the DFL 1x1 (in decode)
    assert len(ir_convs) == 88 and sum(1 for n in ir_convs if ".attn.pe." in n) == 2


def test_native_arena_colouring_matches_reference_rule():
    """osc_arena_assign (the colouring osc_plan_build uses, run on the host) gives
    the same offsets as the BufferAllocator restatement in arena.py, on the YOLO
    plan's live ranges and on random ones."""
    import random

    from onnxsharp_b200 import plan

    g = yolo.build_yolo11n()
    names, first, last = yolo.buffer_lifetimes(g)
    sizes = [64 * 4 * int(np.prod(g.buffers[n])) for n in names]
    f, l_ = [first[n] for n in names], [last[n] for n in names]
    want_off, want_total = arena.plan_offsets([arena.Lifetime(a, b, c) for a, b, c in zip(f, l_, sizes)])
    got_off, got_total = plan.arena_assign(f, l_, sizes)
    assert got_off == want_off and got_total == want_total
    rnd = random.Random(5)
    for _ in range(200):
        n = rnd.randint(1, 30)
        f = [rnd.randint(-1, 20) for _ in range(n)]
        l_ = [max(0, x + rnd.randint(0, 6)) for x in f]
        sz = [rnd.randint(1, 5000) for _ in range(n)]
        want = arena.plan_offsets([arena.Lifetime(a, b, c) for a, b, c in zip(f, l_, sz)])
        assert plan.arena_assign(f, l_, sz) == (list(want[0]), want[1])


def test_concurrent_lanes_arena_is_race_free():
    """With the Detect head's branches on their own streams, two buffers may
    share arena memory only when every node touching one happens before the
    first writer of the other (data dependencies and stream order)."""
    g = yolo.build_yolo11n()
    lane_of = yolo.node_lanes(g, 3)
    assert set(lane_of) == {0, 1, 2}
    deps = yolo.node_deps(g)
    anc = yolo.happens_before(deps, lane_of)
    names, first, last = yolo.buffer_lifetimes(g)
    touch = {n: 0 for n in names}
    for i, node in enumerate(g.nodes):
        for r in list(node.ins) + list(node.outs):
            if r.buf in touch:
                touch[r.buf] |= 1 << i
    sizes = {n: 4 * int(np.prod(g.buffers[n])) for n in names}
    lts = [arena.Lifetime(first[n], last[n], sizes[n]) for n in names]
    offs, _ = arena.plan_offsets_dag(lts, [touch[n] for n in names], anc)
    for (i, a), (j, b) in itertools.combinations(enumerate(names), 2):
        if offs[i] < 0 or offs[j] < 0:
            continue
        if not (offs[i] < offs[j] + sizes[b] and offs[j] < offs[i] + sizes[a]):
            continue
        a_before_b = touch[a] & ~anc[first[b]] == 0
        b_before_a = touch[b] & ~anc[first[a]] == 0
        assert a_before_b or b_before_a, (a, b)
    # the head branches depend only on their neck level: the 80x80 box branch
    # may run while the neck computes the 40x40 and 20x20 levels
    idx = {n.name: k for k, n in enumerate(g.nodes)}
    assert not anc[idx["model.23.cv2.0.0"]] >> idx["model.19.cv2"] & 1
