"""A random-init YOLO11n-shaped detector as a static plan.

The graph follows the node-by-node tensor shapes of the reference's
tests/data/yolo11n.shapes.tsv (input [B,3,640,640] -> output [B,84,8400];
88 Conv, 11 Split, 23 Concat, 16 Add, 3 MaxPool, 2 Resize, the C2PSA
attention and the Detect tail with DFL). Kernel sizes, strides and groups are
not recorded in that table; they are YOLO11n's (width 0.25, depth 0.5):
3x3 stride-2 convs at every spatial halving, 1x1 convs at C3k2 / SPPF /
C2PSA entries and exits, 3x3 bottlenecks, depthwise 3x3 in the class head
and in the PSA positional encoding, 1x1 heads. BN is folded into the convs.

The plan is a small IR (`Graph`): buffers (C, H, W per image) and nodes that
read and write channel slices of buffers (`Ref`). Concat is never a copy: the
producers write into slices of the concatenated buffer; Split outputs are
slices. Residual Adds are fused into the convs that precede them. Two
executors run the same IR: `Net` here (libonnxsharp_cuda, one CUDA graph per
batch size) and the CPU oracle (oracle/yolo_ref.py, test infrastructure).
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

ACT_NONE, ACT_SILU = 0, 1


@dataclass(frozen=True)
class Ref:
    """Channels [c0, c0 + c) of buffer `buf`."""

    buf: str
    c0: int
    c: int


@dataclass
class Node:
    op: str          # conv | maxpool | upsample | psa | decode
    name: str
    ins: list        # list[Ref]
    outs: list       # list[Ref]
    attrs: dict = field(default_factory=dict)


@dataclass
class Graph:
    buffers: dict = field(default_factory=dict)   # name -> (C, H, W)
    nodes: list = field(default_factory=list)
    params: dict = field(default_factory=dict)    # name -> shape
    input: str = "images"
    output: str = "output0"                       # [B, 4 + nc, A] (not a Ref buffer)
    nc: int = 80
    strides: tuple = (8, 16, 32)

    # ---- builder helpers
    def buf(self, name: str, c: int, h: int, w: int) -> Ref:
        assert name not in self.buffers, name
        self.buffers[name] = (c, h, w)
        return Ref(name, 0, c)

    def hw(self, r: Ref) -> tuple[int, int]:
        return self.buffers[r.buf][1], self.buffers[r.buf][2]

    def conv(self, name: str, x: Ref, y: Ref, k: int, s: int = 1, act: int = ACT_SILU, residual: Ref | None = None,
             group: int = 1) -> Ref:
        h, w = self.hw(x)
        oh, ow = (h + 2 * (k // 2) - k) // s + 1, (w + 2 * (k // 2) - k) // s + 1
        assert self.hw(y) == (oh, ow), (name, self.hw(y), (oh, ow))
        assert x.c % group == 0 and y.c % group == 0
        self.params[name + ".w"] = (y.c, x.c // group, k, k)
        self.params[name + ".b"] = (y.c,)
        ins = [x] + ([residual] if residual is not None else [])
        self.nodes.append(Node("conv", name, ins, [y], dict(k=k, s=s, p=k // 2, act=act, group=group,
                                                             residual=residual is not None)))
        return y


def _bottleneck(g: Graph, name: str, x: Ref, y: Ref, e: float, shortcut: bool = True) -> Ref:
    h, w = g.hw(x)
    hid = g.buf(name + ".h", int(y.c * e), h, w)
    g.conv(name + ".cv1", x, hid, 3)
    return g.conv(name + ".cv2", hid, y, 3, residual=x if shortcut else None)


def _c3k(g: Graph, name: str, x: Ref, y: Ref, n: int = 2) -> Ref:
    h, w = g.hw(x)
    c_ = y.c // 2
    cat = g.buf(name + ".cat", 2 * c_, h, w)
    a = g.buf(name + ".a", c_, h, w)
    g.conv(name + ".cv1", x, a, 1)
    g.conv(name + ".cv2", x, Ref(cat.buf, c_, c_), 1)
    prev = a
    for i in range(n):
        out = Ref(cat.buf, 0, c_) if i == n - 1 else g.buf(f"{name}.b{i}", c_, h, w)
        prev = _bottleneck(g, f"{name}.m.{i}", prev, out, 1.0)
    return g.conv(name + ".cv3", cat, y, 1)


def _c3k2(g: Graph, name: str, x: Ref, y: Ref, n: int, c3k: bool, e: float = 0.5) -> Ref:
    h, w = g.hw(x)
    c_ = int(y.c * e)
    cat = g.buf(name + ".cat", (2 + n) * c_, h, w)
    g.conv(name + ".cv1", x, Ref(cat.buf, 0, 2 * c_), 1)
    prev = Ref(cat.buf, c_, c_)
    for i in range(n):
        out = Ref(cat.buf, (2 + i) * c_, c_)
        prev = _c3k(g, f"{name}.m.{i}", prev, out) if c3k else _bottleneck(g, f"{name}.m.{i}", prev, out, 0.5)
    return g.conv(name + ".cv2", cat, y, 1)


def _sppf(g: Graph, name: str, x: Ref, y: Ref, k: int = 5) -> Ref:
    h, w = g.hw(x)
    c_ = x.c // 2
    cat = g.buf(name + ".cat", 4 * c_, h, w)
    g.conv(name + ".cv1", x, Ref(cat.buf, 0, c_), 1)
    for i in range(3):
        g.nodes.append(Node("maxpool", f"{name}.m{i}", [Ref(cat.buf, i * c_, c_)], [Ref(cat.buf, (i + 1) * c_, c_)],
                            dict(k=k, s=1, p=k // 2)))
    return g.conv(name + ".cv2", cat, y, 1)


def _c2psa(g: Graph, name: str, x: Ref, y: Ref) -> Ref:
    h, w = g.hw(x)
    c = x.c // 2
    heads, hd = c // 64, 64
    kd = hd // 2
    cat = g.buf(name + ".cat", 2 * c, h, w)
    g.conv(name + ".cv1", x, cat, 1)
    b = Ref(cat.buf, c, c)
    blk = name + ".m.0"
    qkv = g.buf(blk + ".attn.qkv", heads * (2 * kd + hd), h, w)
    g.conv(blk + ".attn.qkv", b, qkv, 1, act=ACT_NONE)
    att = g.buf(blk + ".attn.out", heads * hd, h, w)
    g.nodes.append(Node("psa", blk + ".attn", [qkv], [att], dict(heads=heads, kd=kd, hd=hd, scale=kd ** -0.5)))
    attpe = g.buf(blk + ".attn.pe_out", heads * hd, h, w)
    for hh in range(heads):  # pe: depthwise 3x3 on v (per head slice of qkv) + the attention output
        v = Ref(qkv.buf, hh * (2 * kd + hd) + 2 * kd, hd)
        g.conv(f"{blk}.attn.pe.{hh}", v, Ref(attpe.buf, hh * hd, hd), 3, act=ACT_NONE,
               residual=Ref(att.buf, hh * hd, hd), group=hd)
    b1 = g.buf(blk + ".x1", c, h, w)
    g.conv(blk + ".attn.proj", attpe, b1, 1, act=ACT_NONE, residual=b)
    f = g.buf(blk + ".ffn", 2 * c, h, w)
    g.conv(blk + ".ffn.0", b1, f, 1)
    g.conv(blk + ".ffn.1", f, b, 1, act=ACT_NONE, residual=b1)
    return g.conv(name + ".cv2", cat, y, 1)


def build_yolo11n(nc: int = 80, size: int = 640) -> Graph:
    """The YOLO11n-shaped graph for an input of [B, 3, size, size]."""
    g = Graph(nc=nc)
    s2, s4, s8, s16, s32 = size // 2, size // 4, size // 8, size // 16, size // 32
    img = g.buf("images", 3, size, size)
    m0 = g.conv("model.0", img, g.buf("m0", 16, s2, s2), 3, 2)
    m1 = g.conv("model.1", m0, g.buf("m1", 32, s4, s4), 3, 2)
    m2 = _c3k2(g, "model.2", m1, g.buf("m2", 64, s4, s4), 1, False, 0.25)
    m3 = g.conv("model.3", m2, g.buf("m3", 64, s8, s8), 3, 2)
    cat15 = g.buf("cat15", 256, s8, s8)
    m4 = _c3k2(g, "model.4", m3, Ref("cat15", 128, 128), 1, False, 0.25)
    m5 = g.conv("model.5", m4, g.buf("m5", 128, s16, s16), 3, 2)
    cat12 = g.buf("cat12", 384, s16, s16)
    m6 = _c3k2(g, "model.6", m5, Ref("cat12", 256, 128), 1, True)
    m7 = g.conv("model.7", m6, g.buf("m7", 256, s32, s32), 3, 2)
    m8 = _c3k2(g, "model.8", m7, g.buf("m8", 256, s32, s32), 1, True)
    m9 = _sppf(g, "model.9", m8, g.buf("m9", 256, s32, s32))
    cat21 = g.buf("cat21", 384, s32, s32)
    m10 = _c2psa(g, "model.10", m9, Ref("cat21", 128, 256))
    g.nodes.append(Node("upsample", "model.11", [m10], [Ref("cat12", 0, 256)], dict(scale=2)))
    cat18 = g.buf("cat18", 192, s16, s16)
    m13 = _c3k2(g, "model.13", cat12, Ref("cat18", 64, 128), 1, False)
    g.nodes.append(Node("upsample", "model.14", [m13], [Ref("cat15", 0, 128)], dict(scale=2)))
    m16 = _c3k2(g, "model.16", cat15, g.buf("m16", 64, s8, s8), 1, False)
    g.conv("model.17", m16, Ref("cat18", 0, 64), 3, 2)
    m19 = _c3k2(g, "model.19", cat18, g.buf("m19", 128, s16, s16), 1, False)
    g.conv("model.20", m19, Ref("cat21", 0, 128), 3, 2)
    m22 = _c3k2(g, "model.22", cat21, g.buf("m22", 256, s32, s32), 1, True)
    # Detect (model.23): box branch 3x3 -> 3x3 -> 1x1 (64 = 4*16), class branch
    # (DW 3x3 -> 1x1) x 2 -> 1x1 (nc); then DFL + dist2bbox + sigmoid.
    boxes, classes = [], []
    for i, x in enumerate((m16, m19, m22)):
        h, w = g.hw(x)
        p = f"model.23.cv2.{i}"
        t = g.conv(p + ".0", x, g.buf(p + ".0", 64, h, w), 3)
        t = g.conv(p + ".1", t, g.buf(p + ".1", 64, h, w), 3)
        boxes.append(g.conv(p + ".2", t, g.buf(p + ".2", 64, h, w), 1, act=ACT_NONE))
        p = f"model.23.cv3.{i}"
        c3 = max(64, min(nc, 100))
        t = g.conv(p + ".0.0", x, g.buf(p + ".0.0", x.c, h, w), 3, group=x.c)
        t = g.conv(p + ".0.1", t, g.buf(p + ".0.1", c3, h, w), 1)
        t = g.conv(p + ".1.0", t, g.buf(p + ".1.0", c3, h, w), 3, group=c3)
        t = g.conv(p + ".1.1", t, g.buf(p + ".1.1", c3, h, w), 1)
        classes.append(g.conv(p + ".2", t, g.buf(p + ".2", nc, h, w), 1, act=ACT_NONE))
    g.nodes.append(Node("decode", "model.23", boxes + classes, [], dict(nc=nc, strides=g.strides)))
    return g


def count_ops(g: Graph) -> dict[str, int]:
    out: dict[str, int] = {}
    for n in g.nodes:
        out[n.op] = out.get(n.op, 0) + 1
    return out


def flops_per_image(g: Graph) -> float:
    """2 * MACs of every conv (the convention of the reference's conv_flops tool) plus the PSA MatMuls."""
    total = 0.0
    for n in g.nodes:
        if n.op == "conv":
            y = n.outs[0]
            oh, ow = g.hw(y)
            k, grp = n.attrs["k"], n.attrs["group"]
            total += 2.0 * y.c * oh * ow * (n.ins[0].c // grp) * k * k
        elif n.op == "psa":
            a = n.attrs
            t = g.hw(n.ins[0])[0] * g.hw(n.ins[0])[1]
            total += 2.0 * a["heads"] * (t * t * a["kd"] + t * t * a["hd"])
    return total


def init_params(g: Graph, seed: int = 0) -> dict[str, np.ndarray]:
    """He-normal conv weights (std sqrt(2/fan_in)), folded-BN biases N(0, 0.01)."""
    rng = np.random.default_rng(seed)
    params = {}
    for name, shape in sorted(g.params.items()):
        if name.endswith(".w"):
            fan_in = shape[1] * shape[2] * shape[3]
            params[name] = (rng.standard_normal(shape) * np.sqrt(2.0 / fan_in)).astype(np.float32)
        else:
            params[name] = rng.normal(0.0, 0.01, shape).astype(np.float32)
    return params


def anchors(g: Graph, size: int = 640):
    """(ax, ay, stride) per anchor, scale-major then row-major (make_anchors)."""
    out = []
    for s in g.strides:
        n = size // s
        ys, xs = np.meshgrid(np.arange(n, dtype=np.float32) + 0.5, np.arange(n, dtype=np.float32) + 0.5, indexing="ij")
        out.append(np.stack([xs.ravel(), ys.ravel(), np.full(n * n, s, np.float32)], 1))
    return np.concatenate(out)


def buffer_lifetimes(g: Graph):
    """(names, first, last): the node index that first writes and last reads each
    intermediate buffer (NetImpl.PrepareForGraph's live ranges). The graph input
    is excluded: it is not in the arena but one of the plan's input slots (a
    separate buffer per slot, so the next batch can be copied in while the
    current one runs), read by every replay of the slot's captured graph."""
    names = [n for n in g.buffers if n != g.input]
    first = {n: -1 for n in names}
    last = {n: 0 for n in names}
    for i, node in enumerate(g.nodes):
        for r in node.outs:
            if first[r.buf] < 0:
                first[r.buf] = i
        for r in node.ins:
            if r.buf != g.input:
                last[r.buf] = max(last[r.buf], i)
    return names, first, last


def node_lanes(g: Graph, lanes: int) -> list[int]:
    """Stream (lane) of each node: the Detect head's box branches on lane 1 and
    its class branches on lane 2 (each a chain of convs that depends only on
    its neck level), everything else on lane 0. The head chains then run
    beside the neck and beside each other, which fills the GPU when a batch
    is too small for one layer to (strong scaling: 8 images per GPU)."""
    out = []
    for n in g.nodes:
        lane = 0
        if lanes > 1 and n.name.startswith("model.23.cv2."):
            lane = 1
        elif lanes > 1 and n.name.startswith("model.23.cv3."):
            lane = 2 if lanes > 2 else 1
        out.append(lane)
    return out


def node_deps(g: Graph) -> list[set]:
    """Earlier nodes each node must wait for: every earlier node that writes a
    channel slice it reads or writes, or reads a slice it writes (RAW, WAW, WAR
    on the plan's buffers; reuse of arena memory is made safe separately)."""
    def overlap(a: Ref, b: Ref) -> bool:
        return a.buf == b.buf and a.c0 < b.c0 + b.c and b.c0 < a.c0 + a.c

    deps = []
    for i, n in enumerate(g.nodes):
        d = set()
        for j in range(i):
            m = g.nodes[j]
            if (any(overlap(w, r) for w in m.outs for r in n.ins) or any(overlap(w, x) for w in m.outs for x in n.outs)
                    or any(overlap(r, x) for r in m.ins for x in n.outs)):
                d.add(j)
        deps.append(d)
    return deps


def happens_before(deps: list[set], lane_of: list[int]) -> list[int]:
    """Bitmask per node of the nodes that complete before it starts: its data
    dependencies, the previous node on its lane, and their ancestors."""
    anc, last_on = [], {}
    for i, d in enumerate(deps):
        preds = set(d)
        if lane_of[i] in last_on:
            preds.add(last_on[lane_of[i]])
        m = 0
        for p in preds:
            m |= anc[p] | (1 << p)
        anc.append(m)
        last_on[lane_of[i]] = i
    return anc


# ---------------------------------------------------------------------------- device executor
class Net:
    """The static plan on one GPU: arena-planned activations, prepacked
    weights, one CUDA graph per batch size (osc_graph_*)."""

    def __init__(self, ctx, g: Graph, params: dict, batch: int, size: int = 640, lanes: int = 3):
        import torch

        from . import arena
        from .runtime import Context, ConvWeights

        self.ctx, self.g, self.batch, self.size = ctx, g, batch, size
        dev = torch.device("cuda", ctx.device)
        # lanes: the plan's nodes run on `lanes` streams, each with its own
        # context (stream + scratch arena, so concurrent layers never share
        # per-call temporaries); cross-lane dependencies are events, captured
        # into the same CUDA graph
        self.lane_of = node_lanes(g, lanes)
        self.lanes = max(self.lane_of) + 1
        self.deps = node_deps(g)
        anc = happens_before(self.deps, self.lane_of)
        self.cross = [sorted(j for j in d if self.lane_of[j] != self.lane_of[i]) for i, d in enumerate(self.deps)]
        self.signals = sorted({j for c in self.cross for j in c})
        names, first, last = buffer_lifetimes(g)
        touch = {n: 0 for n in names}
        for i, node in enumerate(g.nodes):
            for r in list(node.ins) + list(node.outs):
                if r.buf in touch:
                    touch[r.buf] |= 1 << i
        lts = []
        for n in names:
            c, h, w = g.buffers[n]
            lts.append(arena.Lifetime(first[n], last[n], batch * c * h * w * 4))
        offsets, total = arena.plan_offsets_dag(lts, [touch[n] for n in names], anc)
        self.arena_bytes = total
        self.arena = torch.empty(max(total, 256) // 4, dtype=torch.float32, device=dev)
        self.views = {}
        for n, off in zip(names, offsets):
            c, h, w = g.buffers[n]
            if off >= 0:
                self.views[n] = self.arena[off // 4: off // 4 + batch * c * h * w].view(batch, c, h, w)
        self.inputs = [torch.empty((batch,) + tuple(g.buffers[g.input]), dtype=torch.float32, device=dev)]
        self.outputs = [torch.empty((batch, 4 + g.nc, sum((size // s) ** 2 for s in g.strides)),
                                    dtype=torch.float32, device=dev)]
        self.views[g.input] = self.inputs[0]
        self.output = self.outputs[0]
        # weights
        self.dev_params = {k: torch.from_numpy(v).to(dev) for k, v in params.items()}
        self.packed = {}
        for node in g.nodes:
            if node.op == "conv" and self.tensor_core(node):
                self.packed[node.name] = ConvWeights(ctx, self.dev_params[node.name + ".w"], g.params[node.name + ".w"])
        self.graphs = [None]
        self.extra_graphs = []
        self.stream = None
        self.lane_ctx = [ctx] + [Context(ctx.device) for _ in range(self.lanes - 1)]
        self.lane_streams = [None] + [torch.cuda.Stream(device=dev) for _ in range(self.lanes - 1)]
        for c, st in zip(self.lane_ctx[1:], self.lane_streams[1:]):
            c.set_stream(st.cuda_stream)
        self.events = {j: torch.cuda.Event() for j in self.signals}
        self.ev_fork = torch.cuda.Event()
        self.ev_join = [torch.cuda.Event() for _ in range(self.lanes)]

    def launch_count(self) -> int:
        """Library kernel launches made so far by all of the plan's lane contexts."""
        return sum(c.launch_count() for c in self.lane_ctx)

    @staticmethod
    def tensor_core(node) -> bool:
        """Tensor cores for the group-1 convs except the narrow layers: 16 or
        fewer output channels, or a reduction C_in*k*k <= 144 with C_in < 48
        (stem, 16->32 3x3, the 8/16-channel bottlenecks, the 32-channel 1x1s
        at 160x160). There the register-blocked CUDA-core kernel is faster:
        the tensor-core kernels' fixed cost per 128-pixel tile dominates when
        a tile holds few channels (measured per layer at B=64 on B200: 32->32
        1x1 at 160x160 131 us on CUDA cores, 191 on tensor cores; 48->64 316
        and 235). 1x1 convs with 48 or more input channels take the pointwise
        kernel, which reads NCHW directly."""
        if node.attrs["group"] != 1:
            return False
        cin, cout, k = node.ins[0].c, node.outs[0].c, node.attrs["k"]
        if k == 1 and node.attrs["s"] == 1 and cin >= 48:
            return True
        return not (cout <= 16 or (cin * k * k <= 144 and cin < 48))

    def view(self, r: Ref):
        return self.views[r.buf][:, r.c0:r.c0 + r.c]

    def input_view(self, slot: int = 0):
        return self.inputs[slot]

    def _run_nodes(self, serial: bool = False):
        """Enqueue every node. The main lane runs on the context's current
        stream; with serial=False the other lanes fork from it, wait for their
        cross-lane inputs on events and join it at the end (all of which a
        stream capture records as graph edges). serial=True runs every node on
        the main context in plan order (same kernels, same results)."""
        import torch

        if serial or self.lanes == 1:
            for node in self.g.nodes:
                self._run_node(self.ctx, node)
            return
        main = torch.cuda.ExternalStream(self.ctx.get_stream(), device=self.ctx.device)
        streams = [main] + self.lane_streams[1:]
        self.ev_fork.record(main)
        for st in streams[1:]:
            st.wait_event(self.ev_fork)
        for i, node in enumerate(self.g.nodes):
            lane = self.lane_of[i]
            for j in self.cross[i]:
                streams[lane].wait_event(self.events[j])
            self._run_node(self.lane_ctx[lane], node)
            if i in self.events:
                self.events[i].record(streams[lane])
        for lane in range(1, self.lanes):
            self.ev_join[lane].record(streams[lane])
            main.wait_event(self.ev_join[lane])

    def _run_node(self, ctx, node):
        """Enqueue one node's kernels on ctx (its stream and scratch arena)."""
        from . import _lib, ops

        a = node.attrs
        if node.op == "conv":
            x, y = self.view(node.ins[0]), self.view(node.outs[0])
            res = self.view(node.ins[1]) if a["residual"] else None
            b = self.dev_params[node.name + ".b"]
            if node.name in self.packed:
                ops.conv2d_ex(ctx, x, self.packed[node.name], b, y, a["s"], a["p"], 1, a["act"], res)
            else:  # hardware-instruction SiLU, as in the tensor-core epilogues
                act = a["act"] | _lib.ACT_FAST if a["act"] != ACT_NONE else ACT_NONE
                ops.conv2d_direct(ctx, x, self.dev_params[node.name + ".w"], b, y, a["s"], a["p"], 1, a["group"],
                                  act, res)
        elif node.op == "maxpool":
            ops.maxpool2d(ctx, self.view(node.ins[0]), self.view(node.outs[0]), a["k"], a["s"], a["p"])
        elif node.op == "upsample":
            ops.resize_nearest(ctx, self.view(node.ins[0]), self.view(node.outs[0]), a["scale"])
        elif node.op == "psa":
            ops.psa_attention(ctx, self.view(node.ins[0]), self.view(node.outs[0]), a["heads"], a["kd"], a["hd"],
                              a["scale"])
        elif node.op == "decode":
            k = len(node.ins) // 2
            ops.yolo_decode(ctx, [self.view(r) for r in node.ins[:k]], [self.view(r) for r in node.ins[k:]],
                            a["strides"], self.output)
        else:  # pragma: no cover
            raise ValueError(node.op)

    def _bind(self, slot: int):
        """Point the plan at input/output slot `slot` (for eager runs and capture)."""
        self.views[self.g.input] = self.inputs[slot]
        self.output = self.outputs[slot]

    def add_slots(self, n: int):
        """Make `n` input/output slots: each has its own input and output buffer
        and its own captured graph; the activation arena is shared, so the slots'
        graphs must run one after another on the plan's stream."""
        import torch

        while len(self.inputs) < n:
            self.inputs.append(torch.empty_like(self.inputs[0]))
            self.outputs.append(torch.empty_like(self.outputs[0]))
            self.graphs.append(None)

    def plan_stream(self):
        import torch

        if self.stream is None:
            self.stream = torch.cuda.Stream(device=self.ctx.device)
        return self.stream

    def _launch(self, slot: int, use_graph: bool, serial: bool = False):
        """Enqueue one run of the plan for `slot` on the plan's stream."""
        import ctypes as C

        from ._lib import call

        prev = self.ctx.get_stream()
        self.ctx.set_stream(self.plan_stream().cuda_stream)
        self._bind(slot)
        try:
            if not use_graph:
                self._run_nodes(serial)
                return
            if self.graphs[slot] is None:
                self._run_nodes()  # sizes the scratch arena, sets kernel attributes
                self.ctx.synchronize()
                call("osc_graph_begin", self.ctx.handle)
                h = C.c_void_p()
                try:
                    self._run_nodes()
                finally:
                    call("osc_graph_end", self.ctx.handle, C.byref(h))
                self.graphs[slot] = h
            call("osc_graph_launch", self.ctx.handle, self.graphs[slot])
        finally:
            self._bind(0)
            self.ctx.set_stream(prev)

    def capture_slot(self, slot: int, before=None, after=None):
        """Capture one CUDA graph that runs before(), the plan for `slot`, then
        after() on the plan's stream (e.g. letterbox pre-processing and the
        detect tail around the forward pass); returns the osc_graph handle, which
        close() frees. The launches run once eagerly first (scratch sizes,
        kernel attributes)."""
        import ctypes as C

        from ._lib import call

        prev = self.ctx.get_stream()
        self.ctx.set_stream(self.plan_stream().cuda_stream)
        self._bind(slot)

        def body():
            if before is not None:
                before()
            self._run_nodes()
            if after is not None:
                after()

        try:
            body()
            self.ctx.synchronize()
            call("osc_graph_begin", self.ctx.handle)
            h = C.c_void_p()
            try:
                body()
            finally:
                call("osc_graph_end", self.ctx.handle, C.byref(h))
            self.extra_graphs.append(h)
            return h
        finally:
            self._bind(0)
            self.ctx.set_stream(prev)

    def launch_graph(self, handle) -> None:
        """Replay a graph from capture_slot on the plan's stream."""
        from ._lib import call

        prev = self.ctx.get_stream()
        self.ctx.set_stream(self.plan_stream().cuda_stream)
        try:
            call("osc_graph_launch", self.ctx.handle, handle)
        finally:
            self.ctx.set_stream(prev)

    def forward(self, use_graph: bool = True, slot: int = 0, serial: bool = False):
        """Run the plan on the contents of input_view(slot); returns the slot's [B, 84, A] output tensor.

        The plan runs on its own stream (a capturable one), ordered after the
        caller's current stream and before any later work on it."""
        import torch

        stream = self.plan_stream()
        caller = torch.cuda.current_stream(self.ctx.device)
        stream.wait_stream(caller)
        self._launch(slot, use_graph, serial)
        caller.wait_stream(stream)
        return self.outputs[slot]

    def close(self):
        from . import _lib

        for i, h in enumerate(self.graphs):
            if h is not None:
                _lib.load().osc_graph_free(h)
                self.graphs[i] = None
        for h in self.extra_graphs:
            _lib.load().osc_graph_free(h)
        self.extra_graphs = []


class HostPipeline:
    """Serving loop from pinned host memory to pinned host memory.

    Batch i's host->device copy, the plan for batch i-1 and the device->host
    copy of batch i-2's detections run at the same time on three streams
    (copy engines in both directions and the SMs), so a step costs
    max(H2D, plan, D2H) instead of their sum. Each submission has its own
    input and output slot (`depth` of them, round robin); a slot is reused
    only after the plan that read its input and the copy that read its output
    have finished (event waits, no host synchronisation)."""

    def __init__(self, net: Net, depth: int = 2):
        import torch

        if depth < 1:
            raise ValueError("depth must be >= 1")
        self.net, self.depth, self.n = net, depth, 0
        net.add_slots(depth)
        dev = net.ctx.device
        self.h2d = torch.cuda.Stream(device=dev)
        self.d2h = torch.cuda.Stream(device=dev)
        self.ev_h2d = [torch.cuda.Event() for _ in range(depth)]
        self.ev_plan = [torch.cuda.Event() for _ in range(depth)]
        self.ev_d2h = [torch.cuda.Event() for _ in range(depth)]
        # capture every slot's graph up front (capture synchronises the device)
        for slot in range(depth):
            net.forward(use_graph=True, slot=slot)
        torch.cuda.synchronize(dev)

    def submit(self, host_in, host_out):
        """Queue one batch: host_in [B,3,H,W] and host_out [B,84,A] are pinned
        CPU tensors that must stay untouched until the returned event completes."""
        import torch

        net, s, reuse = self.net, self.n % self.depth, self.n >= self.depth
        plan = net.plan_stream()
        with torch.cuda.stream(self.h2d):
            if reuse:
                self.h2d.wait_event(self.ev_plan[s])  # the plan that read this input slot is done
            net.inputs[s].copy_(host_in, non_blocking=True)
            self.ev_h2d[s].record(self.h2d)
        plan.wait_event(self.ev_h2d[s])
        if reuse:
            plan.wait_event(self.ev_d2h[s])  # the copy that read this output slot is done
        net._launch(s, use_graph=True)
        self.ev_plan[s].record(plan)
        with torch.cuda.stream(self.d2h):
            self.d2h.wait_event(self.ev_plan[s])
            host_out.copy_(net.outputs[s], non_blocking=True)
            self.ev_d2h[s].record(self.d2h)
        self.n += 1
        return self.ev_d2h[s]

    def synchronize(self):
        self.d2h.synchronize()


def _main(argv=None) -> int:
    """Run the plan with random-init weights: `python -m onnxsharp_b200.yolo
    --batch 64 --passes 2 [--lanes 1] [--graph]` (eager passes, every kernel on
    the main context in plan order unless --graph replays the captured plan).
    Prints the library launches per pass; used for profiler captures."""
    import argparse

    import torch

    from .runtime import Context

    ap = argparse.ArgumentParser(description=_main.__doc__)
    ap.add_argument("--batch", type=int, default=8)
    ap.add_argument("--passes", type=int, default=2)
    ap.add_argument("--lanes", type=int, default=3)
    ap.add_argument("--graph", action="store_true")
    args = ap.parse_args(argv)
    torch.cuda.set_stream(torch.cuda.Stream())
    ctx = Context(0)
    ctx.use_torch_stream()
    g = build_yolo11n()
    net = Net(ctx, g, init_params(g, 1), args.batch, lanes=args.lanes)
    net.input_view().copy_(torch.rand(net.input_view().shape, device="cuda"))
    l0 = net.launch_count()
    for _ in range(args.passes):
        net.forward(use_graph=args.graph, serial=not args.graph)
    ctx.synchronize()
    print(f"batch {args.batch}: {args.passes} passes, {(net.launch_count() - l0) // max(1, args.passes)} launches per pass")
    net.close()
    return 0


if __name__ == "__main__":
    import sys

    sys.exit(_main())
