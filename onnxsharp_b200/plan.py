"""ctypes mirror of the native static-plan API (osc_plan_*, include/onnxsharp_cuda.h)
and the lowering of the YOLO IR (yolo.Graph) onto it.

The native executor does what the reference's NetImpl.PrepareForGraph /
BufferAllocator.Assign / Interpreter.Run do (src/OnnxSharp/Engine/NetImpl.cs:151-192,
Engine/BufferAllocator.cs:41-138, Core/Interpreter.cs:30-186): live ranges,
lifetime colouring into one device arena, one captured CUDA graph per input
signature. This module only builds its description.
"""
from __future__ import annotations

import ctypes as C

from . import _lib
from ._lib import call, ptr

OP_CONV, OP_CONV_DIRECT, OP_MAXPOOL, OP_RESIZE_NEAREST, OP_PSA = 1, 2, 3, 4, 5
OP_YOLO_DECODE, OP_MATMUL_BIAS, OP_SOFTMAX, OP_UNARY, OP_ATTENTION = 6, 7, 8, 9, 10
MAX_IN = 6


class Ref(C.Structure):
    _fields_ = [("buf", C.c_int), ("c0", C.c_int), ("c", C.c_int)]


class Node(C.Structure):
    _fields_ = [("op", C.c_int), ("n_in", C.c_int), ("n_out", C.c_int), ("inp", Ref * MAX_IN), ("out", Ref * 1),
                ("iattr", C.c_int * 8), ("fattr", C.c_float * 4), ("weights", C.c_void_p), ("bias", C.c_void_p)]


class Desc(C.Structure):
    _fields_ = [("batch", C.c_int), ("n_buffers", C.c_int), ("buf_chw", C.POINTER(C.c_int)), ("input_buf", C.c_int),
                ("n_nodes", C.c_int), ("nodes", C.POINTER(Node))]


def node(op, ins, outs=(), iattr=(), fattr=(), weights=None, bias=None) -> Node:
    """ins / outs: (buffer index, c0, c) triples."""
    n = Node()
    n.op, n.n_in, n.n_out = op, len(ins), len(outs)
    for i, r in enumerate(ins):
        n.inp[i] = Ref(*r)
    for i, r in enumerate(outs):
        n.out[i] = Ref(*r)
    for i, v in enumerate(iattr):
        n.iattr[i] = int(v)
    for i, v in enumerate(fattr):
        n.fattr[i] = float(v)
    if isinstance(weights, C.c_void_p):  # a prepacked handle
        n.weights = weights.value
    else:  # a device tensor, an address or None
        n.weights = ptr(weights)
    n.bias = ptr(bias)
    return n


class Plan:
    """A built osc_plan on a context; `keep` holds whatever the nodes point at (weights, biases)."""

    def __init__(self, ctx, batch: int, buffers, input_buf: int, nodes, keep=()):
        self.ctx, self.batch, self.keep = ctx, batch, list(keep)
        chw = (C.c_int * (3 * len(buffers)))(*[int(v) for b in buffers for v in b])
        arr = (Node * len(nodes))(*nodes)
        d = Desc(int(batch), len(buffers), chw, int(input_buf), len(nodes), arr)
        h = C.c_void_p()
        call("osc_plan_build", ctx.handle, C.byref(d), C.byref(h))
        self.handle = h
        import weakref

        self._finalizer = weakref.finalize(self, _lib.load().osc_plan_free, h)

    def run(self, inp, out=None) -> None:
        call("osc_plan_run", self.handle, ptr(inp), ptr(out))

    def arena_bytes(self) -> int:
        n = C.c_size_t()
        call("osc_plan_arena_bytes", self.handle, C.byref(n))
        return n.value

    def buffer_ptr(self, buf: int, inp) -> int:
        p = C.c_void_p()
        call("osc_plan_buffer", self.handle, int(buf), ptr(inp), C.byref(p), None)
        return p.value

    def close(self) -> None:
        self._finalizer()


def arena_assign(first, last, nbytes) -> tuple[list[int], int]:
    """The native colouring (osc_arena_assign) on the host: byte offsets and arena size."""
    n = len(first)
    f = (C.c_int * n)(*first)
    l_ = (C.c_int * n)(*last)
    b = (C.c_size_t * n)(*nbytes)
    off = (C.c_longlong * n)()
    tot = C.c_size_t()
    call("osc_arena_assign", n, f, l_, b, off, C.byref(tot))
    return list(off), tot.value


def build_yolo_plan(ctx, g, dev_params: dict, packed: dict, batch: int) -> Plan:
    """Lower the YOLO IR to a native plan: the same kernels and routing as yolo.Net
    (tensor-core convs for the wide layers, CUDA-core direct convs for the narrow
    and depthwise ones, fast Sigmoid/SiLU), so the outputs are bit-identical."""
    from . import yolo

    names = list(g.buffers)
    idx = {n: i for i, n in enumerate(names)}
    nodes = []

    def ref(r):
        return (idx[r.buf], r.c0, r.c)

    for nd in g.nodes:
        a = nd.attrs
        if nd.op == "conv":
            ins = [ref(r) for r in nd.ins]
            b = dev_params[nd.name + ".b"]
            if nd.name in packed:
                nodes.append(node(OP_CONV, ins, [ref(nd.outs[0])], [a["s"], a["p"], 1, a["act"], a["k"], 1],
                                  weights=packed[nd.name].handle, bias=b))
            else:
                act = a["act"] | _lib.ACT_FAST if a["act"] != yolo.ACT_NONE else yolo.ACT_NONE
                nodes.append(node(OP_CONV_DIRECT, ins, [ref(nd.outs[0])], [a["s"], a["p"], 1, act, a["k"], a["group"]],
                                  weights=dev_params[nd.name + ".w"], bias=b))
        elif nd.op == "maxpool":
            nodes.append(node(OP_MAXPOOL, [ref(nd.ins[0])], [ref(nd.outs[0])], [a["k"], a["s"], a["p"]]))
        elif nd.op == "upsample":
            nodes.append(node(OP_RESIZE_NEAREST, [ref(nd.ins[0])], [ref(nd.outs[0])], [a["scale"]]))
        elif nd.op == "psa":
            nodes.append(node(OP_PSA, [ref(nd.ins[0])], [ref(nd.outs[0])], [a["heads"], a["kd"], a["hd"]],
                              [a["scale"]]))
        elif nd.op == "decode":
            nodes.append(node(OP_YOLO_DECODE, [ref(r) for r in nd.ins], [], [a["nc"]], list(a["strides"])))
        else:  # pragma: no cover
            raise ValueError(nd.op)
    return Plan(ctx, batch, [g.buffers[n] for n in names], idx[g.input], nodes, keep=[dev_params, packed])
