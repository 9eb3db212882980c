"""Writes the golden fixtures under tests/golden/.

1. ``kat.json`` — known-answer vectors transcribed from the reference's own
   test sources (C#, not runnable here: no .NET in this environment). Each
   entry names the file:line it comes from. These pin the oracle.
2. ``oracle_small.npz`` — seeded small inputs and the oracle's outputs for
   them (GEMM+bias, DQMM, conv+SiLU, attention, DFL, LayerNorm). GPU tests
   compare the CUDA path against these fixed vectors as well as against a
   fresh oracle run, so a change in the oracle itself is caught.
3. ``yolo11n.shapes.tsv`` — the reference's own shape table of the exported
   YOLO11n graph (tests/data/yolo11n.shapes.tsv in the reference checkout,
   copied unchanged: node index, NODE/TENSOR, op type, name, batch flag,
   shape). The YOLO plan is checked against it node by node
   (tests/test_yolo_graph.py). Copied only when ``--reference DIR`` is given.

Run from the repo root: ``python tests/golden/make_golden.py [--reference DIR]``.
"""
from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))

import oracle  # noqa: E402  (test infrastructure)

KAT = {
    "source": "sevencat/OnnxSharp tests/OnnxSharp.Tests (transcribed; C# reference not runnable here)",
    "dynamic_quantize_linear": {
        "ref": "tests/OnnxSharp.Tests/QuantOpsTests.cs:40-50",
        "x": [-1.0, 0.0, 1.0, 2.0],
        "scale": 3.0 / 255.0,
        "scale_tol": 1e-7,
        "zero_point": 85,
        "q": [0, 85, 170, 255],
    },
    "matmul_integer": {
        "ref": "tests/OnnxSharp.Tests/QuantOpsTests.cs:52-76",
        "a": [[1, 2, 3], [4, 5, 6]],
        "b": [[1, 2], [3, 4], [5, 6]],
        "c": [[22, 28], [49, 64]],
    },
    "quantize_u8": {
        "ref": "tests/OnnxSharp.Tests/Int8Tests.cs:157-178",
        "x": [0.0, 0.1, 0.25, -0.5, 10.0, 1.5],
        "scale": 0.5,
        "zero_point": 128,
        "q": [128, 128, 128, 127, 148, 131],
        "saturate_x": 1000.0,
        "saturate_q": 255,
    },
    "gemm_tolerance": {
        "ref": "tests/OnnxSharp.Tests/GemmKernelTests.cs:116-120,182-186,222-227",
        "vs_naive_double": 1e-4,
        "kernel_vs_kernel": 1e-5,
        "metric": "|got-exp| / max(1, |exp|)",
        "naive_shapes": [[257, 64, 257], [257, 257, 64], [64, 64, 64], [257, 384, 1536], [300, 256, 256],
                         [1, 257, 64], [5, 17, 33], [17, 1, 257]],
        "column_bias_shapes": [[257, 384, 1536], [64, 64, 17], [1, 300, 256], [5, 7, 33]],
        "packed_shapes": [[96, 320, 1280], [96, 1280, 320], [257, 384, 1536], [5, 17, 33], [3, 1, 7], [1, 300, 256],
                          [9, 64, 17]],
        "scale_bias_shapes": [[96, 320, 1280], [96, 320, 320], [96, 1280, 320], [7, 33, 45], [4, 8, 3], [2, 96, 17]],
    },
    "int8_f32_substitute_exact": {
        "ref": "tests/OnnxSharp.Tests/Int8Tests.cs:286-326",
        "m": 4, "k": 1280, "n": 32, "a_zero": 121, "w_zero_range": [-20, 20],
        "claim": "F32 accumulation of widened int8 products reproduces the exact int32 sum",
    },
    "yolo_golden_tolerance": {
        "ref": "tests/OnnxSharp.Tests/YoloGoldenTests.cs:21",
        "max_abs": 2e-2,
    },
    "attention_golden_tolerance": {
        "ref": "tests/OnnxSharp.Tests/AttentionTests.cs:20-58",
        "max_abs": 1e-5,
    },
}


def small_fixtures() -> dict[str, np.ndarray]:
    rng = np.random.default_rng(20261201)
    out: dict[str, np.ndarray] = {}
    # GEMM + column bias (awkward shape)
    a = rng.uniform(-1, 1, (67, 45)).astype(np.float32)
    b = rng.uniform(-1, 1, (45, 70)).astype(np.float32)
    bias = rng.uniform(-1, 1, 70).astype(np.float32)
    out.update(gemm_a=a, gemm_b=b, gemm_bias=bias, gemm_c=oracle.gemm(a, b, col_bias=bias, threads=1))
    # DQMM (ragged m and n so both epilogue forms occur)
    a = rng.normal(0, 1, (37, 64)).astype(np.float32)
    w = rng.integers(-127, 128, (64, 50)).astype(np.int8)
    ws = rng.uniform(0.001, 0.02, 50).astype(np.float32)
    bias = rng.normal(0, 0.01, 50).astype(np.float32)
    y, q, acc, (s, z) = oracle.dqmm(a, w, 0, ws, bias, threads=1)
    out.update(dqmm_a=a, dqmm_w=w, dqmm_wscale=ws, dqmm_bias=bias, dqmm_y=y, dqmm_q=q, dqmm_acc=acc,
               dqmm_params=np.array([s, z], np.float32))
    # Conv + SiLU
    x = rng.uniform(0, 1, (2, 8, 11, 13)).astype(np.float32)
    wc = (rng.normal(0, 1, (16, 8, 3, 3)) * np.sqrt(2 / 72)).astype(np.float32)
    bc = rng.normal(0, 0.01, 16).astype(np.float32)
    out.update(conv_x=x, conv_w=wc, conv_b=bc,
               conv_y=oracle.conv2d(x, wc, bc, stride=(1, 1), pads=(1, 1, 1, 1), act=1, threads=1))
    # FusedAttention, heads form, T > 64 (blocked kernel)
    qa = rng.normal(0, 1, (2, 80, 64)).astype(np.float32)
    ka = rng.normal(0, 1, (2, 80, 64)).astype(np.float32)
    va = rng.normal(0, 1, (2, 80, 64)).astype(np.float32)
    out.update(attn_q=qa, attn_k=ka, attn_v=va, attn_o=oracle.attention(qa, ka, va, heads=2, scale=0.25, threads=1))
    # DFL
    xd = rng.normal(0, 2, (2, 64, 100)).astype(np.float32)
    out.update(dfl_x=xd, dfl_y=oracle.dfl(xd, 16, threads=1))
    # LayerNorm
    xl = rng.normal(0, 1, (5, 48)).astype(np.float32)
    g = rng.normal(1, 0.1, 48).astype(np.float32)
    bl = rng.normal(0, 0.1, 48).astype(np.float32)
    out.update(ln_x=xl, ln_g=g, ln_b=bl, ln_y=oracle.layernorm(xl, g, bl, 1e-5, threads=1))
    return out


def main() -> None:
    (HERE / "kat.json").write_text(json.dumps(KAT, indent=1) + "\n")
    np.savez_compressed(HERE / "oracle_small.npz", **small_fixtures())
    print("wrote", HERE / "kat.json", HERE / "oracle_small.npz")
    if "--reference" in sys.argv:
        ref = Path(sys.argv[sys.argv.index("--reference") + 1])
        tsv = (ref / "tests" / "data" / "yolo11n.shapes.tsv").read_bytes()
        (HERE / "yolo11n.shapes.tsv").write_bytes(tsv)
        print("wrote", HERE / "yolo11n.shapes.tsv")


if __name__ == "__main__":
    main()
