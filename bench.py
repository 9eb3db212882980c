#!/usr/bin/env python
"""bench.py — throughput of OnnxSharp's matrix-multiply hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl ours|reference]

One process per GPU (torchrun for N > 1, NCCL process group for the barrier
and the max-over-ranks reduction). Each rank runs the same workload on its own
seeded synthetic data (weak scaling: images / rows are independent, so the
path shards with no data-path collective). Rank 0 prints ONE JSON line.

Timed region: W untimed warm-up steps, then exactly K steps bracketed by a
barrier + cuda synchronize on both sides. Every step is timed with CUDA events
on the stream the kernels run on; L2 is flushed (a 512 MiB device write)
between steps, outside the events. `value` is the whole-job throughput with
inputs resident in HBM; `e2e` is the same metric through the public API with
pinned host buffers (H2D of the step's inputs + D2H of its output inside the
timed region). `roofline` reports the dominant kernel against the measured
peaks in MEASURED_PEAKS.json; `cpu_baseline` times the CPU oracle (a
restatement of the reference's CPU kernels) on a bounded sample.

--impl reference times the reference's CPU algorithm (the oracle port: the
reference is C# and cannot run here) on the host cores, same metric/config.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "GEMM/Conv TFLOPS (% roofline); YOLO11n-shape images/sec at 1/2/4/8 B200"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def load_peaks() -> tuple[dict, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return json.loads(p.read_text()), "measured"
        except (OSError, ValueError):
            pass
    return dict(FALLBACK_PEAKS), "fallback"


def load_traffic(workload: str):
    """DRAM bytes per dominant-kernel launch from a committed ncu summary (profiles/traffic.json)."""
    p = ROOT / "profiles" / "traffic.json"
    try:
        entry = json.loads(p.read_text()).get(workload)
    except (OSError, ValueError):
        return None
    return None if entry is None else entry.get("bytes_per_launch")


def physical_cores() -> int:
    try:
        out = subprocess.run(["lscpu", "-p=core,socket"], capture_output=True, text=True, timeout=10).stdout
        cores = {tuple(l.split(",")) for l in out.splitlines() if l and not l.startswith("#")}
        if cores:
            return len(cores)
    except (OSError, subprocess.SubprocessError):
        pass
    return os.cpu_count() or 1


def cpu_model() -> str:
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


# ----------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=self.file, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=10)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.file.flush()
        rows = []
        for line in Path(self.file.name).read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append((float(parts[1]), float(parts[2]), float(parts[3]), parts[5:9]))
            except ValueError:
                continue
        os.unlink(self.file.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"], "samples": 0}
        loaded = [r for r in rows if r[2] > 250.0] or rows
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in loaded for i, v in enumerate(r[3]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(r[0] for r in loaded), "sm_max_mhz": max(r[1] for r in rows),
                "reasons": reasons, "samples": len(rows), "samples_under_load": len(loaded)}


# ----------------------------------------------------------------- workloads
class Workload:
    """One pass of the hot path over one batch of synthetic input."""

    name = ""
    unit = "TFLOP/s"
    main_kernel = ""   # dominant kernel (profile prefix)
    bound = "tensor"

    def units_per_step(self) -> float:       # FLOPs (or images) per step
        raise NotImplementedError

    def step(self):                           # device-resident inputs
        raise NotImplementedError

    def e2e_step(self):                       # pinned host in, pinned host out
        raise NotImplementedError

    def e2e_bytes(self) -> tuple[int, int]:
        raise NotImplementedError

    def main_kernel_units(self) -> float:     # algorithmic FLOPs (or bytes) of one dominant-kernel launch
        return self.units_per_step()

    def cpu_sample(self, threads: int) -> dict:
        raise NotImplementedError


def _scale(v: float) -> float:
    return v / 1e12


class GemmWorkload(Workload):
    """MatMul+Add(bias) A[2048,512] x B[512,2048] + bias[2048], U(-1,1)."""

    graphed = True
    name = "matmul_bias_f32_2048x512x2048"
    main_kernel = "k_gemm_tf32x3"

    def __init__(self, ctx, rank: int, m=2048, k=512, n=2048):
        import torch

        from onnxsharp_b200.runtime import GemmWeights

        self.m, self.k, self.n = m, k, n
        rng = np.random.default_rng(1234 + rank)
        self.a_h = rng.uniform(-1, 1, (m, k)).astype(np.float32)
        self.b_h = rng.uniform(-1, 1, (k, n)).astype(np.float32)
        self.bias_h = rng.uniform(-1, 1, n).astype(np.float32)
        dev = torch.device("cuda", torch.cuda.current_device())
        self.ctx = ctx
        self.a = torch.from_numpy(self.a_h).to(dev)
        self.bias = torch.from_numpy(self.bias_h).to(dev)
        self.c = torch.empty((m, n), dtype=torch.float32, device=dev)
        self.w = GemmWeights(ctx, torch.from_numpy(self.b_h).to(dev), k, n)
        # e2e: pinned host buffers and device staging
        self.a_pin = torch.from_numpy(self.a_h).pin_memory()
        self.c_pin = torch.empty((m, n), dtype=torch.float32).pin_memory()
        self.a_dev2 = torch.empty_like(self.a)
        self.c_dev2 = torch.empty_like(self.c)
        self.config = {"workload": self.name, "m": m, "k": k, "n": n, "bias": True,
                       "precision": "3xTF32 (tcgen05 kind::tf32), FP32 in/out"}

    def units_per_step(self) -> float:
        return 2.0 * self.m * self.k * self.n

    def step(self):
        from onnxsharp_b200.runtime import gemm_bias

        gemm_bias(self.ctx, self.a, self.w, self.bias, out=self.c)

    def e2e_step(self):
        from onnxsharp_b200.runtime import gemm_bias

        self.ctx.memcpy_htod(self.a_dev2, self.a_pin, self.a_pin.numel() * 4)
        gemm_bias(self.ctx, self.a_dev2, self.w, self.bias, out=self.c_dev2)
        self.ctx.memcpy_dtoh(self.c_pin, self.c_dev2, self.c_pin.numel() * 4)

    def e2e_bytes(self):
        return self.m * self.k * 4, self.m * self.n * 4

    def cpu_sample(self, threads: int) -> dict:
        import oracle

        rows = self.m
        t0 = time.perf_counter()
        reps = 0
        while True:
            oracle.gemm(self.a_h[:rows], self.b_h, col_bias=self.bias_h, threads=threads)
            reps += 1
            if time.perf_counter() - t0 > 1.5:
                break
        dt = time.perf_counter() - t0
        flops = 2.0 * rows * self.k * self.n * reps
        return {"value": _scale(flops / dt), "unit": self.unit, "cores": threads,
                "sample": f"{reps} x full GEMM {rows}x{self.k}x{self.n}+bias ({dt:.2f} s wall)"}


def conv_inputs(seed: int, batch: int):
    """BASELINE config 2 synthetic data: x U(0,1), W He-normal, b N(0, 0.01)."""
    rng = np.random.default_rng(seed)
    x = rng.uniform(0, 1, (batch, 64, 160, 160)).astype(np.float32)
    w = (rng.normal(0, 1, (128, 64, 3, 3)) * np.sqrt(2.0 / (64 * 9))).astype(np.float32)
    b = rng.normal(0, 0.01, 128).astype(np.float32)
    return x, w, b


CONV_FLOPS_PER_IMAGE = 2.0 * 128 * 160 * 160 * 64 * 9


class ConvWorkload(Workload):
    """fused Conv+SiLU, x[16,64,160,160] -> y[16,128,160,160], 3x3 s1 p1."""

    graphed = True
    name = "conv3x3_silu_f32_b16_64to128_160x160"
    main_kernel = "k_conv_tf32x3"

    def __init__(self, ctx, rank: int, batch: int = 16):
        import torch

        from onnxsharp_b200.runtime import ConvWeights

        self.batch = batch
        x, w, b = conv_inputs(4321 + rank, batch)
        self.x_h, self.w_h, self.b_h = x, w, b
        dev = torch.device("cuda", torch.cuda.current_device())
        self.ctx = ctx
        self.x = torch.from_numpy(x).to(dev)
        self.b = torch.from_numpy(b).to(dev)
        self.w = ConvWeights(ctx, torch.from_numpy(w).to(dev), w.shape)
        self.y = torch.empty((batch, 128, 160, 160), dtype=torch.float32, device=dev)
        self.x_pin = torch.from_numpy(x).pin_memory()
        self.y_pin = torch.empty(self.y.shape, dtype=torch.float32).pin_memory()
        self.x2 = torch.empty_like(self.x)
        self.y2 = torch.empty_like(self.y)
        self.config = {"workload": self.name, "batch": batch, "in": [batch, 64, 160, 160], "weight": [128, 64, 3, 3],
                       "stride": 1, "pad": 1, "act": "SiLU",
                       "precision": "3xTF32 implicit GEMM (tcgen05 kind::tf32), FP32 in/out"}

    def units_per_step(self) -> float:
        return CONV_FLOPS_PER_IMAGE * self.batch

    def _run(self, x, y):
        from onnxsharp_b200 import ACT_SILU
        from onnxsharp_b200.runtime import conv2d

        conv2d(self.ctx, x, self.w, self.b, (1, 1), (1, 1, 1, 1), (1, 1), 1, ACT_SILU, out=y)

    def step(self):
        self._run(self.x, self.y)

    def e2e_step(self):
        self.ctx.memcpy_htod(self.x2, self.x_pin, self.x_pin.numel() * 4)
        self._run(self.x2, self.y2)
        self.ctx.memcpy_dtoh(self.y_pin, self.y2, self.y_pin.numel() * 4)

    def e2e_bytes(self):
        return self.x_pin.numel() * 4, self.y_pin.numel() * 4

    def cpu_sample(self, threads: int) -> dict:
        return CpuConv(self.x_h[:1], self.w_h, self.b_h).cpu_sample(threads)


def dqmm_inputs(seed: int, m=4096, k=512, n=2048):
    """A N(0,1), W int8 U[-127,127], w_scale U(0.001,0.02), bias N(0, 0.01)."""
    rng = np.random.default_rng(seed)
    a = rng.normal(0, 1, (m, k)).astype(np.float32)
    w = rng.integers(-127, 128, (k, n)).astype(np.int8)
    ws = rng.uniform(0.001, 0.02, n).astype(np.float32)
    b = rng.normal(0, 0.01, n).astype(np.float32)
    return a, w, ws, b


class DqmmWorkload(Workload):
    """DynamicQuantizeMatMul A[4096,512] f32 x W int8 [512,2048] -> Y[4096,2048] f32."""

    graphed = True
    name = "dqmm_u8s8_4096x512x2048"
    unit = "TOP/s"
    main_kernel = "k_dqmm_i8"
    bound = "hbm"

    def __init__(self, ctx, rank: int, m=4096, k=512, n=2048):
        import torch

        from onnxsharp_b200.runtime import DqmmWeights

        self.m, self.k, self.n = m, k, n
        a, w, ws, b = dqmm_inputs(777 + rank, m, k, n)
        self.a_h, self.w_h, self.ws_h, self.b_h = a, w, ws, b
        dev = torch.device("cuda", torch.cuda.current_device())
        self.ctx = ctx
        self.a = torch.from_numpy(a).to(dev)
        self.ws = torch.from_numpy(ws).to(dev)
        self.b = torch.from_numpy(b).to(dev)
        self.w = DqmmWeights(ctx, torch.from_numpy(w).to(dev), k, n, None)
        self.y = torch.empty((m, n), dtype=torch.float32, device=dev)
        self.a_pin = torch.from_numpy(a).pin_memory()
        self.y_pin = torch.empty((m, n), dtype=torch.float32).pin_memory()
        self.a2 = torch.empty_like(self.a)
        self.y2 = torch.empty_like(self.y)
        self.config = {"workload": self.name, "m": m, "k": k, "n": n,
                       "precision": "dynamic per-tensor u8 activations x s8 weights -> s32 (tcgen05 kind::i8), "
                                    "FP32 epilogue bit-identical to the reference"}

    def units_per_step(self) -> float:
        return 2.0 * self.m * self.k * self.n

    def main_kernel_units(self) -> float:
        kp = (self.k + 127) // 128 * 128
        return self.m * kp + self.n * kp + self.m * self.n * 4 + self.n * 16

    def step(self):
        from onnxsharp_b200.runtime import dqmm

        dqmm(self.ctx, self.a, self.w, self.ws, self.b, out=self.y)

    def e2e_step(self):
        from onnxsharp_b200.runtime import dqmm

        self.ctx.memcpy_htod(self.a2, self.a_pin, self.a_pin.numel() * 4)
        dqmm(self.ctx, self.a2, self.w, self.ws, self.b, out=self.y2)
        self.ctx.memcpy_dtoh(self.y_pin, self.y2, self.y_pin.numel() * 4)

    def e2e_bytes(self):
        return self.m * self.k * 4, self.m * self.n * 4

    def cpu_sample(self, threads: int) -> dict:
        return CpuDqmm(self.a_h, self.w_h, self.ws_h, self.b_h).cpu_sample(threads)


class YoloWorkload(Workload):
    """random-init YOLO11n-shaped detector, [B,3,640,640] U(0,1) -> [B,84,8400], B = 64 per GPU.

    A step is one replay of the plan's CUDA graph. The dominant kernels are the
    tensor-core convs (channel-major implicit GEMM, pixel-major 1x1 / small-
    image convs); their roofline figures come from a profiled eager pass
    (event timing cannot be inserted into a graph replay)."""

    name = "yolo11n_shaped_b64_640"
    unit = "images/s"
    main_kernel = ("k_conv_tf32x3", "k_conv_px_tf32x3")
    bound = "tensor"
    long_step = True

    def __init__(self, ctx, rank: int, batch: int = 64):
        import torch

        from onnxsharp_b200 import yolo

        self.batch = batch
        self.ctx = ctx
        self.g = yolo.build_yolo11n()
        self.params = yolo.init_params(self.g, 2024)
        self.net = yolo.Net(ctx, self.g, self.params, batch)
        rng = np.random.default_rng(9000 + rank)
        self.images_h = rng.uniform(0, 1, (batch, 3, 640, 640)).astype(np.float32)
        self.net.input_view().copy_(torch.from_numpy(self.images_h))
        self.images_pin = torch.from_numpy(self.images_h).pin_memory()
        self.out_pin = torch.empty(self.net.output.shape, dtype=torch.float32).pin_memory()
        # a second host batch and output for the pipelined serving loop
        self.images_pin2 = torch.from_numpy(rng.uniform(0, 1, (batch, 3, 640, 640)).astype(np.float32)).pin_memory()
        self.out_pin2 = torch.empty(self.net.output.shape, dtype=torch.float32).pin_memory()
        self.pipe = None
        self.flops_img = yolo.flops_per_image(self.g)
        self.tc_flops = sum(self._node_flops(n) for n in self.g.nodes
                            if n.op == "conv" and yolo.Net.tensor_core(n)) * batch
        self.tc_launches = sum(1 for n in self.g.nodes if n.op == "conv" and yolo.Net.tensor_core(n))
        self.net.forward(use_graph=True)  # capture
        ctx.synchronize()
        self.config = {"workload": self.name, "batch_per_gpu": batch, "input": [batch, 3, 640, 640],
                       "output": [batch, 84, 8400], "gflop_per_image": round(self.flops_img / 1e9, 3),
                       "arena_mib": round(self.net.arena_bytes / 2 ** 20, 1),
                       "precision": "FP32 in/out; wide convs 3xTF32 tcgen05 (k x k implicit GEMM on NHWC hi/lo, 1x1 "
                                    "straight from NCHW), narrow and depthwise convs FP32 CUDA-core FMA, glue FP32 CUDA "
                                    "cores; conv Sigmoid/SiLU from hardware ex2/rcp (<= 2e-6 from the exact form)",
                       "plan": "static plan replayed as one CUDA graph"}

    def _node_flops(self, n):
        y = n.outs[0]
        oh, ow = self.g.hw(y)
        return 2.0 * y.c * oh * ow * (n.ins[0].c // n.attrs["group"]) * n.attrs["k"] ** 2

    def units_per_step(self) -> float:
        return float(self.batch)

    def main_kernel_units(self) -> float:
        return self.tc_flops / self.tc_launches

    def step(self):
        self.net.forward(use_graph=True)

    def profile_step(self):
        self.net.forward(use_graph=False)

    def e2e_step(self):
        # torch copies on the caller stream (the plan orders itself after it)
        self.net.input_view().copy_(self.images_pin, non_blocking=True)
        self.net.forward(use_graph=True)
        self.out_pin.copy_(self.net.output, non_blocking=True)

    def e2e_bytes(self):
        return self.images_pin.numel() * 4, self.out_pin.numel() * 4

    e2e_mode = ("pipelined: yolo.HostPipeline, depth 2 (H2D of batch i, plan of batch i-1 and D2H of batch "
                "i-2 overlap on three streams); each step copies its own 315 MB input from pinned host memory "
                "and reads its 181 MB output back; device-timed from the first H2D to the last D2H, pipeline "
                "fill and drain included; per-step inputs exceed L2, so no flush")

    def e2e_pipelined(self, warmup: int, steps: int, barrier) -> float:
        """ms per step of the serving loop, device-timed from the first H2D to the last D2H."""
        import torch

        from onnxsharp_b200 import yolo

        if self.pipe is None:
            self.pipe = yolo.HostPipeline(self.net, depth=2)
        ins, outs = (self.images_pin, self.images_pin2), (self.out_pin, self.out_pin2)
        for i in range(max(1, warmup)):
            self.pipe.submit(ins[i % 2], outs[i % 2])
        self.pipe.synchronize()
        barrier()
        torch.cuda.synchronize()
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(self.pipe.h2d)
        for i in range(steps):
            self.pipe.submit(ins[i % 2], outs[i % 2])
        stop.record(self.pipe.d2h)
        stop.synchronize()
        barrier()
        return start.elapsed_time(stop) / steps

    def cpu_sample(self, threads: int) -> dict:
        return CpuYolo(self.g, self.params, self.images_h[:1]).cpu_sample(threads)


ATTN_FLOPS = 4 * 2.0 * 8192 * 512 * 512 + 2 * 2.0 * 64 * 8 * 128 * 128 * 64


class AttentionWorkload(Workload):
    """X[64,128,512] N(0,1) -> Q/K/V projections (MatMul+bias, Xavier-uniform, zero bias)
    -> FusedAttention (H=8, D=64, scale 1/8) -> output projection."""

    graphed = True
    name = "attention_block_b64_t128_h8_d64"
    main_kernel = "k_gemm_tf32x3"

    def __init__(self, ctx, rank: int):
        import torch

        from onnxsharp_b200.runtime import GemmWeights

        rng = np.random.default_rng(5150 + rank)
        self.B, self.T, self.C, self.H = 64, 128, 512, 8
        x = rng.normal(0, 1, (self.B * self.T, self.C)).astype(np.float32)
        lim = np.sqrt(6.0 / (self.C + self.C))
        ws = [rng.uniform(-lim, lim, (self.C, self.C)).astype(np.float32) for _ in range(4)]
        dev = torch.device("cuda", torch.cuda.current_device())
        self.ctx = ctx
        self.x_h = x
        self.ws_h = ws
        self.x = torch.from_numpy(x).to(dev)
        self.bias = torch.zeros(self.C, device=dev)
        self.w = [GemmWeights(ctx, torch.from_numpy(w).to(dev), self.C, self.C) for w in ws]
        self.qkv = [torch.empty(self.B * self.T, self.C, device=dev) for _ in range(3)]
        self.o = torch.empty(self.B, self.T, self.C, device=dev)
        self.y = torch.empty(self.B * self.T, self.C, device=dev)
        self.x_pin = torch.from_numpy(x).pin_memory()
        self.y_pin = torch.empty(self.B * self.T, self.C).pin_memory()
        self.x2 = torch.empty_like(self.x)
        self.config = {"workload": self.name, "x": [64, 128, 512], "heads": 8, "head_dim": 64,
                       "precision": "3xTF32 tcgen05 (projections and QK^T / PV), FP32 softmax"}

    def units_per_step(self) -> float:
        return ATTN_FLOPS

    def main_kernel_units(self) -> float:
        return 2.0 * 8192 * 512 * 512

    def _run(self, x):
        from onnxsharp_b200.runtime import attention, gemm_bias

        for w, out in zip(self.w[:3], self.qkv):
            gemm_bias(self.ctx, x, w, self.bias, out=out)
        q, k, v = (t.view(self.B, self.T, self.C) for t in self.qkv)
        attention(self.ctx, q, k, v, self.H, 0.125, out=self.o)
        gemm_bias(self.ctx, self.o.view(self.B * self.T, self.C), self.w[3], self.bias, out=self.y)

    def step(self):
        self._run(self.x)

    def e2e_step(self):
        self.ctx.memcpy_htod(self.x2, self.x_pin, self.x_pin.numel() * 4)
        self._run(self.x2)
        self.ctx.memcpy_dtoh(self.y_pin, self.y, self.y_pin.numel() * 4)

    def e2e_bytes(self):
        return self.x_pin.numel() * 4, self.y_pin.numel() * 4

    def cpu_sample(self, threads: int) -> dict:
        return CpuAttention(self.x_h, self.ws_h).cpu_sample(threads)


WORKLOADS = {"gemm": GemmWorkload, "conv": ConvWorkload, "dqmm": DqmmWorkload, "yolo": YoloWorkload,
             "attention": AttentionWorkload}
DEFAULT_WORKLOAD = "yolo"
DEFAULT_STEPS = {"gemm": 2000, "conv": 1000, "dqmm": 2000, "yolo": 100, "attention": 500}


# ----------------------------------------------------------------- timing
def flush_l2(buf):
    buf.add_(1.0)


def run_ours(args, peaks, peaks_kind) -> dict | None:
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))

    from onnxsharp_b200.runtime import Context

    # a capturable (non-legacy) stream for the library, the events and the L2 flush
    torch.cuda.set_stream(torch.cuda.Stream())
    ctx = Context(local)
    ctx.use_torch_stream()
    wl = WORKLOADS[args.workload](ctx, rank)
    stream = torch.cuda.current_stream()
    graph = None
    if getattr(wl, "graphed", False):
        # The executor's form: the op's launches replayed as one CUDA graph per step;
        # per-kernel times come from profiled eager passes of the same launches.
        graph = ctx.capture(wl.step)
        wl.profile_step = wl.step
        wl.step = graph.launch
    flush = torch.empty(512 * 1024 * 1024 // 4, dtype=torch.float32, device="cuda")

    def barrier():
        if world > 1:
            dist.barrier()

    # warm-up
    for _ in range(args.warmup):
        wl.step()
        flush_l2(flush)
    ctx.synchronize()

    K = args.steps
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(K)]
    stops = [torch.cuda.Event(enable_timing=True) for _ in range(K)]
    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.3)
    ctx.profile_reset()
    ctx.profile(True)
    launches0 = ctx.launch_count()
    barrier()
    torch.cuda.synchronize()
    for i in range(K):
        starts[i].record(stream)
        wl.step()
        stops[i].record(stream)
        flush_l2(flush)
    torch.cuda.synchronize()
    barrier()
    launches = ctx.launch_count() - launches0
    ctx.profile(False)
    ctx.synchronize()
    step_ms = sum(s.elapsed_time(e) for s, e in zip(starts, stops)) / K
    if hasattr(wl, "profile_step"):
        # Graph replays carry no per-kernel events: count the plan's launches
        # from one eager pass and time its kernels over a profiled eager pass.
        ctx.profile_reset()
        l0 = ctx.launch_count()
        wl.profile_step()
        ctx.synchronize()
        launches = (ctx.launch_count() - l0) * K
        ctx.profile_reset()
        ctx.profile(True)
        for _ in range(args.profile_steps):
            wl.profile_step()
            flush_l2(flush)
        ctx.synchronize()
        ctx.profile(False)
    names = wl.main_kernel if isinstance(wl.main_kernel, tuple) else (wl.main_kernel,)
    kern_ms, kern_n = 0.0, 0
    for name in names:
        ms_, n_ = ctx.profile_read(name)
        kern_ms, kern_n = kern_ms + ms_, kern_n + n_
    all_ms, _ = ctx.profile_read("")
    ctx.profile_reset()

    # e2e through the public API with pinned host buffers
    KE = max(1, min(K, args.e2e_steps))
    if hasattr(wl, "e2e_pipelined"):
        # a serving loop: its own step count (not capped by --steps), so the
        # pipeline's fill (first H2D) and drain (last D2H) stay a small part
        KE = max(1, args.e2e_steps)
        e2e_ms = wl.e2e_pipelined(args.warmup, KE, barrier)
        e2e_mode = wl.e2e_mode
    else:
        for _ in range(max(1, args.warmup)):
            wl.e2e_step()
        ctx.synchronize()
        e_starts = [torch.cuda.Event(enable_timing=True) for _ in range(KE)]
        e_stops = [torch.cuda.Event(enable_timing=True) for _ in range(KE)]
        barrier()
        torch.cuda.synchronize()
        for i in range(KE):
            e_starts[i].record(stream)
            wl.e2e_step()
            e_stops[i].record(stream)
            flush_l2(flush)
        torch.cuda.synchronize()
        barrier()
        e2e_ms = sum(s.elapsed_time(e) for s, e in zip(e_starts, e_stops)) / KE
        e2e_mode = "serial: H2D, compute, D2H per step, L2 flushed between steps"
    clocks = sampler.stop()

    t = torch.tensor([step_ms, e2e_ms], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    step_ms_max, e2e_ms_max = t.tolist()

    result = None
    if rank == 0:
        units = wl.units_per_step() * world
        value = _scale(units / (step_ms_max * 1e-3)) if wl.unit in ("TFLOP/s", "TOP/s") else units / (step_ms_max * 1e-3)
        e2e_value = _scale(units / (e2e_ms_max * 1e-3)) if wl.unit in ("TFLOP/s", "TOP/s") else units / (e2e_ms_max * 1e-3)
        kern_avg_ms = kern_ms / max(1, kern_n)
        if wl.bound == "tensor":
            # burst figure for a kernel timed alone; sustained for kernels timed inside a long step
            pkey = "bf16_tflops_sustained" if getattr(wl, "long_step", False) else "bf16_tflops"
            peak = peaks.get(pkey, FALLBACK_PEAKS[pkey]) / 2.0 / 3.0
            achieved = _scale(wl.main_kernel_units() / (kern_avg_ms * 1e-3))
            rl = {"bound": "tensor", "achieved": round(achieved, 2), "peak": round(peak, 2), "unit": "TFLOP/s",
                  "frac": round(achieved / peak, 4), "traffic": args.traffic,
                  "kernel": "+".join(names), "kernel_ms": round(kern_avg_ms, 5), "kernel_share": round(kern_ms / max(all_ms, 1e-12), 4),
                  "peak_basis": f"3xTF32 = {pkey}/2 (kind::tf32 rate) /3 products, {pkey} of {peaks_kind} "
                                f"{peaks.get(pkey)}; frac of {peaks_kind}"}
        else:
            peak = peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"])
            achieved = wl.main_kernel_units() / (kern_avg_ms * 1e-3) / 1e9
            rl = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                  "frac": round(achieved / peak, 4), "traffic": args.traffic, "kernel": "+".join(names),
                  "kernel_ms": round(kern_avg_ms, 5), "peak_basis": f"hbm_gbs of {peaks_kind}"}
        bi, bo = wl.e2e_bytes()
        result = {
            "metric": METRIC, "value": round(value, 3), "unit": wl.unit, "n_gpus": world, "steps": K,
            "warmup": args.warmup, "ms_per_step": round(step_ms_max, 5), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded numpy), per rank",
            "config": dict(wl.config, l2="flushed between steps (512 MiB write outside the events)",
                           parallelism=f"dp{world} (independent shards, no data-path collective)"),
            "e2e": {"value": round(e2e_value, 3), "unit": wl.unit, "h2d_bytes_per_step": bi, "d2h_bytes_per_step": bo,
                    "ms_per_step": round(e2e_ms_max, 5), "steps": KE, "mode": e2e_mode},
            "roofline": rl,
            "gpu_launches": int(launches),
            "clocks": clocks,
        }
        if not args.no_cpu_baseline and world == 1:
            cores = physical_cores()
            base = wl.cpu_sample(cores)
            base.update(kind="port", cpu=cpu_model())
            try:
                b4 = wl.cpu_sample(min(4, cores))
                base["value_4_threads"] = b4["value"]
            except Exception:  # pragma: no cover
                pass
            result["cpu_baseline"] = base
    if graph is not None:
        graph.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    ctx.close()
    return result


def run_reference(args) -> dict | None:
    """Time the reference's CPU algorithm (oracle port) on the host cores."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return None
    cores = physical_cores()
    os.environ.setdefault("ONNXSHARP_THREADS", str(cores))

    class _Ctx:  # the CPU arm needs no GPU context
        pass

    wl = CPU_WORKLOADS[args.workload]()
    vals = []
    for _ in range(max(1, args.warmup)):
        wl.cpu_sample(cores)
    t0 = time.perf_counter()
    for _ in range(args.ref_steps):
        vals.append(wl.cpu_sample(cores))
    dt = time.perf_counter() - t0
    value = statistics.median(v["value"] for v in vals)
    return {
        "metric": METRIC, "impl": "reference", "value": round(value, 5), "unit": wl.unit, "n_gpus": world,
        "steps": args.ref_steps, "warmup": args.warmup, "ms_per_step": round(dt / args.ref_steps * 1e3, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": wl.config,
        "cpu_baseline": {"value": round(value, 5), "unit": wl.unit, "cores": cores, "kind": "port",
                         "sample": vals[0]["sample"], "cpu": cpu_model()},
        "e2e": {"value": round(value, 5), "unit": wl.unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "reference is C# (OnnxSharp); no .NET runtime on this box, so the CPU restatement of its kernels "
                "(oracle/) is timed with all physical cores",
    }


class CpuGemm:
    unit = "TFLOP/s"

    def __init__(self):
        m, k, n = 2048, 512, 2048
        rng = np.random.default_rng(1234)
        self.a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
        self.b = rng.uniform(-1, 1, (k, n)).astype(np.float32)
        self.bias = rng.uniform(-1, 1, n).astype(np.float32)
        self.config = {"workload": GemmWorkload.name, "m": m, "k": k, "n": n, "bias": True}

    def cpu_sample(self, threads):
        import oracle

        t0 = time.perf_counter()
        oracle.gemm(self.a, self.b, col_bias=self.bias, threads=threads)
        dt = time.perf_counter() - t0
        return {"value": 2.0 * self.a.shape[0] * self.a.shape[1] * self.b.shape[1] / dt / 1e12,
                "sample": "one full 2048x512x2048 GEMM+bias per step"}


class CpuConv:
    """One image of BASELINE config 2 per step through the oracle's im2col-order conv + SiLU."""

    unit = "TFLOP/s"

    def __init__(self, x=None, w=None, b=None):
        if x is None:
            x, w, b = conv_inputs(4321, 1)
        self.x, self.w, self.b = x[:1], w, b
        self.config = {"workload": ConvWorkload.name, "batch": 16, "in": [16, 64, 160, 160],
                       "weight": [128, 64, 3, 3], "stride": 1, "pad": 1, "act": "SiLU"}

    def cpu_sample(self, threads):
        import oracle

        t0 = time.perf_counter()
        oracle.conv2d(self.x, self.w, self.b, pads=(1, 1, 1, 1), act=1, threads=threads)
        dt = time.perf_counter() - t0
        return {"value": CONV_FLOPS_PER_IMAGE / dt / 1e12, "unit": self.unit, "cores": threads,
                "sample": f"1 of 16 images per step (3x3 conv 64->128 @160x160 + SiLU), {dt:.2f} s"}


class CpuDqmm:
    """The full config-3 DynamicQuantizeMatMul per step through the oracle (F32-substitute GEMM, as the reference)."""

    unit = "TOP/s"

    def __init__(self, a=None, w=None, ws=None, b=None):
        if a is None:
            a, w, ws, b = dqmm_inputs(777)
        self.a, self.w, self.ws, self.b = a, w, ws, b
        self.config = {"workload": DqmmWorkload.name, "m": a.shape[0], "k": a.shape[1], "n": w.shape[1]}

    def cpu_sample(self, threads):
        import oracle

        t0 = time.perf_counter()
        oracle.dqmm(self.a, self.w, 0, self.ws, self.b, threads=threads)
        dt = time.perf_counter() - t0
        ops = 2.0 * self.a.shape[0] * self.a.shape[1] * self.w.shape[1]
        return {"value": ops / dt / 1e12, "unit": self.unit, "cores": threads,
                "sample": f"full {self.a.shape[0]}x{self.a.shape[1]}x{self.w.shape[1]} DQMM per step, {dt:.2f} s"}


class CpuYolo:
    """One image per step through the oracle executor of the same plan."""

    unit = "images/s"

    def __init__(self, g=None, params=None, images=None):
        from onnxsharp_b200 import yolo

        if g is None:
            g = yolo.build_yolo11n()
            params = yolo.init_params(g, 2024)
            images = np.random.default_rng(9000).uniform(0, 1, (1, 3, 640, 640)).astype(np.float32)
        self.g, self.params, self.images = g, params, images[:1]
        self.config = {"workload": YoloWorkload.name, "batch_per_gpu": 64, "input": [64, 3, 640, 640],
                       "output": [64, 84, 8400]}

    def cpu_sample(self, threads):
        from oracle import yolo_ref

        t0 = time.perf_counter()
        yolo_ref.run(self.g, self.params, self.images, threads=threads)
        dt = time.perf_counter() - t0
        return {"value": 1.0 / dt, "unit": self.unit, "cores": threads,
                "sample": f"1 image (of 64) per step through the plan, {dt:.2f} s"}


class CpuAttention:
    """8 of the 64 sequences per step through the oracle (projection GEMMs + ComputeBlocks)."""

    unit = "TFLOP/s"

    def __init__(self, x=None, ws=None):
        if x is None:
            rng = np.random.default_rng(5150)
            x = rng.normal(0, 1, (64 * 128, 512)).astype(np.float32)
            lim = np.sqrt(6.0 / 1024)
            ws = [rng.uniform(-lim, lim, (512, 512)).astype(np.float32) for _ in range(4)]
        self.x, self.ws = x[:8 * 128], ws
        self.config = {"workload": AttentionWorkload.name, "x": [64, 128, 512], "heads": 8, "head_dim": 64}

    def cpu_sample(self, threads):
        import oracle

        t0 = time.perf_counter()
        q, k, v = (oracle.gemm(self.x, w, threads=threads).reshape(8, 128, 512) for w in self.ws[:3])
        o = oracle.attention(q, k, v, heads=8, scale=0.125, threads=threads)
        oracle.gemm(o.reshape(8 * 128, 512), self.ws[3], threads=threads)
        dt = time.perf_counter() - t0
        return {"value": ATTN_FLOPS / 8 / dt / 1e12, "unit": self.unit, "cores": threads,
                "sample": f"8 of 64 sequences per step, {dt:.2f} s"}


CPU_WORKLOADS = {"gemm": CpuGemm, "conv": CpuConv, "dqmm": CpuDqmm, "yolo": CpuYolo, "attention": CpuAttention}


def main() -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", default=DEFAULT_WORKLOAD, choices=sorted(WORKLOADS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--e2e-steps", type=int, default=None)
    ap.add_argument("--profile-steps", type=int, default=None,
                    help="eager profiled steps for the dominant-kernel timing of graph-replayed workloads")
    ap.add_argument("--ref-steps", type=int, default=5)
    ap.add_argument("--traffic", type=float, default=None,
                    help="dram bytes per dominant-kernel launch from an ncu capture (reported as-is)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.traffic is None:
        args.traffic = load_traffic(args.workload)
    if args.profile_steps is None:
        args.profile_steps = 5 if args.workload == "yolo" else 50
    if args.e2e_steps is None:
        args.e2e_steps = {"yolo": 30, "conv": 50}.get(args.workload, 200)
    if args.steps is None:
        args.steps = DEFAULT_STEPS.get(args.workload, 100)
    args.warmup = max(3, args.warmup)
    if args.impl == "reference":
        res = run_reference(args)
    else:
        peaks, kind = load_peaks()
        res = run_ours(args, peaks, kind)
    if res is not None:
        print(json.dumps(res), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
