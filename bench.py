#!/usr/bin/env python
"""bench.py — throughput of OnnxSharp's matrix-multiply hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl ours|reference]

One process per GPU (torchrun for N > 1, NCCL process group). The headline
workload (default: the YOLO11n-shaped detector at a global batch of 64,
BASELINE config 5) is sharded by image over the N GPUs and the shards'
[B/N, 84, 8400] outputs are all-gathered over NVLink inside every timed step
(strong scaling: the global batch is the same at every N). Every other
BASELINE config (GEMM, conv B=1 / B=16, DQMM, the attention block, YOLO B=1 /
B=8) is measured in the same process and reported under "configs", sharded the
same way (rows, images or sequences; DQMM adds an NCCL all-reduce of the
per-tensor range; a batch smaller than N runs as replicas).

Timed region: W untimed warm-up steps, then exactly K steps bracketed by a
barrier + cuda synchronize on both sides. Every step is timed with CUDA events
on the stream the kernels and collectives run on; L2 is flushed (a 512 MiB
device write, then a read of it, so no dirty line of the flush is left to
write back) between steps, outside the events; the max over ranks is
reported. `value` is the whole-job throughput with inputs resident in HBM;
`e2e` is the same metric through the library's public API from pinned host
memory (YOLO: frames in, detections out; the other configs: input tensor in,
whole output tensor back on rank 0). `roofline` reports the dominant kernel
against the measured peaks in MEASURED_PEAKS.json; `cpu_baseline` times the
CPU oracle (a restatement of the reference's CPU kernels) on a bounded sample,
beside the reference's own published CPU figures.

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



# ----------------------------------------------------------------- sharding
class Shard:
    """This rank's part of a batch-sharded job (one process per GPU).

    Images (YOLO, conv), sequences (attention) and rows (GEMM, DQMM) are
    independent, so each rank computes a contiguous shard; the shards' outputs
    are all-gathered over NVLink (NCCL) inside the timed step so that every
    rank ends the step holding the whole batch's output, as the reference's
    single Net.Forward returns it (src/OnnxSharp/Core/Net.cs:258-262). A batch
    smaller than the GPU count (B=1) cannot be split: every rank then runs its
    own replica and nothing is exchanged ("replicas")."""

    def __init__(self, world: int, rank: int, group=None):
        self.world, self.rank, self.group = world, rank, group

    def plan(self, n: int) -> tuple[int, int, bool]:
        """(start, count, replicas) of this rank's part of n items."""
        from onnxsharp_b200.shard import shard_range

        if self.world == 1 or n % self.world != 0:
            return 0, n, self.world > 1
        lo, hi = shard_range(n, self.world, self.rank)
        return lo, hi - lo, False

    def all_gather(self, full, local) -> None:
        import torch.distributed as dist

        dist.all_gather_into_tensor(full, local, group=self.group)

    def barrier(self) -> None:
        import torch.distributed as dist

        if self.world > 1:
            dist.barrier(group=self.group)


# ----------------------------------------------------------------- workloads
class Workload:
    """One BASELINE config, sharded over the ranks. A step = compute() (this
    rank's shard; captured as one CUDA graph where `graphed`) + collect() (the
    NCCL all-gather of the shards, or nothing on one GPU / for replicas)."""

    key = ""
    name = ""
    unit = "TFLOP/s"
    bound = "tensor"
    main_kernel: tuple = ()
    graphed = True
    long_step = False
    replicas = False

    def units_per_step(self) -> float:    # whole job (all ranks) per step
        raise NotImplementedError

    def compute(self):
        raise NotImplementedError

    def collect(self):
        pass

    def collect_bytes(self) -> int:        # bytes each rank receives from the others per step
        return 0

    def e2e_step(self):
        raise NotImplementedError

    def e2e_bytes(self) -> tuple[int, int]:  # whole job per step
        raise NotImplementedError

    def main_kernel_units(self) -> float:  # algorithmic FLOPs (or bytes) of one dominant-kernel launch
        raise NotImplementedError

    def cpu_sample(self, threads: int, budget_s: float) -> dict:
        raise NotImplementedError

    def close(self):
        pass


def _dev():
    import torch

    return torch.device("cuda", torch.cuda.current_device())


def _tflops(x: float) -> float:
    return x / 1e12


def _timed(fn, budget_s: float, min_reps: int = 1):
    """Repeat fn until budget_s seconds have passed (at least min_reps times); returns (reps, seconds)."""
    t0 = time.perf_counter()
    reps = 0
    while reps < min_reps or time.perf_counter() - t0 < budget_s:
        fn()
        reps += 1
    return reps, time.perf_counter() - t0


class GemmWorkload(Workload):
    """Config 1: MatMul+Add(bias) A[2048,512] x B[512,2048] + bias[2048], U(-1,1); rows of A sharded."""

    key = "gemm"
    name = "matmul_bias_f32_2048x512x2048"
    main_kernel = ("k_gemm_tf32x3",)

    def __init__(self, ctx, sh: Shard, m=2048, k=512, n=2048):
        import torch

        from onnxsharp_b200.runtime import GemmWeights

        self.ctx, self.sh, self.m, self.k, self.n = ctx, sh, m, k, n
        rng = np.random.default_rng(1234)
        self.a_h = rng.uniform(-1, 1, (m, k)).astype(np.float32)
        self.b_h = rng.uniform(-1, 1, (k, n)).astype(np.float32)
        self.bias_h = rng.uniform(-1, 1, n).astype(np.float32)
        lo, cnt, self.replicas = sh.plan(m)
        self.rows = cnt
        dev = _dev()
        self.a = torch.from_numpy(self.a_h[lo:lo + cnt]).to(dev)
        self.bias = torch.from_numpy(self.bias_h).to(dev)
        self.w = GemmWeights(ctx, torch.from_numpy(self.b_h).to(dev), k, n)
        self.c = torch.empty((cnt, n), dtype=torch.float32, device=dev)
        self.gather = sh.world > 1 and not self.replicas
        self.c_full = torch.empty((m, n), dtype=torch.float32, device=dev) if self.gather else self.c
        self.a_pin = torch.from_numpy(self.a_h[lo:lo + cnt].copy()).pin_memory()
        self.c_pin = torch.empty(self.c_full.shape, dtype=torch.float32).pin_memory()
        self.a2, self.c2 = torch.empty_like(self.a), torch.empty_like(self.c)
        self.c2_full = torch.empty_like(self.c_full) if self.gather else self.c2
        self.config = {"workload": self.name, "m": m, "k": k, "n": n, "rows_per_gpu": cnt, "bias": True,
                       "precision": "3xTF32 (tcgen05 kind::tf32), FP32 in/out"}

    def units_per_step(self):
        return 2.0 * self.m * self.k * self.n * (self.sh.world if self.replicas else 1)

    def main_kernel_units(self):
        return 2.0 * self.rows * self.k * self.n

    def compute(self):
        from onnxsharp_b200.runtime import gemm_bias

        gemm_bias(self.ctx, self.a, self.w, self.bias, out=self.c)

    def collect(self):
        if self.gather:
            self.sh.all_gather(self.c_full, self.c)

    def collect_bytes(self):
        return (self.sh.world - 1) * self.c.numel() * 4 if self.gather else 0

    def e2e_step(self):
        from onnxsharp_b200.runtime import gemm_bias

        self.ctx.memcpy_htod(self.a2, self.a_pin, self.a_pin.numel() * 4)
        gemm_bias(self.ctx, self.a2, self.w, self.bias, out=self.c2)
        if self.gather:
            self.sh.all_gather(self.c2_full, self.c2)
        if self.sh.rank == 0:
            self.ctx.memcpy_dtoh(self.c_pin, self.c2_full, self.c_pin.numel() * 4)

    def e2e_bytes(self):
        r = self.sh.world if self.replicas else 1
        return self.m * self.k * 4 * r, self.m * self.n * 4

    def cpu_sample(self, threads, budget_s):
        return CpuGemm(self.a_h, self.b_h, self.bias_h).cpu_sample(threads, budget_s)


def conv_inputs(seed: int, batch: int):
    """Config 2 synthetic data: x U(0,1), W He-normal, b N(0, 0.01)."""
    rng = np.random.default_rng(seed)
    x = rng.uniform(0, 1, (batch, 64, 160, 160)).astype(np.float32)
    w = (rng.normal(0, 1, (128, 64, 3, 3)) * np.sqrt(2.0 / (64 * 9))).astype(np.float32)
    b = rng.normal(0, 0.01, 128).astype(np.float32)
    return x, w, b


CONV_FLOPS_PER_IMAGE = 2.0 * 128 * 160 * 160 * 64 * 9


class ConvWorkload(Workload):
    """Config 2: fused Conv+SiLU, x[B,64,160,160] -> y[B,128,160,160], 3x3 s1 p1, B in {1, 16}; images sharded."""

    main_kernel = ("k_conv_tf32x3", "k_conv_px_tf32x3")  # channel-major or pixel-major tiles, one launch per conv

    def __init__(self, ctx, sh: Shard, batch: int = 16):
        import torch

        from onnxsharp_b200.runtime import ConvWeights

        self.ctx, self.sh, self.batch = ctx, sh, batch
        self.key = f"conv_b{batch}"
        self.name = f"conv3x3_silu_f32_b{batch}_64to128_160x160"
        x, w, b = conv_inputs(4321, batch)
        self.x_h, self.w_h, self.b_h = x, w, b
        lo, cnt, self.replicas = sh.plan(batch)
        self.local = cnt
        dev = _dev()
        self.x = torch.from_numpy(x[lo:lo + cnt]).to(dev)
        self.b = torch.from_numpy(b).to(dev)
        self.w = ConvWeights(ctx, torch.from_numpy(w).to(dev), w.shape)
        self.y = torch.empty((cnt, 128, 160, 160), dtype=torch.float32, device=dev)
        self.gather = sh.world > 1 and not self.replicas
        self.y_full = torch.empty((batch, 128, 160, 160), dtype=torch.float32, device=dev) if self.gather else self.y
        self.x_pin = torch.from_numpy(x[lo:lo + cnt].copy()).pin_memory()
        self.y_pin = torch.empty(self.y_full.shape, dtype=torch.float32).pin_memory()
        self.x2, self.y2 = torch.empty_like(self.x), torch.empty_like(self.y)
        self.y2_full = torch.empty_like(self.y_full) if self.gather else self.y2
        self.config = {"workload": self.name, "batch": batch, "images_per_gpu": cnt, "in": [batch, 64, 160, 160],
                       "weight": [128, 64, 3, 3], "stride": 1, "pad": 1, "act": "SiLU",
                       "precision": "3xTF32 implicit GEMM (tcgen05 kind::tf32), FP32 in/out"}

    def units_per_step(self):
        return CONV_FLOPS_PER_IMAGE * self.batch * (self.sh.world if self.replicas else 1)

    def main_kernel_units(self):
        return CONV_FLOPS_PER_IMAGE * self.local

    def _run(self, x, y):
        from onnxsharp_b200 import ACT_SILU
        from onnxsharp_b200.runtime import conv2d

        conv2d(self.ctx, x, self.w, self.b, (1, 1), (1, 1, 1, 1), (1, 1), 1, ACT_SILU, out=y)

    def compute(self):
        self._run(self.x, self.y)

    def collect(self):
        if self.gather:
            self.sh.all_gather(self.y_full, self.y)

    def collect_bytes(self):
        return (self.sh.world - 1) * self.y.numel() * 4 if self.gather else 0

    def e2e_step(self):
        self.ctx.memcpy_htod(self.x2, self.x_pin, self.x_pin.numel() * 4)
        self._run(self.x2, self.y2)
        if self.gather:
            self.sh.all_gather(self.y2_full, self.y2)
        if self.sh.rank == 0:
            self.ctx.memcpy_dtoh(self.y_pin, self.y2_full, self.y_pin.numel() * 4)

    def e2e_bytes(self):
        r = self.sh.world if self.replicas else 1
        return self.x_h.nbytes * r, self.y_pin.numel() * 4

    def cpu_sample(self, threads, budget_s):
        return CpuConv(self.x_h, self.w_h, self.b_h, self.batch).cpu_sample(threads, budget_s)


def dqmm_inputs(seed: int, m=4096, k=512, n=2048):
    """Config 3: A N(0,1), W int8 U[-127,127], w_scale U(0.001,0.02), bias N(0, 0.01)."""
    rng = np.random.default_rng(seed)
    a = rng.normal(0, 1, (m, k)).astype(np.float32)
    w = rng.integers(-127, 128, (k, n)).astype(np.int8)
    ws = rng.uniform(0.001, 0.02, n).astype(np.float32)
    b = rng.normal(0, 0.01, n).astype(np.float32)
    return a, w, ws, b


class DqmmWorkload(Workload):
    """Config 3: DynamicQuantizeMatMul A[4096,512] f32 x W int8 [512,2048] -> Y[4096,2048] f32.

    Rows are sharded; the per-tensor range is the one real exchange step: each
    rank reduces its rows' {min, max}, the ranks all-reduce it (NCCL, 2 floats)
    and every shard quantises with the global range, so q and the int32
    accumulators are those of the unsharded tensor."""

    key = "dqmm"
    name = "dqmm_u8s8_4096x512x2048"
    unit = "TOP/s"
    main_kernel = ("k_dqmm_i8",)
    bound = "hbm"

    def __init__(self, ctx, sh: Shard, m=4096, k=512, n=2048):
        import torch

        from onnxsharp_b200.runtime import DqmmWeights

        self.ctx, self.sh, self.m, self.k, self.n = ctx, sh, m, k, n
        a, w, ws, b = dqmm_inputs(777, m, k, n)
        self.a_h, self.w_h, self.ws_h, self.b_h = a, w, ws, b
        lo, cnt, self.replicas = sh.plan(m)
        self.rows, self.row0 = cnt, lo
        dev = _dev()
        self.a = torch.from_numpy(a[lo:lo + cnt]).to(dev)
        self.ws = torch.from_numpy(ws).to(dev)
        self.b = torch.from_numpy(b).to(dev)
        self.w = DqmmWeights(ctx, torch.from_numpy(w).to(dev), k, n, None)
        self.y = torch.empty((cnt, n), dtype=torch.float32, device=dev)
        self.sharded = sh.world > 1 and not self.replicas
        self.graphed = not self.sharded  # the range all-reduce sits between two library calls
        self.mm = torch.zeros(2, dtype=torch.float32, device=dev)
        self.y_full = torch.empty((m, n), dtype=torch.float32, device=dev) if self.sharded else self.y
        self.a_pin = torch.from_numpy(a[lo:lo + cnt].copy()).pin_memory()
        self.y_pin = torch.empty(self.y_full.shape, dtype=torch.float32).pin_memory()
        self.a2, self.y2 = torch.empty_like(self.a), torch.empty_like(self.y)
        self.y2_full = torch.empty_like(self.y_full) if self.sharded else self.y2
        self.config = {"workload": self.name, "m": m, "k": k, "n": n, "rows_per_gpu": cnt,
                       "precision": "dynamic per-tensor u8 activations x s8 weights -> s32 (tcgen05 kind::i8), "
                                    "FP32 epilogue bit-identical to the reference"}
        if self.sharded:
            self.config["exchange"] = "NCCL all-reduce of the shards' {min, max} (2 floats) before quantising"

    def units_per_step(self):
        return 2.0 * self.m * self.k * self.n * (self.sh.world if self.replicas else 1)

    def main_kernel_units(self):
        kp = (self.k + 127) // 128 * 128
        return self.rows * kp + self.n * kp + self.rows * self.n * 4 + self.n * 16

    def _run(self, a, y):
        from onnxsharp_b200 import shard
        from onnxsharp_b200.runtime import dqmm, minmax

        if self.sharded:
            minmax(self.ctx, a, out=self.mm)
            shard.global_minmax(self.mm, group=self.sh.group)
            dqmm(self.ctx, a, self.w, self.ws, self.b, out=y, minmax_override=self.mm, row0=self.row0,
                 rows_total=self.m)
        else:
            dqmm(self.ctx, a, self.w, self.ws, self.b, out=y)

    def compute(self):
        self._run(self.a, self.y)

    def collect(self):
        if self.sharded:
            self.sh.all_gather(self.y_full, self.y)

    def collect_bytes(self):
        return (self.sh.world - 1) * self.y.numel() * 4 if self.sharded else 0

    def e2e_step(self):
        self.ctx.memcpy_htod(self.a2, self.a_pin, self.a_pin.numel() * 4)
        self._run(self.a2, self.y2)
        if self.sharded:
            self.sh.all_gather(self.y2_full, self.y2)
        if self.sh.rank == 0:
            self.ctx.memcpy_dtoh(self.y_pin, self.y2_full, self.y_pin.numel() * 4)

    def e2e_bytes(self):
        r = self.sh.world if self.replicas else 1
        return self.a_h.nbytes * r, self.y_pin.numel() * 4

    def cpu_sample(self, threads, budget_s):
        return CpuDqmm(self.a_h, self.w_h, self.ws_h, self.b_h).cpu_sample(threads, budget_s)


ATTN_FLOPS = 4 * 2.0 * 8192 * 512 * 512 + 2 * 2.0 * 64 * 8 * 128 * 128 * 64


class AttentionWorkload(Workload):
    """Config 4: X[64,128,512] N(0,1) -> Q/K/V projections (MatMul+bias, Xavier-uniform, zero bias)
    -> FusedAttention (H=8, D=64, scale 1/8) -> output projection; sequences sharded."""

    key = "attention"
    name = "attention_block_b64_t128_h8_d64"
    main_kernel = ("k_gemm_tf32x3",)

    def __init__(self, ctx, sh: Shard):
        import torch

        from onnxsharp_b200.runtime import GemmWeights

        self.ctx, self.sh = ctx, sh
        rng = np.random.default_rng(5150)
        self.B, self.T, self.C, self.H = 64, 128, 512, 8
        x = rng.normal(0, 1, (self.B * self.T, self.C)).astype(np.float32)
        lim = np.sqrt(6.0 / (self.C + self.C))
        ws = [rng.uniform(-lim, lim, (self.C, self.C)).astype(np.float32) for _ in range(4)]
        self.x_h, self.ws_h = x, ws
        lo, cnt, self.replicas = sh.plan(self.B)
        self.seqs = cnt
        rows = slice(lo * self.T, (lo + cnt) * self.T)
        dev = _dev()
        self.x = torch.from_numpy(x[rows]).to(dev)
        self.bias = torch.zeros(self.C, device=dev)
        self.w = [GemmWeights(ctx, torch.from_numpy(w).to(dev), self.C, self.C) for w in ws]
        self.qkv = [torch.empty(cnt * self.T, self.C, device=dev) for _ in range(3)]
        self.x_split = (torch.empty(cnt * self.T, self.C, device=dev), torch.empty(cnt * self.T, self.C, device=dev))
        self.o = torch.empty(cnt, self.T, self.C, device=dev)
        self.y = torch.empty(cnt * self.T, self.C, device=dev)
        self.gather = sh.world > 1 and not self.replicas
        self.y_full = torch.empty(self.B * self.T, self.C, device=dev) if self.gather else self.y
        self.x_pin = torch.from_numpy(x[rows].copy()).pin_memory()
        self.y_pin = torch.empty(self.y_full.shape).pin_memory()
        self.x2 = torch.empty_like(self.x)
        self.config = {"workload": self.name, "x": [64, 128, 512], "heads": 8, "head_dim": 64,
                       "sequences_per_gpu": cnt,
                       "precision": "3xTF32 tcgen05 (projections and QK^T / PV), FP32 softmax"}

    def units_per_step(self):
        return ATTN_FLOPS * (self.sh.world if self.replicas else 1)

    def main_kernel_units(self):
        return 2.0 * self.seqs * self.T * 512 * 512

    def _run(self, x):
        from onnxsharp_b200.runtime import attention, gemm_bias, gemm_bias_presplit, gemm_split_a

        # the three projections share their input: split it once
        split = gemm_split_a(self.ctx, x, self.C, out=self.x_split)
        for w, out in zip(self.w[:3], self.qkv):
            gemm_bias_presplit(self.ctx, split, w, self.bias, out=out)
        q, k, v = (t.view(self.seqs, self.T, self.C) for t in self.qkv)
        attention(self.ctx, q, k, v, self.H, 0.125, out=self.o)
        gemm_bias(self.ctx, self.o.view(self.seqs * self.T, self.C), self.w[3], self.bias, out=self.y)

    def compute(self):
        self._run(self.x)

    def collect(self):
        if self.gather:
            self.sh.all_gather(self.y_full, self.y)

    def collect_bytes(self):
        return (self.sh.world - 1) * self.y.numel() * 4 if self.gather else 0

    def e2e_step(self):
        self.ctx.memcpy_htod(self.x2, self.x_pin, self.x_pin.numel() * 4)
        self._run(self.x2)
        self.collect()
        if self.sh.rank == 0:
            self.ctx.memcpy_dtoh(self.y_pin, self.y_full, self.y_pin.numel() * 4)

    def e2e_bytes(self):
        r = self.sh.world if self.replicas else 1
        return self.x_h.nbytes * r, self.y_pin.numel() * 4

    def cpu_sample(self, threads, budget_s):
        return CpuAttention(self.x_h, self.ws_h).cpu_sample(threads, budget_s)


FRAME_HW = (720, 1280)  # source frames of the serving e2e: 1280x720 BGR u8 (letterboxed to 640x640 on the device)


class YoloWorkload(Workload):
    """Config 5: random-init YOLO11n-shaped detector, [B,3,640,640] U(0,1) -> [B,84,8400], B in {1, 8, 64}
    global, images sharded over the GPUs and the [B/N,84,8400] outputs all-gathered.

    A step is one replay of the plan's CUDA graph plus the all-gather. The
    dominant kernels are the tensor-core convs (channel-major implicit GEMM,
    pixel-major 1x1 / small-image convs); their time comes from a profiled
    eager pass (event timing cannot be inserted into a graph replay).

    e2e is the reference's YoloDetector.Detect path (frames in, detections
    out, onnxsharp_b200.serve.DetectPipeline): u8 1280x720 frames from pinned
    host memory, batched letterbox + forward + decode/NMS as one CUDA graph,
    the packed detections all-gathered and read back on rank 0; batches are
    pipelined (H2D, graph and D2H of consecutive batches overlap)."""

    unit = "images/s"
    main_kernel = ("k_conv_tf32x3", "k_conv_px_tf32x3")
    long_step = True

    def __init__(self, ctx, sh: Shard, batch: int = 64, tensor_e2e: bool = False):
        import torch

        from onnxsharp_b200 import yolo

        self.ctx, self.sh, self.batch = ctx, sh, batch
        self.key = f"yolo_b{batch}"
        self.name = f"yolo11n_shaped_b{batch}_640"
        lo, cnt, self.replicas = sh.plan(batch)
        self.local = cnt
        self.g = yolo.build_yolo11n()
        self.params = yolo.init_params(self.g, 2024)
        self.net = yolo.Net(ctx, self.g, self.params, cnt)
        rng = np.random.default_rng(9000)
        self.images_h = rng.uniform(0, 1, (batch, 3, 640, 640)).astype(np.float32)
        self.net.input_view().copy_(torch.from_numpy(self.images_h[lo:lo + cnt]))
        self.gather = sh.world > 1 and not self.replicas
        dev = _dev()
        self.out_full = (torch.empty((batch, 84, 8400), dtype=torch.float32, device=dev) if self.gather
                         else self.net.output)
        self.flops_img = yolo.flops_per_image(self.g)
        self.tc_flops = sum(self._node_flops(n) for n in self.g.nodes
                            if n.op == "conv" and yolo.Net.tensor_core(n)) * cnt
        self.tc_launches = sum(1 for n in self.g.nodes if n.op == "conv" and yolo.Net.tensor_core(n))
        self.net.forward(use_graph=True)  # capture
        ctx.synchronize()
        self.pipe = None
        self.tensor_e2e = tensor_e2e
        self.config = {"workload": self.name, "global_batch": batch, "images_per_gpu": cnt,
                       "input": [batch, 3, 640, 640], "output": [batch, 84, 8400],
                       "gflop_per_image": round(self.flops_img / 1e9, 3),
                       "arena_mib": round(self.net.arena_bytes / 2 ** 20, 1),
                       "precision": "FP32 in/out; wide convs 3xTF32 tcgen05 (k x k implicit GEMM on NHWC hi/lo, 1x1 "
                                    "straight from NCHW), narrow and depthwise convs FP32 CUDA-core FMA, glue FP32 CUDA "
                                    "cores; conv Sigmoid/SiLU from hardware ex2/rcp (<= 2e-6 from the exact form)",
                       "plan": "static plan replayed as one CUDA graph; the Detect head's box and class branches on two more streams (lanes) beside the neck"}

    def _node_flops(self, n):
        y = n.outs[0]
        oh, ow = self.g.hw(y)
        return 2.0 * y.c * oh * ow * (n.ins[0].c // n.attrs["group"]) * n.attrs["k"] ** 2

    def units_per_step(self):
        return float(self.batch * (self.sh.world if self.replicas else 1))

    def main_kernel_units(self):
        return self.tc_flops / self.tc_launches

    def compute(self):
        self.net.forward(use_graph=True)

    def profile_compute(self):
        # one lane: every kernel on the profiled context, in plan order
        self.net.forward(use_graph=False, serial=True)

    def collect(self):
        if self.gather:
            self.sh.all_gather(self.out_full, self.net.output)

    def collect_bytes(self):
        return (self.sh.world - 1) * self.net.output.numel() * 4 if self.gather else 0

    # -- serving e2e: frames in, detections out
    def _pipeline(self):
        import torch

        from onnxsharp_b200.serve import DetectPipeline

        if self.pipe is None:
            self.pipe = DetectPipeline(self.net, frame_hw=FRAME_HW, bgr=True, depth=2, gather=self.gather,
                                       group=self.sh.group)
            rng = np.random.default_rng(77 + self.sh.rank)
            self.frames_pin, self.result_pin = [], []
            for _ in range(2):
                f, r = self.pipe.host_buffers()
                f.copy_(torch.from_numpy(rng.integers(0, 256, f.shape, dtype=np.uint8)))
                self.frames_pin.append(f)
                self.result_pin.append(r if self.sh.rank == 0 or not self.gather else None)
        return self.pipe

    def e2e_pipelined(self, warmup: int, steps: int) -> float:
        """ms per step of the serving loop, device-timed from the first H2D to the last D2H."""
        import torch

        pipe = self._pipeline()
        for i in range(max(1, warmup)):
            pipe.submit(self.frames_pin[i % 2], self.result_pin[i % 2])
        pipe.synchronize()
        self.sh.barrier()
        torch.cuda.synchronize()
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(pipe.h2d)
        for i in range(steps):
            pipe.submit(self.frames_pin[i % 2], self.result_pin[i % 2])
        stop.record(pipe.d2h)
        stop.synchronize()
        pipe.synchronize()
        self.sh.barrier()
        return start.elapsed_time(stop) / steps

    def e2e_bytes(self):
        r = self.sh.world if self.replicas else 1
        h2d = self.batch * r * FRAME_HW[0] * FRAME_HW[1] * 3
        pack = self.local * (300 * 6 + 1) * 4
        return h2d, pack * self.sh.world  # gathered to rank 0, or one pack per replica

    e2e_mode = ("pipelined serving loop (onnxsharp_b200.serve.DetectPipeline, depth 2): per step each GPU copies "
                "its images' 1280x720 BGR u8 frames from pinned host memory, one CUDA graph runs the batched "
                "letterbox and the forward pass, a second one on its own stream decode + NMS (conf 0.25, IoU 0.45, "
                "max 300 per image; beside the next batch's forward pass), the packed detections are all-gathered "
                "over NCCL and rank 0 reads the whole batch's detections back; device-timed from the first H2D to "
                "the last D2H, fill and drain included")

    def e2e_tensor(self, warmup: int, steps: int) -> float:
        """ms per step of FP32 tensor in / FP32 tensor out through yolo.HostPipeline (each rank its own images)."""
        import torch

        from onnxsharp_b200 import yolo

        pipe = yolo.HostPipeline(self.net, depth=2)
        rng = np.random.default_rng(5 + self.sh.rank)
        ins = [torch.from_numpy(rng.uniform(0, 1, self.net.inputs[0].shape).astype(np.float32)).pin_memory()
               for _ in range(2)]
        outs = [torch.empty(self.net.outputs[0].shape, dtype=torch.float32).pin_memory() for _ in range(2)]
        for i in range(max(1, warmup)):
            pipe.submit(ins[i % 2], outs[i % 2])
        pipe.synchronize()
        self.sh.barrier()
        torch.cuda.synchronize()
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(pipe.h2d)
        for i in range(steps):
            pipe.submit(ins[i % 2], outs[i % 2])
        stop.record(pipe.d2h)
        stop.synchronize()
        self.sh.barrier()
        return start.elapsed_time(stop) / steps

    def cpu_sample(self, threads, budget_s):
        return CpuYolo(self.g, self.params, self.images_h, self.batch).cpu_sample(threads, budget_s)

    def close(self):
        if getattr(self, "pipe", None) is not None:
            self.pipe.close()
        self.net.close()


WORKLOADS = {"gemm": lambda c, s: GemmWorkload(c, s), "conv_b16": lambda c, s: ConvWorkload(c, s, 16),
             "conv_b1": lambda c, s: ConvWorkload(c, s, 1), "dqmm": lambda c, s: DqmmWorkload(c, s),
             "attention": lambda c, s: AttentionWorkload(c, s), "yolo_b1": lambda c, s: YoloWorkload(c, s, 1),
             "yolo_b8": lambda c, s: YoloWorkload(c, s, 8), "yolo": lambda c, s: YoloWorkload(c, s, 64)}
ALIASES = {"conv": "conv_b16", "yolo_b64": "yolo"}
DEFAULT_WORKLOAD = "yolo"
CONFIG_ORDER = ["gemm", "conv_b1", "conv_b16", "dqmm", "attention", "yolo_b1", "yolo_b8"]
DEFAULT_STEPS = {"gemm": 1000, "conv_b16": 200, "conv_b1": 500, "dqmm": 1000, "attention": 300, "yolo_b1": 300,
                 "yolo_b8": 150, "yolo": 100}
CONFIG_STEPS = {"gemm": 200, "conv_b16": 40, "conv_b1": 200, "dqmm": 200, "attention": 100, "yolo_b1": 100,
                "yolo_b8": 50}
# The reference's own published CPU figures (4 threads, Ryzen 7 8845HS, .NET 10), shown beside the timed CPU baseline.
PUBLISHED = {
    "gemm": {"value": 0.3938, "unit": "TFLOP/s", "threads": 4,
             "what": "packed GEMM 1028x384x1536, 393.8 GFLOPS", "source": "bench.md:961-970"},
    "yolo": {"value": 1000.0 / 29.2, "unit": "images/s", "threads": 4,
             "what": "yolo11n 640x640 batch 1, 29.2 ms median", "source": "README.md:1743-1748"},
}


# ----------------------------------------------------------------- timing
def flush_l2(buf):
    """Evict L2 between steps: write the 512 MiB buffer (none of the step's data
    stays in the 126 MB L2), then read it, so that the lines L2 keeps are clean
    and the next step pays no write-back of the flush's own dirty lines."""
    buf.add_(1.0)
    buf.amax()


def _events(n):
    import torch

    return [torch.cuda.Event(enable_timing=True) for _ in range(n)], [torch.cuda.Event(enable_timing=True)
                                                                      for _ in range(n)]


def time_steps(step, K, flush, stream, sh: Shard) -> float:
    """Mean ms of K steps, each bracketed by CUDA events on `stream`, L2 flushed between steps."""
    import torch

    starts, stops = _events(K)
    sh.barrier()
    torch.cuda.synchronize()
    for i in range(K):
        starts[i].record(stream)
        step()
        stops[i].record(stream)
        flush_l2(flush)
    torch.cuda.synchronize()
    sh.barrier()
    return sum(s.elapsed_time(e) for s, e in zip(starts, stops)) / K


def measure(wl: Workload, ctx, sh: Shard, K: int, W: int, flush, stream, profile_steps: int, e2e_steps: int,
            tensor_e2e: bool = False) -> dict:
    """Device-resident step time, dominant-kernel time, launches, collective time and e2e of one workload
    (every rank calls this in the same order: the collectives inside line up)."""
    graph = ctx.capture(wl.compute) if wl.graphed and not isinstance(wl, YoloWorkload) else None
    compute = graph.launch if graph is not None else wl.compute
    profile_compute = getattr(wl, "profile_compute", wl.compute)

    def step():
        compute()
        wl.collect()

    for _ in range(W):
        step()
        flush_l2(flush)
    ctx.synchronize()
    launches0 = ctx.launch_count()
    step_ms = time_steps(step, K, flush, stream, sh)
    if graph is None and not isinstance(wl, YoloWorkload):
        launches = ctx.launch_count() - launches0
    else:  # graph replays: count one eager pass's launches
        l0 = ctx.launch_count()
        profile_compute()
        ctx.synchronize()
        launches = (ctx.launch_count() - l0) * K
    # the collective alone
    coll_ms = time_steps(wl.collect, max(5, K // 4), flush, stream, sh) if wl.collect_bytes() else 0.0
    # dominant kernel time from profiled eager passes
    ctx.profile_reset()
    ctx.profile(True)
    for _ in range(profile_steps):
        profile_compute()
        flush_l2(flush)
    ctx.synchronize()
    ctx.profile(False)
    kern_ms, kern_n = 0.0, 0
    for name in wl.main_kernel:
        ms_, n_ = ctx.profile_read(name)
        kern_ms, kern_n = kern_ms + ms_, kern_n + n_
    all_ms, _ = ctx.profile_read("")
    ctx.profile_reset()
    # e2e through the public API with pinned host buffers
    e2e_tensor_ms = None
    if isinstance(wl, YoloWorkload):
        e2e_ms = wl.e2e_pipelined(W, e2e_steps)
        e2e_mode = wl.e2e_mode
        if tensor_e2e:
            e2e_tensor_ms = wl.e2e_tensor(W, e2e_steps)
    else:
        import torch

        for _ in range(W):
            wl.e2e_step()
        ctx.synchronize()
        e2e_ms = time_steps(wl.e2e_step, e2e_steps, flush, stream, sh)
        e2e_mode = ("serial: H2D of this GPU's shard, compute, all-gather of the shards (N > 1), D2H of the whole "
                    "output on rank 0; L2 flushed between steps")
        torch.cuda.synchronize()
    if graph is not None:
        graph.close()
    return {"step_ms": step_ms, "kern_ms": kern_ms / max(1, kern_n), "kern_share": kern_ms / max(all_ms, 1e-12),
            "launches": launches, "coll_ms": coll_ms, "e2e_ms": e2e_ms, "e2e_mode": e2e_mode,
            "e2e_tensor_ms": e2e_tensor_ms}


def roofline(wl: Workload, kern_ms: float, peaks: dict, peaks_kind: str, traffic) -> dict:
    if kern_ms <= 0.0:  # the dominant kernel did not run in the profiled passes: no figure rather than a fake one
        return {"bound": wl.bound, "achieved": None, "peak": None, "frac": None, "traffic": traffic,
                "kernel": "+".join(wl.main_kernel), "kernel_ms": 0.0, "note": "main kernel not launched"}
    if wl.bound == "tensor":
        pkey = "bf16_tflops_sustained" if wl.long_step else "bf16_tflops"
        peak = peaks.get(pkey, FALLBACK_PEAKS[pkey]) / 2.0 / 3.0
        achieved = _tflops(wl.main_kernel_units() / (kern_ms * 1e-3))
        return {"bound": "tensor", "achieved": round(achieved, 2), "peak": round(peak, 2), "unit": "TFLOP/s",
                "frac": round(achieved / peak, 4), "traffic": traffic, "kernel": "+".join(wl.main_kernel),
                "kernel_ms": round(kern_ms, 5),
                "peak_basis": f"3xTF32 = {pkey}/2 (kind::tf32 rate) /3 products, {pkey} {peaks.get(pkey)} "
                              f"({peaks_kind}); frac of {peaks_kind}"}
    peak = peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"])
    achieved = wl.main_kernel_units() / (kern_ms * 1e-3) / 1e9
    return {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
            "frac": round(achieved / peak, 4), "traffic": traffic, "kernel": "+".join(wl.main_kernel),
            "kernel_ms": round(kern_ms, 5), "peak_basis": f"hbm_gbs ({peaks_kind}); frac of {peaks_kind}"}


def _rate(wl: Workload, units: float, ms: float) -> float:
    v = units / (ms * 1e-3)
    return _tflops(v) if wl.unit in ("TFLOP/s", "TOP/s") else v


def cpu_baseline(wl: Workload, budget_s: float) -> dict:
    cores = physical_cores()
    base = wl.cpu_sample(cores, budget_s)
    base.update(kind="port", cpu=cpu_model())
    try:
        base["value_4_threads"] = wl.cpu_sample(min(4, cores), budget_s / 2)["value"]
    except Exception:  # pragma: no cover
        pass
    pub = PUBLISHED.get(wl.key) or PUBLISHED.get(wl.key.split("_b")[0])
    if pub is not None:
        base["reference_published"] = pub
    return base


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
    sh = Shard(world, rank)

    from onnxsharp_b200.runtime import Context

    # a capturable (non-legacy) stream for the library, the events, the collectives and the L2 flush
    torch.cuda.set_stream(torch.cuda.Stream())
    ctx = Context(local)
    ctx.use_torch_stream()
    stream = torch.cuda.current_stream()
    flush = torch.empty(512 * 1024 * 1024 // 4, dtype=torch.float32, device="cuda")

    # --- headline
    head = WORKLOADS[args.workload](ctx, sh)
    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.3)
    m = measure(head, ctx, sh, args.steps, args.warmup, flush, stream, args.profile_steps, args.e2e_steps,
                tensor_e2e=isinstance(head, YoloWorkload))
    clocks = sampler.stop()
    weak_ms = None
    if world > 1 and isinstance(head, YoloWorkload) and not args.no_weak:
        # secondary: weak scaling, every GPU its own batch of 64 (no collective)
        solo = YoloWorkload(ctx, Shard(1, 0), head.batch)
        weak_ms = time_steps(solo.compute, max(10, args.steps // 2), flush, stream, sh)
        solo.close()
    head.close()

    # --- every other BASELINE config, same process
    sub = {}
    if not args.no_configs:
        for key in CONFIG_ORDER:
            if key == args.workload:
                continue
            wl = WORKLOADS[key](ctx, sh)
            K = CONFIG_STEPS[key]
            sub[key] = (wl, measure(wl, ctx, sh, K, args.warmup, flush, stream, max(3, args.profile_steps // 2),
                                    max(5, min(K, args.e2e_steps))), K)
            wl.close()

    # max over ranks of every timing, one collective
    vals = [m["step_ms"], m["e2e_ms"], m["coll_ms"], m["e2e_tensor_ms"] or 0.0, weak_ms or 0.0]
    for key in sub:
        r = sub[key][1]
        vals += [r["step_ms"], r["e2e_ms"], r["coll_ms"]]
    t = torch.tensor(vals, dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    vals = t.tolist()

    result = None
    if rank == 0:
        step_ms, e2e_ms, coll_ms, e2e_t_ms, weak_ms_max = vals[:5]
        units = head.units_per_step()
        bi, bo = head.e2e_bytes()
        par = (f"dp{world}: batch sharded over {world} GPUs, shard outputs all-gathered over NVLink (NCCL) inside "
               f"the timed step" if world > 1 and not head.replicas else
               (f"{world} replicas (batch smaller than the GPU count)" if head.replicas else "single GPU"))
        result = {
            "metric": METRIC, "value": round(_rate(head, units, step_ms), 3), "unit": head.unit, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(step_ms, 5), "higher_is_better": True,
            "scaling": "weak" if head.replicas else "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded numpy, same global batch on every N)",
            "config": dict(head.config, l2="flushed between steps (512 MiB write then read, outside the events)",
                           parallelism=par),
            "e2e": {"value": round(_rate(head, units, e2e_ms), 3), "unit": head.unit, "h2d_bytes_per_step": bi,
                    "d2h_bytes_per_step": bo, "ms_per_step": round(e2e_ms, 5), "steps": args.e2e_steps,
                    "mode": m["e2e_mode"]},
            "roofline": roofline(head, m["kern_ms"], peaks, peaks_kind, load_traffic(head.key)),
            "gpu_launches": int(m["launches"]),
            "clocks": clocks,
        }
        result["roofline"]["kernel_share"] = round(m["kern_share"], 4)
        if head.collect_bytes():
            cb = head.collect_bytes()
            result["collective"] = {"op": "ncclAllGather (torch.distributed.all_gather_into_tensor)",
                                    "bytes_received_per_gpu": cb, "ms_per_step": round(coll_ms, 5),
                                    "algbw_gbs_per_gpu": round(cb / (coll_ms * 1e-3) / 1e9, 1),
                                    "share_of_step": round(coll_ms / step_ms, 4)}
        if e2e_t_ms:
            result["e2e_tensor"] = {
                "value": round(_rate(head, units, e2e_t_ms), 3),
                "unit": head.unit, "ms_per_step": round(e2e_t_ms, 5),
                "h2d_bytes_per_step": head.net.inputs[0].numel() * 4 * world,
                "d2h_bytes_per_step": head.net.outputs[0].numel() * 4 * world,
                "mode": "pipelined yolo.HostPipeline: each GPU copies its images' FP32 [B/N,3,640,640] tensor in and "
                        "its FP32 [B/N,84,8400] output back (no gather)"}
        if weak_ms_max:
            result["weak"] = {"value": round(head.batch * world / (weak_ms_max * 1e-3), 3), "unit": head.unit,
                              "ms_per_step": round(weak_ms_max, 5), "images_per_gpu": head.batch,
                              "note": "secondary: every GPU its own batch, no collective"}
        if not args.no_cpu_baseline and world == 1:
            result["cpu_baseline"] = cpu_baseline(head, args.cpu_budget)
        if sub:
            cfgs = {}
            off = 5
            for key, (wl, r, K) in sub.items():
                s_ms, e_ms, c_ms = vals[off:off + 3]
                off += 3
                u = wl.units_per_step()
                bi, bo = wl.e2e_bytes()
                entry = {"workload": wl.name, "value": round(_rate(wl, u, s_ms), 3), "unit": wl.unit,
                         "ms_per_step": round(s_ms, 5), "steps": K,
                         "scaling": "weak" if wl.replicas else "strong",
                         "config": wl.config,
                         "roofline": roofline(wl, r["kern_ms"], peaks, peaks_kind, load_traffic(wl.key)),
                         "e2e": {"value": round(_rate(wl, u, e_ms), 3), "unit": wl.unit, "ms_per_step": round(e_ms, 5),
                                 "h2d_bytes_per_step": bi, "d2h_bytes_per_step": bo, "mode": r["e2e_mode"]},
                         "gpu_launches": int(r["launches"])}
                entry["roofline"]["kernel_share"] = round(r["kern_share"], 4)
                if wl.collect_bytes():
                    entry["collective"] = {"bytes_received_per_gpu": wl.collect_bytes(), "ms_per_step": round(c_ms, 5)}
                if not args.no_cpu_baseline and world == 1:
                    entry["cpu_baseline"] = cpu_baseline(wl, args.cpu_budget / 4)
                cfgs[key] = entry
            result["configs"] = cfgs
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    ctx.close()
    return result


def run_reference(args) -> dict | None:
    """Time the reference's CPU algorithm (the oracle port: the reference is C#) on the host cores."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return None
    cores = physical_cores()
    os.environ.setdefault("ONNXSHARP_THREADS", str(cores))
    wl = CPU_WORKLOADS[args.workload]()
    budget = min(2.0, 90.0 / max(1, args.steps + args.warmup))
    for _ in range(args.warmup):
        wl.cpu_sample(cores, 0.0)
    vals = []
    t0 = time.perf_counter()
    for _ in range(args.steps):
        vals.append(wl.cpu_sample(cores, budget))
    dt = time.perf_counter() - t0
    value = statistics.median(v["value"] for v in vals)
    return {
        "metric": METRIC, "impl": "reference", "value": round(value, 5), "unit": wl.unit, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt / args.steps * 1e3, 3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": wl.config,
        "cpu_baseline": {"value": round(value, 5), "unit": wl.unit, "cores": cores, "kind": "port",
                         "sample": vals[0]["sample"], "cpu": cpu_model(),
                         "reference_published": PUBLISHED.get(args.workload)},
        "e2e": {"value": round(value, 5), "unit": wl.unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "reference is C# (OnnxSharp); no .NET runtime on this box, so the CPU restatement of its kernels "
                "(oracle/) is timed with all physical cores",
    }


# ----------------------------------------------------------------- CPU baselines (the oracle port)
class CpuGemm:
    """Config 1 through the oracle's GEMM (the reference's per-element FMA chain, register-blocked panels)."""

    unit = "TFLOP/s"

    def __init__(self, a=None, b=None, bias=None):
        if a is None:
            rng = np.random.default_rng(1234)
            a = rng.uniform(-1, 1, (2048, 512)).astype(np.float32)
            b = rng.uniform(-1, 1, (512, 2048)).astype(np.float32)
            bias = rng.uniform(-1, 1, 2048).astype(np.float32)
        self.a, self.b, self.bias = a, b, bias
        self.config = {"workload": GemmWorkload.name, "m": 2048, "k": 512, "n": 2048, "bias": True}

    def cpu_sample(self, threads, budget_s=1.0):
        import oracle

        reps, dt = _timed(lambda: oracle.gemm(self.a, self.b, col_bias=self.bias, threads=threads), budget_s)
        flops = 2.0 * self.a.shape[0] * self.a.shape[1] * self.b.shape[1] * reps
        return {"value": _tflops(flops / dt), "unit": self.unit, "cores": threads,
                "sample": f"{reps} x full 2048x512x2048 GEMM+bias ({dt:.2f} s)"}


class CpuConv:
    """Config 2 images through the oracle's im2col-order conv + SiLU (one image per repetition)."""

    unit = "TFLOP/s"

    def __init__(self, x=None, w=None, b=None, batch: int = 16):
        if x is None:
            x, w, b = conv_inputs(4321, 1)
        self.x, self.w, self.b, self.batch = x, w, b, batch
        self.config = {"workload": f"conv3x3_silu_f32_b{batch}_64to128_160x160", "batch": batch,
                       "in": [batch, 64, 160, 160], "weight": [128, 64, 3, 3], "stride": 1, "pad": 1, "act": "SiLU"}

    def cpu_sample(self, threads, budget_s=1.0):
        import oracle

        i = [0]

        def one():
            j = i[0] % self.x.shape[0]
            oracle.conv2d(self.x[j:j + 1], self.w, self.b, pads=(1, 1, 1, 1), act=1, threads=threads)
            i[0] += 1

        reps, dt = _timed(one, budget_s)
        return {"value": _tflops(CONV_FLOPS_PER_IMAGE * reps / dt), "unit": self.unit, "cores": threads,
                "sample": f"{reps} image(s) of the batch of {self.batch} (3x3 conv 64->128 @160x160 + SiLU), "
                          f"{dt:.2f} s"}


class CpuDqmm:
    """The full config-3 DynamicQuantizeMatMul per repetition (F32-substitute GEMM, as the reference)."""

    unit = "TOP/s"

    def __init__(self, a=None, w=None, ws=None, b=None):
        if a is None:
            a, w, ws, b = dqmm_inputs(777)
        self.a, self.w, self.ws, self.b = a, w, ws, b
        self.config = {"workload": DqmmWorkload.name, "m": a.shape[0], "k": a.shape[1], "n": w.shape[1]}

    def cpu_sample(self, threads, budget_s=1.0):
        import oracle

        reps, dt = _timed(lambda: oracle.dqmm(self.a, self.w, 0, self.ws, self.b, threads=threads), budget_s)
        ops = 2.0 * self.a.shape[0] * self.a.shape[1] * self.w.shape[1] * reps
        return {"value": _tflops(ops / dt), "unit": self.unit, "cores": threads,
                "sample": f"{reps} x full {self.a.shape[0]}x{self.a.shape[1]}x{self.w.shape[1]} DQMM ({dt:.2f} s)"}


class CpuYolo:
    """Images through the oracle executor of the same plan (one image per repetition)."""

    unit = "images/s"

    def __init__(self, g=None, params=None, images=None, batch: int = 64):
        from onnxsharp_b200 import yolo

        if g is None:
            g = yolo.build_yolo11n()
            params = yolo.init_params(g, 2024)
            images = np.random.default_rng(9000).uniform(0, 1, (1, 3, 640, 640)).astype(np.float32)
        self.g, self.params, self.images, self.batch = g, params, images, batch
        self.config = {"workload": f"yolo11n_shaped_b{batch}_640", "global_batch": batch,
                       "input": [batch, 3, 640, 640], "output": [batch, 84, 8400]}

    def cpu_sample(self, threads, budget_s=1.0):
        from oracle import yolo_ref

        i = [0]

        def one():
            j = i[0] % self.images.shape[0]
            yolo_ref.run(self.g, self.params, self.images[j:j + 1], threads=threads)
            i[0] += 1

        reps, dt = _timed(one, budget_s)
        return {"value": reps / dt, "unit": self.unit, "cores": threads,
                "sample": f"{reps} image(s) of the batch of {self.batch} through the plan, {dt:.2f} s"}


class CpuAttention:
    """Sequences of config 4 through the oracle (projection GEMMs + ComputeBlocks), 8 per repetition."""

    unit = "TFLOP/s"

    def __init__(self, x=None, ws=None):
        if x is None:
            rng = np.random.default_rng(5150)
            x = rng.normal(0, 1, (64 * 128, 512)).astype(np.float32)
            lim = np.sqrt(6.0 / 1024)
            ws = [rng.uniform(-lim, lim, (512, 512)).astype(np.float32) for _ in range(4)]
        self.x, self.ws = x[:8 * 128], ws
        self.config = {"workload": AttentionWorkload.name, "x": [64, 128, 512], "heads": 8, "head_dim": 64}

    def cpu_sample(self, threads, budget_s=1.0):
        import oracle

        def one():
            q, k, v = (oracle.gemm(self.x, w, threads=threads).reshape(8, 128, 512) for w in self.ws[:3])
            o = oracle.attention(q, k, v, heads=8, scale=0.125, threads=threads)
            oracle.gemm(o.reshape(8 * 128, 512), self.ws[3], threads=threads)

        reps, dt = _timed(one, budget_s)
        return {"value": _tflops(ATTN_FLOPS / 8 * reps / dt), "unit": self.unit, "cores": threads,
                "sample": f"{reps} x 8 of the 64 sequences, {dt:.2f} s"}


CPU_WORKLOADS = {"gemm": CpuGemm, "conv_b16": CpuConv, "conv_b1": lambda: CpuConv(batch=1), "dqmm": CpuDqmm,
                 "yolo": CpuYolo, "yolo_b1": lambda: CpuYolo(batch=1), "yolo_b8": lambda: CpuYolo(batch=8),
                 "attention": CpuAttention}


def main() -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", default=DEFAULT_WORKLOAD, choices=sorted(set(WORKLOADS) | set(ALIASES)))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--e2e-steps", type=int, default=None)
    ap.add_argument("--profile-steps", type=int, default=None,
                    help="eager profiled passes for the dominant-kernel timing of graph-replayed workloads")
    ap.add_argument("--cpu-budget", type=float, default=12.0,
                    help="seconds of CPU-baseline sampling for the headline (a quarter of it per other config)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-configs", action="store_true", help="time only the headline workload")
    ap.add_argument("--no-weak", action="store_true", help="skip the secondary weak-scaling figure (N > 1)")
    args = ap.parse_args()
    args.workload = ALIASES.get(args.workload, args.workload)
    if args.profile_steps is None:
        args.profile_steps = 5 if args.workload.startswith("yolo") else 30
    if args.e2e_steps is None:
        args.e2e_steps = 30 if args.workload.startswith("yolo") else 100
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
