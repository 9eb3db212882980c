"""Batch-level sharding over the GPUs of one node (needs at least 2 GPUs; the
tests skip on a single-GPU box).

1. The C ABI group (osc_group_*, one process, NCCL clique): row-sharded
   DynamicQuantizeMatMul whose per-tensor range crosses the GPUs through
   osc_group_allreduce_minmax gives q, the int32 accumulators and y
   bit-identical to the oracle on the whole tensor, and the all-gathered y is
   the same on every GPU.
2. osc_group_run_sharded: the YOLO plan captured per GPU on its half of the
   batch, replayed and all-gathered, equals the single-GPU plan over the whole
   batch within the plan's parity tolerance (a half batch may split a conv's
   K differently, so its FP32 sums round differently), and the gathered
   tensor is the same on every GPU bit for bit.
3. The torch.distributed path bench.py uses (one process per GPU, NCCL
   all_gather_into_tensor; the serving pipeline's gathered detections),
   checked by tests/dist_shard_check.py under torchrun."""
from __future__ import annotations

import os
import socket
import subprocess
import sys

import numpy as np
import pytest

import oracle
from conftest import ROOT, rel_err

pytestmark = pytest.mark.gpu


def _two_gpus():
    import torch

    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")


@pytest.fixture(scope="module")
def group():
    _two_gpus()
    from onnxsharp_b200.runtime import Group

    g = Group([0, 1])
    yield g
    g.close()


def test_group_shape(group):
    import ctypes as C

    from onnxsharp_b200 import _lib

    n = C.c_int()
    assert _lib.load().osc_group_size(group.handle, C.byref(n)) == 0 and n.value == 2
    assert [c.device for c in group.ctxs] == [0, 1]


def test_group_dqmm_row_shards_bit_exact(group):
    import torch

    from onnxsharp_b200.runtime import DqmmWeights, dqmm, minmax

    rng = np.random.default_rng(41)
    m, k, n = 1024, 512, 768
    a = rng.normal(0, 1, (m, k)).astype(np.float32)
    a[700, 3] = 9.5  # the global maximum lives in the second shard only
    w = rng.integers(-127, 128, (k, n)).astype(np.int8)
    ws = rng.uniform(0.001, 0.02, n).astype(np.float32)
    b = rng.normal(0, 0.01, n).astype(np.float32)
    ry, rq, racc, (rs, rz) = oracle.dqmm(a, w, 0, ws, b)
    half = m // 2
    per = []
    for r, ctx in enumerate(group.ctxs):
        dev = torch.device("cuda", r)
        W = DqmmWeights(ctx, torch.from_numpy(w).to(dev), k, n, 0)
        t = dict(a=torch.from_numpy(a[r * half:(r + 1) * half]).to(dev), W=W, ws=torch.from_numpy(ws).to(dev),
                 b=torch.from_numpy(b).to(dev), mm=torch.zeros(2, device=dev),
                 q=torch.empty((half, k), dtype=torch.uint8, device=dev),
                 acc=torch.empty((half, n), dtype=torch.int32, device=dev),
                 y=torch.empty((half, n), device=dev), yall=torch.empty((m, n), device=dev),
                 params=torch.empty(2, device=dev))
        torch.cuda.synchronize(dev)
        minmax(ctx, t["a"], out=t["mm"])
        per.append(t)
    group.allreduce_minmax([t["mm"] for t in per])
    for r, (ctx, t) in enumerate(zip(group.ctxs, per)):
        dqmm(ctx, t["a"], t["W"], t["ws"], t["b"], out=t["y"], minmax_override=t["mm"], q_out=t["q"],
             acc_out=t["acc"], params_out=t["params"], row0=r * half, rows_total=m)
    group.all_gather([t["y"] for t in per], [t["yall"] for t in per], half * n * 4)
    group.synchronize()
    for r, t in enumerate(per):
        rows = slice(r * half, (r + 1) * half)
        p = t["params"].cpu().numpy()
        assert p[0] == np.float32(rs) and int(p[1]) == rz, r
        assert np.array_equal(t["q"].cpu().numpy(), rq[rows]), r
        assert np.array_equal(t["acc"].cpu().numpy(), racc[rows]), r
        assert np.array_equal(t["yall"].cpu().numpy().view(np.uint32), ry.view(np.uint32)), r


def test_group_run_sharded_yolo_matches_single_gpu(group):
    import torch

    from onnxsharp_b200 import yolo
    from onnxsharp_b200.runtime import Context

    g = yolo.build_yolo11n()
    params = yolo.init_params(g, 42)
    images = np.random.default_rng(42).uniform(0, 1, (4, 3, 640, 640)).astype(np.float32)
    # single GPU, whole batch
    solo_ctx = Context(0)
    solo = yolo.Net(solo_ctx, g, params, 4)
    solo.input_view().copy_(torch.from_numpy(images))
    want = solo.forward(use_graph=True).cpu().numpy()
    solo.close()
    solo_ctx.close()
    # two GPUs, two images each, plans replayed and gathered by the group
    nets, graphs, gathered = [], [], []
    for r, ctx in enumerate(group.ctxs):
        net = yolo.Net(ctx, g, params, 2)
        net.input_view().copy_(torch.from_numpy(images[2 * r:2 * r + 2]))
        net.forward(use_graph=True)  # captures the slot's graph
        nets.append(net)
        graphs.append(net.graphs[0])
        gathered.append(torch.full((4, 84, 8400), float("nan"), device=torch.device("cuda", r)))
    for r in range(2):
        torch.cuda.synchronize(r)
    group.run_sharded(graphs, [n.outputs[0] for n in nets], gathered, 2 * 84 * 8400 * 4)
    group.synchronize()
    got0 = gathered[0].cpu().numpy()
    assert rel_err(got0[:, :4], want[:, :4]) <= 1e-4  # boxes
    assert np.max(np.abs(got0[:, 4:] - want[:, 4:])) <= 1e-4  # class scores
    assert np.array_equal(gathered[1].cpu().numpy().view(np.uint32), got0.view(np.uint32))
    for n in nets:
        n.close()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_torch_distributed_sharding_matches_single_gpu():
    _two_gpus()
    env = dict(os.environ, PYTHONPATH=str(ROOT), NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", f"--master-port={_free_port()}",
           str(ROOT / "tests" / "dist_shard_check.py")]
    r = subprocess.run(cmd, capture_output=True, text=True, env=env, cwd=ROOT, timeout=700)
    assert r.returncode == 0, (r.stdout[-3000:], r.stderr[-3000:])
    assert "dist shard check ok" in r.stdout
