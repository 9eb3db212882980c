"""The N > 1 host logic on CPU with world_size-2 gloo process groups: shard
ranges, the DQMM range exchange (sharded quantisation with the all-reduced
range reproduces the whole tensor's q / int32 accumulators / outputs bit for
bit) and the max-over-ranks timing reduction. A rank that fails raises in its
child process and the test reports it (no GPU involved)."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from onnxsharp_b200.shard import shard_range


def test_shard_range_covers_exactly():
    for n in (0, 1, 7, 4096):
        for world in (1, 2, 3, 8):
            spans = [shard_range(n, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            assert max(e - s for s, e in spans) - min(e - s for s, e in spans) <= 1
    with pytest.raises(ValueError):
        shard_range(10, 2, 2)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, a, w, ws, b, results):
    import sys

    import torch
    import torch.distributed as dist

    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import oracle
    from onnxsharp_b200.shard import global_minmax, max_over_ranks, shard_range

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        s, e = shard_range(a.shape[0], world, rank)
        shard = a[s:e]
        mm = torch.tensor(oracle.minmax(shard), dtype=torch.float32)
        global_minmax(mm)
        scale, zp = oracle.dql_params(float(mm[0]), float(mm[1]))
        q = oracle.quantize_u8(shard, scale, zp)
        acc = oracle.matmul_integer(q, zp, w, 0)
        t = torch.tensor([float(rank + 1)], dtype=torch.float64)
        max_over_ranks(t)
        results[rank] = (s, e, scale, zp, q, acc, float(t[0]))
    finally:
        dist.destroy_process_group()


def test_dqmm_range_exchange_two_ranks():
    rng = np.random.default_rng(17)
    a = rng.normal(0, 1, (64, 48)).astype(np.float32)
    a[50, 3] = 9.0  # the global max lives in rank 1's shard only
    w = rng.integers(-127, 128, (48, 16)).astype(np.int8)
    ws = rng.uniform(0.001, 0.02, 16).astype(np.float32)
    b = rng.normal(0, 0.01, 16).astype(np.float32)
    import oracle

    y, q_ref, acc_ref, (s_ref, z_ref) = oracle.dqmm(a, w, 0, ws, b)
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    results = mgr.dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, a, w, ws, b, results)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0, "a rank failed"
    got = [results[r] for r in range(2)]
    assert all(g[2] == np.float32(s_ref) and g[3] == z_ref for g in got)
    assert np.array_equal(np.concatenate([g[4] for g in got]), q_ref)
    assert np.array_equal(np.concatenate([g[5] for g in got]), acc_ref)
    assert all(g[6] == 2.0 for g in got)  # max over ranks
