"""Run under torchrun with 2 GPUs by tests/test_multigpu_gpu.py (not collected
by pytest itself): the torch.distributed path bench.py uses.

Each rank runs the YOLO plan on its half of a batch of 4 and the ranks
all-gather the [2, 84, 8400] outputs (NCCL); rank 0 checks the gathered
tensor against the single-GPU plan over the whole batch within the plan's
parity tolerance (a half batch may split a conv's K differently, so FP32 sums
round differently). Then the serving pipeline (frames in, detections out)
runs sharded with its packed detections all-gathered, and rank 0 checks every
image's detections against the unsharded pipeline: the same count and
classes, scores and boxes within 1e-4. Exits non-zero on any mismatch."""
from __future__ import annotations

import os
import sys
from datetime import timedelta
from pathlib import Path

import numpy as np

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))


def main() -> int:
    import torch
    import torch.distributed as dist

    from onnxsharp_b200 import yolo
    from onnxsharp_b200.runtime import Context
    from onnxsharp_b200.serve import DetectPipeline

    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    torch.cuda.set_stream(torch.cuda.Stream())
    ctx = Context(local)
    ctx.use_torch_stream()
    g = yolo.build_yolo11n()
    params = yolo.init_params(g, 43)
    B, per = 4, 4 // world
    images = np.random.default_rng(43).uniform(0, 1, (B, 3, 640, 640)).astype(np.float32)
    net = yolo.Net(ctx, g, params, per)
    net.input_view().copy_(torch.from_numpy(images[rank * per:(rank + 1) * per]))
    out = net.forward(use_graph=True)
    full = torch.empty((B, 84, 8400), device="cuda")
    dist.all_gather_into_tensor(full, out)
    ok = True
    solo = None
    if rank == 0:
        solo = yolo.Net(ctx, g, params, B)
        solo.input_view().copy_(torch.from_numpy(images))
        want = solo.forward(use_graph=True).cpu().numpy()
        got = full.cpu().numpy()
        box_err = float(np.max(np.abs(got[:, :4] - want[:, :4]) / np.maximum(1.0, np.abs(want[:, :4]))))
        cls_err = float(np.max(np.abs(got[:, 4:] - want[:, 4:])))
        if box_err > 1e-4 or cls_err > 1e-4:
            print(f"gathered plan output differs from the single-GPU plan: boxes {box_err}, scores {cls_err}",
                  flush=True)
            ok = False
    # serving pipeline, sharded, detections gathered to rank 0
    hw = (360, 640)
    frames = np.random.default_rng(44).integers(0, 256, (B,) + hw + (3,), dtype=np.uint8)
    pipe = DetectPipeline(net, frame_hw=hw, gather=True)
    f, r = pipe.host_buffers()
    f.copy_(torch.from_numpy(frames[rank * per:(rank + 1) * per]))
    pipe.submit(f, r if rank == 0 else None)
    pipe.synchronize()
    if rank == 0:
        got = pipe.unpack(r.numpy())
        ref_pipe = DetectPipeline(solo, frame_hw=hw)
        f2, r2 = ref_pipe.host_buffers()
        f2.copy_(torch.from_numpy(frames))
        ref_pipe.submit(f2, r2)
        ref_pipe.synchronize()
        want = ref_pipe.unpack(r2.numpy())
        def same(a, b):  # class ids exact, scores and boxes within the parity tolerance
            return (a.shape == b.shape and np.array_equal(a[:, 0], b[:, 0])
                    and bool(np.all(np.abs(a[:, 1:] - b[:, 1:]) <= 1e-4 * np.maximum(1.0, np.abs(b[:, 1:])))))

        if len(got) != B or not all(same(a, b) for a, b in zip(got, want)):
            print("gathered detections differ from the single-GPU pipeline", flush=True)
            ok = False
        if sum(a.shape[0] for a in got) == 0:
            print("no detections at all", flush=True)
            ok = False
        solo.close()
    dist.barrier()
    net.close()
    dist.destroy_process_group()
    if rank == 0 and ok:
        print("dist shard check ok", flush=True)
    return 0 if ok else 1


if __name__ == "__main__":
    sys.exit(main())
