"""Frames in, detections out: the serving loop of the reference's
YoloDetector.Detect (src/OnnxSharp/Vision/YoloDetector.cs:117 — Letterbox,
Net.Forward, YoloDecoder.Decode + DetectionNms) on the device, optionally
sharded by image across the GPUs of one node.

Per submitted batch (one input slot of the plan, `depth` slots round robin):
  1. H2D of the batch's u8 frames from pinned host memory (copy stream);
  2. one CUDA graph on the plan's stream: batched letterbox into the plan's
     input and the forward pass into the slot's output;
  3. one CUDA graph on the tail stream (its own library context, so its
     scratch is its own): the detect tail (argmax, score sort, greedy NMS,
     mapping back to source pixels) into a packed detections buffer;
  4. with a process group of N ranks: an NCCL all-gather of the packed
     detections over NVLink (tail stream), so rank 0 holds the whole global
     batch's result (the single-Net contract: one Forward returns the whole
     batch);
  5. D2H of the (gathered) detections on rank 0 (copy stream).
Consecutive batches overlap: batch i's H2D, batch i-1's forward pass, batch
i-2's detect tail (whose CTAs are one per image, so the SMs it leaves idle run
the next forward pass) and D2H run at the same time. A slot is reused only
after the work that read it finished: its frames (the forward pass), its
output (the detect tail) and its detections (the copy) -- event waits.

Packed detections per image: max_det x 6 floats (class, score, x, y, w, h),
then per batch B int32 counts, so one collective moves both.
"""
from __future__ import annotations

import numpy as np

from . import ops
from .runtime import Context


def letterbox_transforms(batch: int, src_w: int, src_h: int, placement) -> np.ndarray:
    """[B][6] = {resized_w, resized_h, offset_x, offset_y, source_w, source_h} (osc_yolo_detect_f32)."""
    rw, rh, ox, oy = placement
    return np.tile(np.array([rw, rh, ox, oy, src_w, src_h], np.float32), (batch, 1))


class DetectPipeline:
    """See the module docstring. With gather=True the ranks of `group` (None:
    the default process group) each serve their own images and the packed
    detections are all-gathered, so rank 0 receives the whole global batch."""

    def __init__(self, net, frame_hw=(720, 1280), bgr: bool = True, depth: int = 2, conf: float = 0.25,
                 iou: float = 0.45, max_det: int = 300, gather: bool = False, group=None):
        import torch
        import torch.distributed as dist

        if depth < 1:
            raise ValueError("depth must be >= 1")
        self.net, self.depth, self.n = net, depth, 0
        self.max_det, self.conf, self.iou, self.bgr = max_det, conf, iou, bgr
        self.group = group
        self.world = dist.get_world_size(group) if gather else 1
        self.rank = dist.get_rank(group) if gather else 0
        B = net.batch
        h, w = frame_hw
        dev = torch.device("cuda", net.ctx.device)
        net.add_slots(depth)
        self.frames = [torch.zeros((B, h, w, 3), dtype=torch.uint8, device=dev) for _ in range(depth)]
        self.pack_len = B * max_det * 6 + B
        self.pack = [torch.zeros(self.pack_len, dtype=torch.float32, device=dev) for _ in range(depth)]
        self.gathered = [torch.zeros(self.world * self.pack_len, dtype=torch.float32, device=dev)
                         for _ in range(depth)] if self.world > 1 else self.pack
        # the placement is the same for every frame of a size; the detect tail maps boxes back with it
        probe = torch.zeros((1, 3, net.size, net.size), device=dev)
        pl = ops.letterbox_batch(net.ctx, self.frames[0][:1], probe, bgr=bgr)
        self.transforms = torch.from_numpy(letterbox_transforms(B, w, h, pl)).to(dev)
        self.placement = pl
        self.graphs = []
        self.tail = torch.cuda.Stream(device=dev)
        self.tail_ctx = Context(net.ctx.device)
        self.tail_ctx.set_stream(self.tail.cuda_stream)
        self.tail_graphs = []
        for s in range(depth):
            dets = self.pack[s][: B * max_det * 6].view(B, max_det, 6)
            counts = self.pack[s][B * max_det * 6:].view(torch.int32)

            def before(s=s):
                ops.letterbox_batch(net.ctx, self.frames[s], net.inputs[s], bgr=bgr)

            def tail(s=s, dets=dets, counts=counts):
                ops.yolo_detect_into(self.tail_ctx, net.outputs[s], dets, counts, conf=conf, iou=iou,
                                     transforms=self.transforms)

            self.graphs.append(net.capture_slot(s, before))
            torch.cuda.synchronize(dev)
            self.tail_graphs.append(self.tail_ctx.capture(tail))
        self.h2d = torch.cuda.Stream(device=dev)
        self.d2h = torch.cuda.Stream(device=dev)
        self.ev_h2d = [torch.cuda.Event() for _ in range(depth)]
        self.ev_fwd = [torch.cuda.Event() for _ in range(depth)]
        self.ev_plan = [torch.cuda.Event() for _ in range(depth)]  # the slot's detect tail (and gather) done
        self.ev_d2h = [torch.cuda.Event() for _ in range(depth)]
        torch.cuda.synchronize(dev)

    def close(self):
        """Free the tail graphs and context (the forward graphs belong to the Net)."""
        self.synchronize()
        for g in self.tail_graphs:
            g.close()
        self.tail_graphs = []
        self.tail_ctx.close()

    def host_buffers(self):
        """(pinned frames [B, H, W, 3] u8, pinned result [world * pack_len] f32) for submit()."""
        import torch

        f = torch.empty(self.frames[0].shape, dtype=torch.uint8).pin_memory()
        r = torch.empty(self.world * self.pack_len, dtype=torch.float32).pin_memory()
        return f, r

    def submit(self, host_frames, host_result=None):
        """Queue one batch. host_frames (pinned u8 [B, H, W, 3]) and host_result (pinned; None on
        the ranks other than 0 when gathering) must stay untouched until the returned event completes."""
        import torch
        import torch.distributed as dist

        net, s, reuse = self.net, self.n % self.depth, self.n >= self.depth
        plan = net.plan_stream()
        with torch.cuda.stream(self.h2d):
            if reuse:
                self.h2d.wait_event(self.ev_fwd[s])  # the letterbox that read these frames is done
            self.frames[s].copy_(host_frames, non_blocking=True)
            self.ev_h2d[s].record(self.h2d)
        plan.wait_event(self.ev_h2d[s])
        if reuse:
            plan.wait_event(self.ev_plan[s])  # the detect tail that read this slot's output is done
        net.launch_graph(self.graphs[s])
        self.ev_fwd[s].record(plan)
        self.tail.wait_event(self.ev_fwd[s])
        if reuse:
            self.tail.wait_event(self.ev_d2h[s])  # the copy that read this slot's detections is done
        self.tail_graphs[s].launch()
        if self.world > 1:
            with torch.cuda.stream(self.tail):
                dist.all_gather_into_tensor(self.gathered[s], self.pack[s], group=self.group)
        self.ev_plan[s].record(self.tail)
        with torch.cuda.stream(self.d2h):
            self.d2h.wait_event(self.ev_plan[s])
            if host_result is not None:
                host_result.copy_(self.gathered[s], non_blocking=True)
            self.ev_d2h[s].record(self.d2h)
        self.n += 1
        return self.ev_d2h[s]

    def unpack(self, result) -> list[np.ndarray]:
        """Per-image detections [(count, 6) arrays] of a host result buffer, ranks in order."""
        B, md = self.net.batch, self.max_det
        r = np.asarray(result).reshape(self.world, self.pack_len)
        out = []
        for k in range(self.world):
            dets = r[k, : B * md * 6].reshape(B, md, 6)
            counts = r[k, B * md * 6:].view(np.int32)
            out += [dets[i, : counts[i]] for i in range(B)]
        return out

    def synchronize(self):
        self.d2h.synchronize()
        self.tail.synchronize()
        self.net.plan_stream().synchronize()

    def bytes_per_step(self) -> tuple[int, int]:
        """(H2D bytes, D2H bytes) of one submitted batch on this rank."""
        return self.frames[0].numel(), (self.world * self.pack_len * 4 if self.rank == 0 else 0)
