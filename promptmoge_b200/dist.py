"""Multi-GPU frame sharding for batched refinement (benchmark configuration 4: many independent frames over 1-8 GPUs).

Frames are independent units (the reference batches them column-wise with per-frame z offsets, moge/model/v3.py:333,
and fits them row by row, prompt_stem.py:211-240), so each rank refines a contiguous range of frames with its own
captured graph and no data-path collective.  The only exchange is one all-gather of the per-frame fit states at the
end (72 bytes per frame), so every rank can report every frame's (s, t).  One process per GPU, launched by torchrun;
NCCL over NVLink on GPUs, gloo on the CPU (tests).
"""
from __future__ import annotations

import numpy as np
import torch
import torch.distributed as dist


def frame_range(n_frames: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous [begin, end) share of n_frames for rank: sizes differ by at most one, lower ranks take the extra."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    base, extra = divmod(n_frames, world)
    begin = rank * base + min(rank, extra)
    return begin, begin + base + (1 if rank < extra else 0)


def gather_frame_states(local: torch.Tensor, n_frames: int, group=None) -> torch.Tensor:
    """All-gather the per-frame fit states ([n_local, 18] int32, pmg_fit_state words) of every rank's frame range into
    [n_frames, 18] in frame order.  Ranges may differ by one frame: each rank pads to the largest share."""
    world = dist.get_world_size(group)
    share = max(e - b for b, e in (frame_range(n_frames, r, world) for r in range(world)))
    padded = torch.zeros((share, local.shape[1]), dtype=local.dtype, device=local.device)
    padded[: local.shape[0]] = local
    if dist.get_backend(group) == "nccl":
        out = torch.empty((world * share, local.shape[1]), dtype=local.dtype, device=local.device)
        dist.all_gather_into_tensor(out, padded, group=group)
        parts = list(out.split(share))
    else:
        parts = [torch.empty_like(padded) for _ in range(world)]
        dist.all_gather(parts, padded, group=group)
    rows = []
    for r, p in enumerate(parts):
        b, e = frame_range(n_frames, r, world)
        rows.append(p[: e - b])
    return torch.cat(rows)


class ShardedRefiner:
    """Refines this rank's share of a frame set, `batch` frames per graph replay, and gathers every frame's fit.

    frames(i) must return frame i's host inputs (point_coord [1,H,W,3], lidar_depth [1,1,h,w], lidar_conf [1,1,h,w],
    encoder_feature [1,1024,h',w'] fp16, uv_bias [1,C,h',w'] or None)."""

    def __init__(self, refiner, n_frames: int, group=None):
        self.refiner = refiner
        self.n_frames = n_frames
        self.group = group
        world = dist.get_world_size(group) if dist.is_initialized() else 1
        rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.begin, self.end = frame_range(n_frames, rank, world)

    def run(self, frames, K: int = 1, batch_frames=None, out: torch.Tensor | None = None):
        """Returns (refined point maps of this rank's frames [n_local,H,W,3] host, all frames' fit states
        [n_frames, 18] int32 on this rank's device).  batch_frames(ids), when given, returns the five inputs of a
        whole batch of frames at once (already concatenated, e.g. pinned host tensors), instead of frames(i) per
        frame.  out: a host tensor [n_local,H,W,3] (pinned: the refined maps are copied into it directly)."""
        B = self.refiner.geo.batch
        outs, fits = [], []
        for f0 in range(self.begin, self.end, B):
            ids = [min(f, self.end - 1) for f in range(f0, f0 + B)]      # the last batch repeats its final frame
            if batch_frames is not None:
                cat = list(batch_frames(ids))
            else:
                parts = [frames(i) for i in ids]
                cat = [np.concatenate([p[k] for p in parts]) if parts[0][k] is not None else None for k in range(5)]
            n = min(B, self.end - f0)
            whole = out is not None and n == B
            dst = out[f0 - self.begin:f0 - self.begin + B] if whole else None
            # with a whole batch copied straight into `out`, nothing on the host waits for the batch: the next
            # batch's copies and graph queue up behind it (the plan's buffers are stream-ordered)
            pc, _ = self.refiner.refine(*cat[:4], uv_bias=cat[4], K=K, out=dst, sync=not whole)
            if out is not None and not whole:
                out[f0 - self.begin:f0 - self.begin + n] = pc[:n]
            elif out is None:
                outs.append(pc[:n].clone())
            fits.append(self.refiner.engine._fit[:n].clone())          # device copy, stream-ordered
        torch.cuda.current_stream(self.refiner.device).synchronize()
        if out is not None:
            local_pc = out
        else:
            local_pc = torch.cat(outs) if outs else torch.empty(0)
        local_fit = torch.cat(fits).cpu() if fits else torch.empty((0, 18), dtype=torch.int32)
        if dist.is_initialized() and dist.get_world_size(self.group) > 1:
            dev = self.refiner.device if dist.get_backend(self.group) == "nccl" else torch.device("cpu")
            all_fit = gather_frame_states(local_fit.to(dev), self.n_frames, self.group)
        else:
            all_fit = local_fit
        return local_pc, all_fit
