"""Camera-sharded DFA over several GPUs (optional mode).

The reference splits the 6 cameras over a 1x2 Tenstorrent mesh, softmaxes the weights over
each device's own 3 cameras and all-reduces the partial sums
(``model/sparse4d_head.py:92-93,326-330``, ``model/deformable_feature_aggregation.py:925-931``),
which gives every group a total weight of 2 instead of 1.  Here every rank computes the FULL
logits and the softmax over all cameras (cheap and replicated), samples only its own
cameras, and the fp32 partial sums are combined with one NCCL collective -- the result is the
single-GPU result up to summation order.

With 6 cameras and 8 GPUs the split is 2-D: ``frame_groups x camera_groups`` ranks (e.g.
4 x 2), frames sharded over the first axis, cameras over the second; ``make_groups`` builds
the camera sub-communicators.

Two ways to combine the partial sums (``DeformableFeatureAggregation``'s
``model_config["CAMERA_REDUCE"]``):

* ``"all_reduce"`` -- every rank of the camera group ends with all ``bs * A`` rows (the
  reference's ``ttnn.all_reduce``);
* ``"reduce_scatter"`` -- NCCL reduce-scatter over the flattened ``(frame, anchor)`` rows: rank
  ``r`` of a group of ``n`` ends with rows ``[r * bs * A / n, (r + 1) * bs * A / n)`` (whole
  frames when ``n`` divides ``bs``), half the bytes of the all-reduce on the wire, and runs
  ``output_proj`` on its shard only (``shard_rows``).
"""
from __future__ import annotations

from typing import List, Optional, Tuple

import torch
import torch.distributed as dist


def camera_split(num_cams: int, parts: int) -> List[Tuple[int, int]]:
    """Contiguous camera ranges, sizes differing by at most one."""
    if parts <= 0:
        raise ValueError("parts must be positive")
    base, extra = divmod(num_cams, parts)
    out, start = [], 0
    for r in range(parts):
        n = base + (1 if r < extra else 0)
        out.append((start, start + n))
        start += n
    return out


def rank_camera_range(num_cams: int, group: Optional[dist.ProcessGroup] = None) -> Tuple[int, int]:
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    return camera_split(num_cams, world)[rank]


def make_groups(world_size: int, camera_groups: int):
    """Ranks ``0..world_size-1`` as a ``(world_size // camera_groups) x camera_groups`` grid.

    Returns ``(frame_group_index, camera_group)`` for the calling rank, where
    ``camera_group`` is the sub-communicator of the ranks that share its frames.  Every rank
    must call this (``new_group`` is collective)."""
    if world_size % camera_groups:
        raise ValueError("world_size must be a multiple of camera_groups")
    rank = dist.get_rank()
    mine = None
    for f in range(world_size // camera_groups):
        ranks = list(range(f * camera_groups, (f + 1) * camera_groups))
        g = dist.new_group(ranks)
        if rank in ranks:
            mine = (f, g)
    return mine


def shard_rows(rows: int, group: Optional[dist.ProcessGroup] = None) -> Tuple[int, int]:
    """``[begin, end)`` of the flattened ``(frame, anchor)`` rows this rank holds after a
    row reduce-scatter over ``group`` (``rows`` must divide by the group size)."""
    n = dist.get_world_size(group)
    if rows % n:
        raise ValueError(f"reduce-scatter needs bs * num_anchor ({rows}) divisible by the camera group size ({n})")
    r = dist.get_rank(group)
    return r * (rows // n), (r + 1) * (rows // n)


def reduce_partial_sums(partial: torch.Tensor, group: Optional[dist.ProcessGroup] = None,
                        scatter: bool = False) -> torch.Tensor:
    """Combine per-camera-shard partial sums, ``[bs, A, C]`` or flattened rows ``[R, C]``.

    ``scatter=False``: all-reduce in place, every rank gets the full tensor.
    ``scatter=True`` on ``[R, C]``: reduce-scatter over the rows, rank r gets rows
    ``shard_rows(R, group)`` as ``[R/n, C]`` (no copy before the collective).
    ``scatter=True`` on ``[bs, A, C]``: reduce-scatter over anchors within every frame, rank r
    gets anchors ``[r*A/n, (r+1)*A/n)`` of each frame as ``[bs, A/n, C]`` (A must divide by the
    group size; the per-frame chunks are gathered into one buffer first)."""
    if not scatter:
        dist.all_reduce(partial, group=group)
        return partial
    n = dist.get_world_size(group)
    if partial.dim() == 2:
        rows, C = partial.shape
        b, e = shard_rows(rows, group)
        out = torch.empty(e - b, C, dtype=partial.dtype, device=partial.device)
        dist.reduce_scatter_tensor(out, partial.contiguous(), group=group)
        return out
    bs, A, C = partial.shape
    if A % n:
        raise ValueError("reduce-scatter needs num_anchor divisible by the camera group size")
    chunks = partial.reshape(bs, n, A // n, C).transpose(0, 1).contiguous()  # [n, bs, A/n, C]
    out = torch.empty(bs, A // n, C, dtype=partial.dtype, device=partial.device)
    dist.reduce_scatter_tensor(out, chunks.reshape(n * bs, A // n, C), group=group)
    return out
