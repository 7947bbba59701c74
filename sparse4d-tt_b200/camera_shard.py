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
  ``output_proj`` on its shard only (``shard_rows``);
* ``"p2p"`` (groups of 2 GPUs, tensor-core linears) -- the same row shards without a collective
  kernel: each rank's gather writes its partial sums into a buffer the other rank has mapped
  (``PeerPartialSums``, CUDA IPC), a bounded flag exchange over NVLink orders the two GPUs, and
  ``output_proj`` reads its rows of both partial sums -- the peer's over NVLink -- and adds them
  in the tensor-core accumulator (``s4d_dfa_output_proj_sum``).
"""
from __future__ import annotations

import ctypes
from typing import Dict, List, Optional, Tuple

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


def _export(t: torch.Tensor) -> Tuple[bytes, int]:
    """(IPC handle, byte offset) of a device tensor's memory (s4d_ipc_export)."""
    from . import _lib as L

    lib = L.lib()
    handle = ctypes.create_string_buffer(lib.s4d_ipc_handle_bytes())
    offset = ctypes.c_uint64(0)
    L.check("ipc_export", lib.s4d_ipc_export(t.data_ptr(), handle, ctypes.byref(offset)))
    return handle.raw, int(offset.value)


class PeerPartialSums:
    """Partial-sum buffers of a 2-rank camera group, shared over CUDA IPC (``CAMERA_REDUCE="p2p"``).

    Each rank owns two ``[capacity, C]`` fp32 buffers -- alternate calls use alternate buffers,
    so a rank's next gather never overwrites what the other rank may still be reading -- and a
    slot array in which the other rank publishes its epoch.  Per call: the gather writes
    ``current()``; ``exchange()`` launches the bounded flag exchange on the current stream and
    returns the device address of the other rank's buffer of the same call, for
    ``ops.output_proj_sum_into``.  Construction and ``close()`` are collective over the group;
    the two ranks must be on different GPUs (their waits must run at the same time).  A wait
    that gives up after ``limit_ns`` sets ``S4D_FLAG_PEER_TIMEOUT`` in ``error_flag``
    (``check()`` reads it)."""

    def __init__(self, capacity: int, channels: int, group: dist.ProcessGroup, device: torch.device,
                 limit_ns: int = 2_000_000_000) -> None:
        from . import _lib as L

        if dist.get_world_size(group) != 2:
            raise ValueError("CAMERA_REDUCE='p2p' needs camera groups of exactly 2 ranks")
        self.group, self.device = group, torch.device(device)
        self.rank = dist.get_rank(group)
        self.peer = 1 - self.rank
        self.capacity, self.channels = int(capacity), int(channels)
        self.limit_ns = int(limit_ns)
        self.bufs = [torch.empty(self.capacity, channels, dtype=torch.float32, device=self.device) for _ in range(2)]
        self.slots = torch.zeros(8, dtype=torch.int32, device=self.device)
        self.error_flag = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.epoch = 0
        torch.cuda.synchronize(self.device)  # the zeroed slots are in place before the peer can write them
        uuid = str(torch.cuda.get_device_properties(self.device).uuid)
        mine = (uuid, [_export(t) for t in (*self.bufs, self.slots)])
        everyone: List = [None, None]
        dist.all_gather_object(everyone, mine, group=group)
        peer_uuid, peer_entries = everyone[self.peer]
        if peer_uuid == uuid:
            raise ValueError("CAMERA_REDUCE='p2p': the two ranks of a camera group share one GPU")
        self._bases: Dict[bytes, int] = {}
        ptrs = []
        for handle, offset in peer_entries:
            if handle not in self._bases:
                base = ctypes.c_void_p()
                L.check("ipc_open", L.lib().s4d_ipc_open(handle, ctypes.byref(base)))
                self._bases[handle] = int(base.value)
            ptrs.append(self._bases[handle] + offset)
        self.peer_bufs, self.peer_slots = ptrs[:2], ptrs[2]
        self._slot_array = (ctypes.c_void_p * 8)()
        self._slot_array[self.peer] = self.peer_slots

    def current(self, rows: int) -> torch.Tensor:
        """``[rows, C]`` view of this call's buffer (the gather's output)."""
        if rows > self.capacity:
            raise ValueError(f"{rows} rows exceed the shared buffers' {self.capacity}")
        return self.bufs[self.epoch & 1][:rows]

    def exchange(self) -> int:
        """Launch the flag exchange of this call on the current stream; returns the address of the
        other rank's buffer of the same call."""
        from . import _lib as L

        idx = self.epoch & 1
        self.epoch += 1
        st = L.lib().s4d_peer_signal_wait(self.slots.data_ptr(), ctypes.cast(self._slot_array, ctypes.c_void_p),
                                          self.rank, 2, self.epoch & 0xFFFFFFFF, self.limit_ns,
                                          self.error_flag.data_ptr(), torch.cuda.current_stream(self.device).cuda_stream)
        L.check("peer_signal_wait", st)
        return self.peer_bufs[idx]

    def check(self) -> None:
        """Raise if a wait gave up (synchronises with the device)."""
        from . import _lib as L

        if int(self.error_flag.item()) & L.S4D_FLAG_PEER_TIMEOUT:
            raise RuntimeError("peer_signal_wait gave up waiting for the other rank of the camera group")

    def close(self) -> None:
        """Collective: both ranks finish their work, then unmap the other's buffers."""
        from . import _lib as L

        if not self._bases:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        for base in self._bases.values():
            L.check("ipc_close", L.lib().s4d_ipc_close(base))
        self._bases = {}
        dist.barrier(group=self.group)  # neither rank frees its buffers while the other maps them
