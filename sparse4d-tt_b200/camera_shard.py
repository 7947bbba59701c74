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
  kernel: each rank's gather writes the other rank's rows of its partial sums straight into that
  rank's receive buffer over NVLink (``PeerPartialSums``, CUDA IPC; the transfer overlaps the
  gather), a bounded flag exchange orders the two GPUs, and ``output_proj`` sums its own partial
  sums and the received ones, both in local memory, in the tensor-core accumulator
  (``s4d_dfa_output_proj_sum``).
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

    Each rank owns ``part`` (its own partial sums of its own rows) and ``recv`` (the other
    rank's partial sums of this rank's rows, written by the other rank's gather over NVLink),
    both ``[capacity, C]`` fp32 rows with the flattened (frame, anchor) indexing; two slot arrays
    in which the other rank publishes its epochs (partial sums sent; receive buffer free again);
    and a device epoch counter.  Per call: ``begin()`` launches the "consumed" exchange (this
    rank has finished reading its ``recv`` of the previous call, and waits until the other rank
    has finished reading its own, which this call's gather is about to overwrite) and returns the
    ``part`` view; the gather writes this rank's rows to ``part`` and the other rank's rows to
    ``peer_recv``; ``exchange()`` launches the "ready" exchange; then ``output_proj`` sums ``part``
    and ``recv``, both local.  The epochs live on the device (``s4d_peer_signal_wait_counter``),
    so a CUDA graph that captured a call replays correctly, and eager calls and replays may be
    mixed, as long as both ranks make the same sequence of calls.  Construction and ``close()``
    are collective over the group; the two ranks must be on different GPUs (their waits must run
    at the same time).  A wait that gives up after ``limit_ns`` sets ``S4D_FLAG_PEER_TIMEOUT``
    in ``error_flag`` (``check()`` reads it)."""

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
        self.part = torch.empty(self.capacity, channels, dtype=torch.float32, device=self.device)
        self.recv = torch.empty(self.capacity, channels, dtype=torch.float32, device=self.device)
        # slots [0:8] ready epochs, [8:16] consumed epochs (slot r written by rank r), [16] the
        # epoch counter (calls whose ready exchange has run)
        self.slots = torch.zeros(24, dtype=torch.int32, device=self.device)
        self.error_flag = torch.zeros(1, dtype=torch.int32, device=self.device)
        torch.cuda.synchronize(self.device)  # the zeroed slots are in place before the peer can write them
        uuid = str(torch.cuda.get_device_properties(self.device).uuid)
        mine = (uuid, [_export(t) for t in (self.recv, self.slots)])
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
        self.peer_recv, peer_slots = ptrs
        self._ready = (ctypes.c_void_p * 8)()
        self._ready[self.peer] = peer_slots
        self._consumed = (ctypes.c_void_p * 8)()
        self._consumed[self.peer] = peer_slots + 8 * 4
        self.closed = False

    def _signal(self, own_offset: int, peers, advance: int) -> None:
        from . import _lib as L

        if self.closed:
            raise RuntimeError("PeerPartialSums: used after close() (the other rank's buffers are unmapped)")
        base = self.slots.data_ptr()
        st = L.lib().s4d_peer_signal_wait_counter(base + own_offset * 4, ctypes.cast(peers, ctypes.c_void_p),
                                                  self.rank, 2, base + 16 * 4, advance, self.limit_ns,
                                                  self.error_flag.data_ptr(),
                                                  torch.cuda.current_stream(self.device).cuda_stream)
        L.check("peer_signal_wait_counter", st)

    def begin(self, rows: int) -> torch.Tensor:
        """Launch this call's "consumed" exchange; returns the ``[rows, C]`` view of ``part``."""
        if self.closed:
            raise RuntimeError("PeerPartialSums: used after close() (the other rank's buffers are unmapped)")
        if rows > self.capacity:
            raise ValueError(f"{rows} rows exceed the shared buffers' {self.capacity}")
        self._signal(8, self._consumed, 0)
        return self.part[:rows]

    def exchange(self) -> torch.Tensor:
        """Launch this call's "ready" exchange (after the gather) on the current stream; returns
        ``recv``, which then holds the other rank's partial sums of this rank's rows."""
        self._signal(0, self._ready, 1)
        return self.recv

    def check(self) -> None:
        """Raise if a wait gave up (synchronises with the device)."""
        from . import _lib as L

        if int(self.error_flag.item()) & L.S4D_FLAG_PEER_TIMEOUT:
            raise RuntimeError("peer_signal_wait gave up waiting for the other rank of the camera group")

    def epochs(self) -> int:
        """Calls whose ready exchange has run on this rank (synchronises with the device)."""
        return int(self.slots[16].item())

    def close(self) -> None:
        """Collective: both ranks finish their work, then unmap the other's buffers."""
        from . import _lib as L

        if self.closed:
            return
        self.closed = True
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        for base in self._bases.values():
            L.check("ipc_close", L.lib().s4d_ipc_close(base))
        self._bases = {}
        self.peer_recv = None
        dist.barrier(group=self.group)  # neither rank frees its buffers while the other maps them
