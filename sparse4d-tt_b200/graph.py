"""CUDA-graph execution of DFA layers: a stack of ``DeformableFeatureAggregation`` calls over one
batch of frames captured once and replayed, so that a decoder pass costs one graph launch
instead of seven kernel launches (and their host-side work) per layer.

The reference runs its decoder eagerly (``model/sparse4d_head.py:405-461`` calls each DFA layer
in turn); the work per replay is identical to the eager calls: every kernel, including the
per-frame camera encoder, runs on every replay.

* ``capture(fn)`` -- records any callable that only launches work on the current stream and
  allocates through torch (every operator of this package qualifies) and returns a
  ``CapturedCall`` whose ``replay()`` re-runs it on the same buffers.
* ``DFAStack`` -- static input buffers + the captured chain ``inst -> layer 0 -> ... -> layer
  L-1`` (each layer fed the previous layer's first C output channels, as stacked decoder layers
  are), with ``run(...)`` copying new inputs in, replaying and returning the static output.
"""
from __future__ import annotations

import contextlib
from typing import Callable, List, Optional, Sequence, Tuple

import torch

from . import ops

Tensor = torch.Tensor


class CapturedCall:
    """A callable captured into a CUDA graph; ``replay()`` re-runs it and returns its output
    (the same tensors every time)."""

    def __init__(self, graph: torch.cuda.CUDAGraph, output):
        self.graph = graph
        self.output = output

    def replay(self):
        self.graph.replay()
        return self.output


def capture(fn: Callable[[], object], warmup: int = 2, pool=None,
            before_capture: Optional[Callable[[], None]] = None) -> CapturedCall:
    """Runs ``fn`` ``warmup`` times on a side stream (so allocations and lazy set-up happen
    outside the graph), calls ``before_capture`` (if given), then records one call.  ``fn`` must
    launch its work on the current stream and must not synchronise with the host."""
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(warmup):
            fn()
    torch.cuda.current_stream().wait_stream(side)
    if before_capture is not None:
        before_capture()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, pool=pool):
        out = fn()
    return CapturedCall(g, out)


@contextlib.contextmanager
def chained_camera_terms(layers: Sequence):
    """Within the block, each DFA layer of ``layers`` (run in this order on the same frames)
    starts the next layer's per-frame camera terms just before its own gather
    (``DeformableFeatureAggregation.next_layer``); the links are removed on exit."""
    layers = list(layers)
    for a, b in zip(layers[:-1], layers[1:]):
        a.next_layer = b
    try:
        yield
    finally:
        for m in layers:
            m.next_layer = None


class DFAStack:
    """``len(layers)`` stacked DFA layers over ``bs`` frames as one CUDA graph.

    Static inputs (write them in place, or pass tensors to ``run``): ``instance_feature [bs, A,
    C]``, per-layer ``anchors[i] [bs, A, 11]`` and ``anchor_embeds[i] [bs, A, C]``, the packed
    maps ``mc_ms_feat [bs, num_feat, C]`` (with ``spatial_shape`` / ``scale_start_index``),
    ``projection_mat [bs, Ncam, 4, 4]`` and ``image_wh [bs, Ncam, 2]``.  The output is the last
    layer's ``[bs, A, 2C]`` (residual ``cat``) or ``[bs, A, C]``."""

    def __init__(self, layers: Sequence, bs: int, num_anchor: int, spatial_shapes: Sequence[Tuple[int, int]],
                 feature_dtype: torch.dtype = torch.bfloat16, warmup: int = 2, time_gathers: bool = False):
        if not layers:
            raise ValueError("DFAStack needs at least one layer")
        m0 = layers[0]
        dev = m0.device
        C, nc = m0.embed_dims, m0.num_cams
        self.layers = list(layers)
        self.bs, self.num_anchor, self.spatial_shapes = bs, num_anchor, [tuple(s) for s in spatial_shapes]
        self.spatial_shape, self.scale_start_index, num_feat = ops.level_tables(self.spatial_shapes, nc, device=dev)
        self.mc_ms_feat = torch.zeros(bs, num_feat, C, dtype=feature_dtype, device=dev)
        self.instance_feature = torch.zeros(bs, num_anchor, C, device=dev)
        self.anchors = [torch.zeros(bs, num_anchor, 11, device=dev) for _ in layers]
        self.anchor_embeds = [torch.zeros(bs, num_anchor, C, device=dev) for _ in layers]
        self.projection_mat = torch.zeros(bs, nc, 4, 4, device=dev)
        self.projection_mat[..., 2, 2] = 1.0  # finite camera terms during warm-up
        self.projection_mat[..., 3, 3] = 1.0
        self.image_wh = torch.ones(bs, nc, 2, device=dev)
        self._gather_events = None
        if not time_gathers:
            self._call = capture(self._forward, warmup=warmup)
            return
        # Each layer's gather is bracketed by two event-record nodes of the graph: after a replay
        # has completed they hold that replay's device timestamps.
        def log_on():
            for mod in self.layers:
                mod.event_log = []

        self._call = capture(self._forward, warmup=warmup, before_capture=log_on)
        self._gather_events = [pair for mod in self.layers for pair in mod.event_log]
        for mod in self.layers:
            mod.event_log = None

    def _forward(self) -> Tensor:
        packed = (self.mc_ms_feat, self.spatial_shape, self.scale_start_index)
        inst, out = self.instance_feature, None
        C = self.layers[0].embed_dims
        for mod in self.layers:  # a new batch of frames: the camera terms are recomputed
            mod.reset_frame_cache()
        with chained_camera_terms(self.layers):
            for i, mod in enumerate(self.layers):
                out = mod.run(inst, self.anchors[i], self.anchor_embeds[i], packed, self.projection_mat, self.image_wh,
                              self.spatial_shapes, self.bs, self.num_anchor)
                inst = out[..., :C]
        for mod in self.layers:
            mod.join_timing_stream()
        return out

    @property
    def output(self) -> Tensor:
        return self._call.output

    def replay(self) -> Tensor:
        return self._call.replay()

    def gather_times_ms(self) -> List[float]:
        """Device time of every layer's gather launch in the latest completed replay, in
        milliseconds (built with ``time_gathers=True``; call after the replay has finished)."""
        if self._gather_events is None:
            raise RuntimeError("DFAStack was built without time_gathers")
        return [s.elapsed_time(e) for s, e in self._gather_events]

    def run(self, instance_feature: Optional[Tensor] = None, anchors: Optional[List[Tensor]] = None,
            anchor_embeds: Optional[List[Tensor]] = None, mc_ms_feat: Optional[Tensor] = None,
            projection_mat: Optional[Tensor] = None, image_wh: Optional[Tensor] = None) -> Tensor:
        """Copies the given inputs (host or device tensors; pinned host memory copies
        asynchronously) into the static buffers, replays and returns the static output."""
        def put(dst, src):
            if src is not None:
                dst.copy_(src, non_blocking=True)

        put(self.instance_feature, instance_feature)
        for d, s in zip(self.anchors, anchors or []):
            put(d, s)
        for d, s in zip(self.anchor_embeds, anchor_embeds or []):
            put(d, s)
        put(self.mc_ms_feat, mc_ms_feat)
        put(self.projection_mat, projection_mat)
        put(self.image_wh, image_wh)
        return self.replay()


class PipelinedDFAStack:
    """Batches streamed from host memory through two ``DFAStack`` graphs of the same layers, so
    that the upload of batch ``k + 1`` overlaps the replay of batch ``k``.

    ``submit(...)`` takes one batch's inputs (pinned host tensors for asynchronous copies; the
    argument meaning of ``DFAStack.run``) and returns at once.  Its copies run on a copy stream
    into the static buffers of graph ``k % 2`` as soon as that graph's previous replay (batch
    ``k - 2``) has read them; the replay runs on the current stream after the copies, and the
    output is copied into ``out`` (a pinned host tensor, if given) behind it.  The host tensors of
    a batch must stay unchanged until its copies are done: ``wait(k)`` (or ``synchronize()``)
    returns when batch ``k`` is complete.  Graph ``k % 2``'s output tensor holds batch ``k``'s
    result until batch ``k + 2`` replays."""

    def __init__(self, layers: Sequence, bs: int, num_anchor: int, spatial_shapes: Sequence[Tuple[int, int]],
                 feature_dtype: torch.dtype = torch.bfloat16, warmup: int = 2):
        self.stacks = [DFAStack(layers, bs, num_anchor, spatial_shapes, feature_dtype, warmup) for _ in range(2)]
        dev = layers[0].device
        self.copy_stream = torch.cuda.Stream(dev)
        self._freed = [torch.cuda.Event() for _ in range(2)]  # the graph's last replay has read its inputs
        self._copied = [torch.cuda.Event() for _ in range(2)]
        self._done: List[Optional[torch.cuda.Event]] = []
        self._count = 0

    def submit(self, instance_feature: Optional[Tensor] = None, anchors: Optional[List[Tensor]] = None,
               anchor_embeds: Optional[List[Tensor]] = None, mc_ms_feat: Optional[Tensor] = None,
               projection_mat: Optional[Tensor] = None, image_wh: Optional[Tensor] = None,
               out: Optional[Tensor] = None) -> int:
        k = self._count
        j = k % 2
        st = self.stacks[j]
        cur = torch.cuda.current_stream()
        if k >= 2:
            self.copy_stream.wait_event(self._freed[j])
        with torch.cuda.stream(self.copy_stream):
            def put(dst, src):
                if src is not None:
                    dst.copy_(src, non_blocking=True)

            put(st.instance_feature, instance_feature)
            for d, s in zip(st.anchors, anchors or []):
                put(d, s)
            for d, s in zip(st.anchor_embeds, anchor_embeds or []):
                put(d, s)
            put(st.mc_ms_feat, mc_ms_feat)
            put(st.projection_mat, projection_mat)
            put(st.image_wh, image_wh)
            self._copied[j].record(self.copy_stream)
        cur.wait_event(self._copied[j])
        st.replay()
        self._freed[j].record(cur)
        if out is not None:
            out.copy_(st.output, non_blocking=True)
        done = torch.cuda.Event()
        done.record(cur)
        self._done.append(done)
        self._count += 1
        return k

    def output(self, k: int) -> Tensor:
        """Device output of batch ``k`` (valid until batch ``k + 2`` replays)."""
        return self.stacks[k % 2].output

    def wait(self, k: int) -> None:
        self._done[k].synchronize()

    def synchronize(self) -> None:
        if self._done:
            self._done[-1].synchronize()
