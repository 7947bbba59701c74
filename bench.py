#!/usr/bin/env python
"""Benchmark of the B200 DFA hot path (Sparse4D v3 DeformableFeatureAggregation).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N --master-addr 127.0.0.1 ... bench.py --gpus N ...

One step = six stacked DFA layers (different weights, anchors refined between layers, each
layer's output feeding the next) over a batch of 32 frames per GPU at the Sparse4D v3 R50
shape: 900 anchors x 13 keypoints x 6 cameras x 4 levels x 256 channels, bf16 channels-last
maps of a 704x256 image, fp32 accumulation.  Each layer runs through the drop-in
``DeformableFeatureAggregation.run`` (this library's tensor-core weights_fc and output_proj,
the camera kernels and the fused keypoint + softmax + gather kernel), the 6 layers captured
as one CUDA graph.  Frames shard across GPUs with no collective in the timed region (weak
scaling: 32 frames per GPU).

Printed (rank 0, one JSON line): DFA calls/s for the whole job (calls = frames x layers),
the gather kernel's roofline (algorithmic bytes per launch over its CUDA-event duration,
against the measured HBM peak), the CPU baseline (the oracle's torch port of the reference
DFA on this host), end-to-end calls/s through the module with host buffers, and a bs=1
latency figure with L2 flushed between iterations.

``--impl reference`` times the reference algorithm on the host CPU instead (the oracle port:
the reference is a Tenstorrent TT-NN program and its PyTorch DFA is the CPU implementation),
one single-frame DFA layer per step.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

import torch  # noqa: E402

METRIC = "DFA calls/s and keypoint-samples/s per B200 (bf16) at 1/2/4/8 GPUs; % HBM roofline"
UNIT = "DFA calls/s"
SAMPLES_PER_CALL = 900 * 13 * 6 * 4  # logical keypoint samples of one frame through one layer
FALLBACK_HBM_GBS = 6650.0
# bf16 maps (fp32 accumulation); the layer's linears on TF32 tensor cores with fp32
# accumulation (the reference's TT path runs them in bf16); parity of exactly this
# configuration: tests/test_gpu_dfa_layer.py::test_layer_bf16_tf32_linears
MODEL_CONFIG = {"FEATURE_DTYPE": torch.bfloat16, "MATMUL_PRECISION": "tf32"}


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--frames", type=int, default=32, help="frames per GPU")
    ap.add_argument("--layers", type=int, default=6)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-bs1", action="store_true")
    ap.add_argument("--no-highres", action="store_true")
    ap.add_argument("--profile-gather", action="store_true",
                    help="profiling case: one layer over --frames frames, one warm-up call then one call "
                         "inside the NVTX range 'profile' (few launches before the profiled gather)")
    return ap.parse_args()


def env_dist():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


def measured_hbm():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def workload_config(frames, layers, world):
    return {
        "workload": f"{layers} stacked DFA layers x {frames} frames per GPU; 900 anchors x 13 pts x 6 cams x "
                    f"4 levels x 256 ch; 704x256 image (maps 64x176, 32x88, 16x44, 8x22); bf16 maps",
        "frames_per_gpu": frames, "layers": layers, "global_batch": frames * world,
        "anchors": 900, "num_pts": 13, "num_cams": 6, "num_levels": 4, "embed_dims": 256, "num_groups": 8,
        "accumulate": "f32", "logits": "split (per-anchor + per-camera terms, summed in the gather kernel)",
        "linears": "TF32 operands, fp32 accumulation: weights_fc + learnable_fc (embed add fused) and "
                   "output_proj (residual cat fused) on this library's tcgen05 kernels; the per-frame "
                   "camera encoder + per-camera logits on this library's fp32 kernels, recomputed every step",
        "parallelism": f"dp{world} (frames)",
        "l2": "inputs larger than L2 (1.47 GB of maps per GPU, re-read by every layer)",
    }


# ---------------------------------------------------------------------------------------------
# clocks
# ---------------------------------------------------------------------------------------------
class ClockSampler:
    """SM clock and clock-event reasons sampled during the timed region: NVML polled every
    2 ms from a thread (read-only queries), or nvidia-smi at 200 ms when NVML is missing."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")
    # NVML clocks-event reason bits
    REASON_BITS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20,
                   "hw_thermal_slowdown": 0x40, "hw_power_brake_slowdown": 0x80}

    def __init__(self, device):
        self.proc = None
        self.lines = []
        self.nvml = None
        try:
            import pynvml

            pynvml.nvmlInit()
            uuid = str(torch.cuda.get_device_properties(device).uuid)
            gid = uuid if uuid.startswith("GPU-") else f"GPU-{uuid}"
            h = pynvml.nvmlDeviceGetHandleByUUID(gid)
            reasons = getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                pynvml.nvmlDeviceGetCurrentClocksThrottleReasons
            self.nvml = (pynvml, h, reasons)
            self.samples = []
            self.stop_flag = threading.Event()
            self.t = threading.Thread(target=self._poll, daemon=True)
            self.t.start()
            return
        except Exception:
            self.nvml = None
        try:
            uuid = str(torch.cuda.get_device_properties(device).uuid)
            gid = uuid if uuid.startswith("GPU-") else f"GPU-{uuid}"
            self.proc = subprocess.Popen(["nvidia-smi", "-i", gid, f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None

    def _read(self):
        for ln in self.proc.stdout:
            self.lines.append(ln.strip())

    def _poll(self):
        pynvml, h, reasons = self.nvml
        while not self.stop_flag.is_set():
            try:
                self.samples.append((pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM),
                                     pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM), int(reasons(h))))
            except Exception:
                pass
            self.stop_flag.wait(0.002)

    def stop(self):
        if self.nvml is not None:
            self.stop_flag.set()
            self.t.join(timeout=2)
            if not self.samples:
                return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"], "source": "nvml"}
            found = sorted({n for _, _, r in self.samples for n, bit in self.REASON_BITS.items() if r & bit})
            return {"sm_mhz": statistics.median(s for s, _, _ in self.samples),
                    "sm_max_mhz": max(m for _, m, _ in self.samples), "reasons": found,
                    "samples": len(self.samples), "source": "nvml, polled every 2 ms"}
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.t.join(timeout=2)
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[0]))
                smax.append(float(parts[1]))
            except ValueError:
                continue
            for n, v in zip(names, parts[4:8]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(smax), "reasons": sorted(reasons),
                "samples": len(sm)}


# ---------------------------------------------------------------------------------------------
# workload
# ---------------------------------------------------------------------------------------------
class Workload:
    """Device-resident inputs of one step on one GPU (the standard 704x256, 900-anchor shape
    unless ``cfg`` says otherwise; ``mesh_device`` / ``model_config`` go to every layer)."""

    def __init__(self, frames, layers, device, seed, cfg=None, mesh_device=None, model_config=None):
        from sparse4d_tt_b200 import DeformableFeatureAggregation, ops
        from sparse4d_tt_b200 import synthetic as syn

        self.cfg = syn.DFAConfig(bs=frames) if cfg is None else cfg
        cfg = self.cfg
        mc = MODEL_CONFIG if model_config is None else model_config
        self.frames, self.layers, self.device = frames, layers, device
        gen = torch.Generator().manual_seed(seed)
        self.shape, self.start, self.num_feat = ops.level_tables(cfg.spatial_shapes, cfg.num_cams, device=device)
        dgen = torch.Generator(device=device).manual_seed(seed)
        self.feat = torch.randn(frames, self.num_feat, cfg.embed_dims, device=device, generator=dgen,
                                dtype=torch.bfloat16)
        self.packed = (self.feat, self.shape, self.start)
        self.inst0 = torch.randn(frames, cfg.num_anchor, cfg.embed_dims, generator=gen).to(device)
        a = syn.make_anchors(frames, cfg.num_anchor, gen)
        self.anchors, self.embeds, self.mods, self.params = [], [], [], []
        for layer in range(layers):
            self.anchors.append(a.to(device))
            self.embeds.append(torch.randn(frames, cfg.num_anchor, cfg.embed_dims, generator=gen).to(device))
            params = syn.make_params(cfg, torch.Generator().manual_seed(seed * 100 + layer))
            self.params.append(params)
            self.mods.append(DeformableFeatureAggregation(device, params, mc, split_logits=True,
                                                          mesh_device=mesh_device))
            a = syn.refine_anchors(a, gen)
        self.proj = syn.camera_ring(cfg.num_cams, cfg.image_wh)[None].expand(frames, -1, -1, -1).contiguous().to(device)
        self.wh = torch.tensor(cfg.image_wh, dtype=torch.float32).expand(frames, cfg.num_cams, 2).contiguous().to(device)

    def step(self, inst=None, anchors=None, embeds=None, packed=None, proj=None, wh=None):
        from sparse4d_tt_b200 import chained_camera_terms

        inst = self.inst0 if inst is None else inst
        anchors = self.anchors if anchors is None else anchors
        embeds = self.embeds if embeds is None else embeds
        packed = self.packed if packed is None else packed
        proj = self.proj if proj is None else proj
        wh = self.wh if wh is None else wh
        out = None
        for mod in self.mods:  # a new batch of frames: per-frame camera caches start empty
            mod.reset_frame_cache()
        with chained_camera_terms(self.mods):  # each layer starts the next one's camera terms
            for layer, mod in enumerate(self.mods):
                out = mod.run(inst, anchors[layer], embeds[layer], packed, proj, wh, self.cfg.spatial_shapes,
                              self.frames, self.cfg.num_anchor)
                inst = out[..., : self.cfg.embed_dims]
        return out

    def graph_stack(self):
        """The same step as one CUDA graph (DFAStack over these modules), static inputs filled
        from this workload; each layer's gather launch is bracketed by event-record nodes."""
        from sparse4d_tt_b200 import DFAStack

        st = DFAStack(self.mods, self.frames, self.cfg.num_anchor, self.cfg.spatial_shapes, time_gathers=True)
        st.run(self.inst0, self.anchors, self.embeds, self.feat, self.proj, self.wh)
        return st

    @torch.no_grad()
    def algorithmic_bytes_per_layer(self):
        """Compulsory HBM bytes of each layer's gather launch: unique in-bounds tap pixels x
        256 ch x 2 B + split logits + sample locations + output.  Computed from the sample
        locations of an untimed pass (replaying the module's own keypoint step).  Returns per
        layer (bytes, unique tap pixels, in-bounds samples)."""
        import torch.nn.functional as F

        from sparse4d_tt_b200 import ops

        cfg, dev = self.cfg, self.device
        inst = self.inst0
        out_bytes = []
        for layer, mod in enumerate(self.mods):
            learn = F.linear(inst, mod.learnable_fc_weight, mod.learnable_fc_bias).contiguous()
            loc = torch.empty(self.frames, cfg.num_anchor, cfg.num_cams, cfg.num_pts, 2, device=dev)
            ops.kps_project_into(self.anchors[layer], learn, mod.fix_scale, self.proj, self.wh, sample_location=loc)
            touched = unique_tap_pixels(loc, cfg.spatial_shapes, self.start, self.num_feat)
            inb = inbounds_samples(loc, cfg.spatial_shapes)
            lpg = cfg.num_levels * cfg.num_pts * cfg.num_groups
            if mod.fused_keypoints:  # the gather reads the anchors + keypoint logits, not locations
                kps_in = (self.anchors[layer].numel() + learn.numel() + self.proj.numel() + self.wh.numel()) * 4
            else:
                kps_in = loc.numel() * 4
            b = (touched * cfg.embed_dims * 2
                 + self.frames * cfg.num_anchor * lpg * 4 + self.frames * cfg.num_cams * lpg * 4
                 + kps_in + self.frames * cfg.num_anchor * cfg.embed_dims * 4)
            out_bytes.append((b, touched, inb))
            out = mod.run(inst, self.anchors[layer], self.embeds[layer], self.packed, self.proj, self.wh,
                          cfg.spatial_shapes, self.frames, cfg.num_anchor)
            inst = out[..., : cfg.embed_dims]
        return out_bytes


def launches_per_layer(w):
    """This library's kernels per DFA layer: the gather, plus the keypoints unless the gather
    computes them; with split logits the camera terms (one launch with the softmax factors for
    the Sparse4D v3 shape, else the two camera-encoder launches); the two tensor-core linears
    (weights_fc + learnable_fc, output_proj + residual) when the layer runs them."""
    m = w.mods[0]
    one_launch = m._factors_ok and w.frames <= m.camera_terms_max_frames
    camera = (1 if one_launch else 2 + (1 if m._factors_ok else 0)) if m.split_logits else 0
    return 1 + (0 if m.fused_keypoints else 1) + camera + (2 if m._tc else 0)


def inbounds_samples(loc, spatial_shapes):
    """Number of (batch, anchor, camera, point, level) samples of ``loc [bs, A, Ncam, P, 2]``
    with at least one in-bounds bilinear tap (grid_sample, align_corners=False): the samples
    whose taps the gather loads."""
    n = 0
    for h, w in spatial_shapes:
        ix = ((loc[..., 0] * 2 - 1 + 1) * w - 1) * 0.5
        iy = ((loc[..., 1] * 2 - 1 + 1) * h - 1) * 0.5
        n += int(((ix > -1) & (ix < w) & (iy > -1) & (iy < h)).sum())
    return n


def unique_tap_pixels(loc, spatial_shapes, start, num_feat):
    """Number of distinct feature rows (batch, camera, level, y, x) that the in-bounds bilinear
    taps of ``loc [bs, A, Ncam, P, 2]`` touch (grid_sample, align_corners=False)."""
    bs, A, nc, P, _ = loc.shape
    dev = loc.device
    mark = torch.zeros(bs * num_feat, dtype=torch.bool, device=dev)
    b_idx = torch.arange(bs, device=dev).view(bs, 1, 1, 1)
    starts = start.to(torch.int64)
    for l, (h, w) in enumerate(spatial_shapes):
        ix = ((loc[..., 0] * 2 - 1 + 1) * w - 1) * 0.5
        iy = ((loc[..., 1] * 2 - 1 + 1) * h - 1) * 0.5
        x0, y0 = ix.floor(), iy.floor()
        cam_start = starts[:, l].view(1, 1, nc, 1)
        for dx in (0, 1):
            for dy in (0, 1):
                x, y = x0 + dx, y0 + dy
                ok = (x >= 0) & (x < w) & (y >= 0) & (y < h)
                pix = b_idx * num_feat + cam_start + y.clamp(0, h - 1).long() * w + x.clamp(0, w - 1).long()
                mark[pix[ok]] = True
    return int(mark.sum())


# ---------------------------------------------------------------------------------------------
# legs
# ---------------------------------------------------------------------------------------------
def time_steps(fn, steps, sync_barrier):
    sync_barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.nvtx.range_push("timed")
    e0.record()
    for _ in range(steps):
        fn()
    e1.record()
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    sync_barrier()
    return e0.elapsed_time(e1)


def h2d_bandwidth(host, device, reps=3):
    """Best-of-``reps`` GB/s of one plain copy of the pinned host tensor ``host`` to the device
    (CUDA events on the current stream)."""
    dst = torch.empty(host.shape, dtype=host.dtype, device=device)
    best = None
    for _ in range(reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        dst.copy_(host, non_blocking=True)
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1)
        best = ms if best is None else min(best, ms)
    nbytes = host.numel() * host.element_size()
    del dst
    return nbytes / best / 1e6


def gpu_numa_node(device):
    """NUMA node of the GPU's PCI device (sysfs), or None."""
    try:
        p = torch.cuda.get_device_properties(device)
        bus = f"{p.pci_domain_id:04x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
        with open(f"/sys/bus/pci/devices/{bus}/numa_node") as f:
            return int(f.read().strip())
    except Exception:
        return None


def e2e_leg(w, steps, warmup, sync_barrier):
    """The step end to end through the library's public API: ``PipelinedDFAStack.submit`` with
    every input copied from pinned host memory inside the timed region and the final output
    read back into pinned host memory.  The two graphs of the pipeline let step k + 1's uploads
    (on a copy stream) overlap step k's replay, so the step is bound by the host-to-device
    copies; their floor is the bytes over the plain pinned-copy bandwidth measured here."""
    from sparse4d_tt_b200 import PipelinedDFAStack

    host = {
        "mc_ms_feat": w.feat.cpu().pin_memory(), "instance_feature": w.inst0.cpu().pin_memory(),
        "anchors": [a.cpu().pin_memory() for a in w.anchors],
        "anchor_embeds": [e.cpu().pin_memory() for e in w.embeds],
        "projection_mat": w.proj.cpu().pin_memory(), "image_wh": w.wh.cpu().pin_memory(),
    }
    outs = [torch.empty(w.frames, w.cfg.num_anchor, 2 * w.cfg.embed_dims, pin_memory=True) for _ in range(2)]
    h2d = (host["mc_ms_feat"].numel() * 2 + host["instance_feature"].numel() * 4
           + sum(a.numel() * 4 for a in host["anchors"]) + sum(e.numel() * 4 for e in host["anchor_embeds"])
           + host["projection_mat"].numel() * 4 + host["image_wh"].numel() * 4)
    d2h = outs[0].numel() * 4
    pipe = PipelinedDFAStack(w.mods, w.frames, w.cfg.num_anchor, w.cfg.spatial_shapes)
    count = [0]

    def step():
        pipe.submit(out=outs[count[0] % 2], **host)
        count[0] += 1

    for _ in range(warmup):
        step()
    pipe.synchronize()
    ms = time_steps(step, steps, sync_barrier)
    gbs = h2d_bandwidth(host["mc_ms_feat"], w.device)
    del pipe
    torch.cuda.empty_cache()
    return ms, h2d, d2h, gbs


def bs1_leg(device, iters=200):
    """Single frame, single layer (the Sparse4D bs=1 inference shape): the gather kernel timed
    alone with a >= 2x L2 write between iterations, and the whole layer (eager) timed the same
    way."""
    import torch.nn.functional as F

    from sparse4d_tt_b200 import DeformableFeatureAggregation, ops
    from sparse4d_tt_b200 import synthetic as syn

    cfg = syn.config_standard(1)
    ins = syn.make_inputs(cfg, 0, feature_dtype=torch.bfloat16)
    params = syn.make_params(cfg, torch.Generator().manual_seed(100))
    mod = DeformableFeatureAggregation(device, params, MODEL_CONFIG, split_logits=True)
    packed = ops.pack_feature_maps([m.to(device) for m in ins.feature_maps], dtype=torch.bfloat16)
    inst, anchor, embed = (t.to(device) for t in (ins.instance_feature, ins.anchor, ins.anchor_embed))
    proj, wh = ins.projection_mat.to(device), ins.image_wh.to(device)
    wa, wc = mod._get_weights(inst, embed, proj, 1, 900)
    wa, wc = wa.contiguous(), wc.contiguous()
    learn = F.linear(inst, mod.learnable_fc_weight, mod.learnable_fc_bias).contiguous()
    loc = torch.empty(1, 900, 6, 13, 2, device=device)
    ops.kps_project_into(anchor, learn, mod.fix_scale, proj, wh, sample_location=loc)
    out = torch.empty(1, 900, 256, device=device)
    l2 = torch.cuda.get_device_properties(device).L2_cache_size
    flush = torch.empty(max(2 * l2, 256 << 20) // 4, dtype=torch.float32, device=device)
    touched = unique_tap_pixels(loc, cfg.spatial_shapes, packed[2], packed[0].shape[1])
    lpg = 4 * 13 * 8
    alg_loc = touched * 512 + 900 * lpg * 4 + 6 * lpg * 4 + loc.numel() * 4 + out.numel() * 4
    # the module's own gather at bs=1 (as DeformableFeatureAggregation.run launches it): the
    # sample locations computed in the kernel from the anchors and keypoint logits, with the
    # per-frame camera factors in the workspace
    mod.reset_frame_cache()
    mod.run(inst, anchor, embed, packed, proj, wh, cfg.spatial_shapes, 1, 900)
    assert mod.fused_keypoints
    ws, wc_mod = mod._cached_camera_factors, mod._cached_camera_logits
    logits = torch.empty(1, 900, 4, 13, 8, device=device)
    learn_tc = torch.empty(1, 900, 18, device=device)
    ops.weights_fc_into(logits.view(900, -1), learn_tc.view(900, -1), ops.row_view(inst, 256),
                        ops.row_view(embed, 256), mod.weights_fc_weight, mod.learnable_fc_weight, mod.learnable_fc_bias)
    alg = (touched * 512 + 900 * lpg * 4 + 6 * lpg * 4 + (anchor.numel() + learn_tc.numel() + proj.numel()
                                                          + wh.numel()) * 4 + out.numel() * 4)

    def gather():
        ops.deformable_aggregation_anchors_into(out, packed[0], packed[1], packed[2], anchor, mod.fix_scale,
                                                learn_tc.view(900, -1), proj, wh, logits, wc_mod, ws)

    def gather_loc():
        ops.deformable_aggregation_into(out, packed[0], packed[1], packed[2], loc, wa, True, wc)

    def layer():
        mod.reset_frame_cache()
        mod.run(inst, anchor, embed, packed, proj, wh, cfg.spatial_shapes, 1, 900)

    # The same layer as one CUDA graph (graph.DFAStack): one launch per call instead of seven
    # kernels with their host-side work; every kernel, the camera encoder included, still runs.
    from sparse4d_tt_b200 import DFAStack

    stack = DFAStack([mod], 1, 900, cfg.spatial_shapes)
    stack.run(inst, [anchor], [embed], packed[0], proj, wh)

    res = {}
    for name, fn in (("gather", gather), ("gather_loc", gather_loc), ("layer", layer), ("layer_graph", stack.replay)):
        for _ in range(20):  # warm-up
            fn()
        times = []
        for _ in range(iters):
            flush.fill_(1.0)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            times.append((e0, e1))
        torch.cuda.synchronize()
        ms = sorted(s.elapsed_time(e) for s, e in times)
        res[name] = {"median_us": 1000 * ms[len(ms) // 2], "p10_us": 1000 * ms[len(ms) // 10],
                     "p90_us": 1000 * ms[(9 * len(ms)) // 10]}
    peak, src = measured_hbm()
    g_s = res["gather"]["median_us"] * 1e-6
    gl_s = res["gather_loc"]["median_us"] * 1e-6
    rot = bs1_rotating(device, mod, cfg)
    return {
        "workload": "1 frame, 1 DFA layer, 900 anchors, bf16 maps (704x256 image); L2 written (>= 2x L2) "
                    "before every iteration",
        "gather_kernel": "the module's gather: s4d_deformable_aggregation_anchors (keypoints + projection + "
                         "softmax + gather in one launch, camera factors ready)",
        "gather_kernel_us": res["gather"], "layer_us": res["layer"], "layer_graph_us": res["layer_graph"],
        "layer_calls_per_s": 1e6 / res["layer"]["median_us"],
        "layer_graph_calls_per_s": 1e6 / res["layer_graph"]["median_us"],
        "algorithmic_bytes": alg, "unique_tap_pixels": touched,
        "gather_achieved_gbs": alg / g_s / 1e9, "gather_frac_of_hbm": alg / g_s / 1e9 / peak,
        "gather_loc": {"kernel": "s4d_deformable_aggregation reading a sample-location buffer (CTA per anchor)",
                       "us": res["gather_loc"], "algorithmic_bytes": alg_loc,
                       "frac_of_hbm": alg_loc / gl_s / 1e9 / peak},
        "peak_gbs": peak, "peak_source": src,
        "rotating": rot,
    }


def bs1_rotating(device, mod, cfg, sets=16, replays=13):
    """The module's bs = 1 gather back to back over ``sets`` independent single-frame inputs
    (each its own 46 MB of bf16 maps, anchors and logits: 736 MB of maps in all, so a set's rows
    are long gone from the 126 MB L2 when its turn comes again), the ``sets`` launches captured
    as one CUDA graph and replayed ``replays`` times: per-call time of a stream of bs = 1 calls,
    without the per-call event and L2-flush overhead of the flushed figure."""
    from sparse4d_tt_b200 import ops
    from sparse4d_tt_b200 import synthetic as syn

    shape, start, num_feat = ops.level_tables(cfg.spatial_shapes, cfg.num_cams, device=device)
    proj = syn.camera_ring(6, cfg.image_wh)[None].contiguous().to(device)
    wh = torch.tensor(cfg.image_wh, dtype=torch.float32).expand(1, 6, 2).contiguous().to(device)
    wc = mod._cached_camera_logits
    calls, alg = [], []
    dgen = torch.Generator(device=device).manual_seed(77)
    for r in range(sets):
        gen = torch.Generator().manual_seed(500 + r)
        feat = torch.randn(1, num_feat, 256, device=device, generator=dgen, dtype=torch.bfloat16)
        anchor = syn.make_anchors(1, 900, gen).to(device)
        inst = torch.randn(900, 256, generator=gen).to(device)
        embed = torch.randn(900, 256, generator=gen).to(device)
        logits = torch.empty(1, 900, 4, 13, 8, device=device)
        learn = torch.empty(900, 18, device=device)
        ops.weights_fc_into(logits.view(900, -1), learn, inst, embed, mod.weights_fc_weight, mod.learnable_fc_weight,
                            mod.learnable_fc_bias)
        ws = ops.camera_factors_into(ops.dfa_workspace(1, 6, 4, 13, 8, device), wc)
        out = torch.empty(1, 900, 256, device=device)
        loc = torch.empty(1, 900, 6, 13, 2, device=device)
        ops.kps_project_into(anchor, learn.view(1, 900, 18), mod.fix_scale, proj, wh, sample_location=loc)
        touched = unique_tap_pixels(loc, cfg.spatial_shapes, start, num_feat)
        alg.append(touched * 512 + 900 * 416 * 4 + 6 * 416 * 4 + (anchor.numel() + learn.numel() + proj.numel()
                                                                  + wh.numel()) * 4 + out.numel() * 4)
        calls.append((out, feat, anchor, learn, logits, ws))

    def run_all():
        for out, feat, anchor, learn, logits, ws in calls:
            ops.deformable_aggregation_anchors_into(out, feat, shape, start, anchor, mod.fix_scale, learn, proj, wh,
                                                    logits, wc, ws)

    from sparse4d_tt_b200.graph import capture

    g = capture(run_all, warmup=2)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(replays):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    per_call_us = e0.elapsed_time(e1) * 1e3 / (replays * sets)
    peak, src = measured_hbm()
    a = statistics.mean(alg)
    res = {"workload": f"{sets} independent single-frame inputs (900 anchors, 704x256 bf16 maps, 46 MB each) "
                       f"cycled: {sets} gather launches per CUDA graph replay, {replays} replays timed",
           "per_call_us": per_call_us, "calls_per_s": 1e6 / per_call_us, "algorithmic_bytes": a,
           "achieved_gbs": a / per_call_us / 1e3, "frac_of_hbm": a / per_call_us / 1e3 / peak}
    del calls, g
    torch.cuda.empty_cache()
    return res


def kps_leg(device, iters=200):
    """Keypoints only (one frame, 900 anchors, 13 points, 6 cameras): s4d_kps_project_linear
    computing the learnable keypoint logits (the keypoint generator's learnable_fc) from the
    instance features, then the keypoints, projection, depth mask and the compacted visible (b,
    anchor, cam, pt) list -- the same work the CPU baseline's keypoint leg times -- timed alone
    with a >= 2x L2 write between iterations."""
    from sparse4d_tt_b200 import DeformableFeatureAggregation, ops
    from sparse4d_tt_b200 import synthetic as syn

    cfg = syn.config_standard(1)
    ins = syn.make_inputs(cfg, 0)
    params = syn.make_params(cfg, torch.Generator().manual_seed(100))
    mod = DeformableFeatureAggregation(device, params, {"FEATURE_DTYPE": torch.float32}, split_logits=True)
    anchor, inst = ins.anchor.to(device), ins.instance_feature.to(device)
    proj, wh = ins.projection_mat.to(device), ins.image_wh.to(device)
    inst2d = ops.row_view(inst, cfg.embed_dims)
    A, nc, P = cfg.num_anchor, cfg.num_cams, cfg.num_pts
    loc = torch.empty(1, A, nc, P, 2, device=device)
    mask = torch.empty(1, A, nc, P, dtype=torch.uint8, device=device)
    idx = torch.empty(A * nc * P, 4, dtype=torch.int32, device=device)
    cnt = torch.zeros(1, dtype=torch.int32, device=device)
    ws = torch.empty(max(ops.kps_workspace_bytes(1, A, nc, P), 16), dtype=torch.uint8, device=device)
    l2 = torch.cuda.get_device_properties(device).L2_cache_size
    flush = torch.empty(max(2 * l2, 256 << 20) // 4, dtype=torch.float32, device=device)

    def call():
        ops.kps_project_linear_into(anchor, inst2d, mod.learnable_fc_weight, mod.learnable_fc_bias, mod.fix_scale,
                                    proj, wh, sample_location=loc, depth_mask=mask, visible_idx=idx,
                                    visible_count=cnt, workspace=ws)

    for _ in range(20):  # warm-up
        call()
    times = []
    for _ in range(iters):
        flush.fill_(1.0)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        call()
        e1.record()
        times.append((e0, e1))
    torch.cuda.synchronize()
    ms = sorted(s.elapsed_time(e) for s, e in times)
    med_us = 1000 * ms[len(ms) // 2]
    return {"workload": "1 frame, 900 anchors x 13 points x 6 cameras: learnable keypoint logits (learnable_fc), "
                        "keypoints, projection, depth mask and compacted visible indices; L2 written (>= 2x L2) "
                        "before every iteration",
            "entry": "s4d_kps_project_linear (learnable_fc + keypoints + projection + masks, then the compaction)",
            "median_us": med_us, "p10_us": 1000 * ms[len(ms) // 10], "p90_us": 1000 * ms[(9 * len(ms)) // 10],
            "calls_per_s": 1e6 / med_us, "visible": int(cnt.item()), "launches_per_call": 2}


def pack_leg(device, frames=32, iters=10):
    """FPN outputs -> packed mc_ms_feat: 32 frames of NCHW fp32 maps (6 cams, 4 levels, 256 ch)
    transposed and cast to the packed bf16 layout (s4d_pack_feature_maps), timed with CUDA
    events; inputs (2.9 GB) are larger than L2."""
    from sparse4d_tt_b200 import ops
    from sparse4d_tt_b200 import synthetic as syn

    cfg = syn.DFAConfig(bs=frames)
    g = torch.Generator(device=device).manual_seed(5)
    maps = [torch.randn(frames, cfg.num_cams, cfg.embed_dims, h, w, generator=g, device=device)
            for h, w in cfg.spatial_shapes]
    out, _, _ = ops.pack_feature_maps(maps, dtype=torch.bfloat16)
    for _ in range(3):
        ops.pack_feature_maps(maps, dtype=torch.bfloat16, out=out)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        ops.pack_feature_maps(maps, dtype=torch.bfloat16, out=out)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / iters
    n = sum(m.numel() for m in maps)
    nbytes = n * (4 + 2)
    peak, src = measured_hbm()
    res = {"workload": f"{frames} frames x 6 cams x 4 levels x 256 ch, NCHW fp32 -> packed channels-last bf16",
           "ms": ms, "algorithmic_bytes": nbytes, "achieved_gbs": nbytes / ms / 1e6,
           "frac_of_hbm": nbytes / ms / 1e6 / peak, "peak_gbs": peak, "peak_source": src,
           "launches_per_call": len(maps)}
    del maps, out
    torch.cuda.empty_cache()
    return res


def bank_metas(frames, step):
    """Synthetic per-frame ego poses and timestamps of one step of the InstanceBank workload:
    frame f at time 0.5 * step, yawed and shifted a little more every step."""
    import numpy as np

    img = []
    for f in range(frames):
        yaw, sx, sy = 0.01 * (f + 3 * step), 0.4 * step + 0.01 * f, 0.1 * step
        c, s_ = np.cos(yaw), np.sin(yaw)
        tg = np.array([[c, -s_, 0, sx], [s_, c, 0, sy], [0, 0, 1, 0], [0, 0, 0, 1]], dtype=np.float64)
        img.append({"T_global": tg, "T_global_inv": np.linalg.inv(tg)})
    return {"timestamp": torch.full((frames,), 0.5 * step, dtype=torch.float64), "img_metas": img}


def bank_inputs(frames, seed=700):
    """The learnable anchors and features of the bank, and one set of decoder outputs (new
    features, anchors, class scores) per frame, seeded."""
    from sparse4d_tt_b200 import synthetic as syn

    g = torch.Generator().manual_seed(seed)
    anchor_data = syn.make_anchors(1, 900, g)[0]
    feat_data = torch.randn(900, 256, generator=g)
    new = (torch.randn(frames, 900, 256, generator=g), syn.make_anchors(frames, 900, g),
           torch.randn(frames, 900, 10, generator=g))
    return anchor_data, feat_data, new


def instance_bank_leg(device, frames, steps=40, warmup=3):
    """The temporal InstanceBank around the decoder (model/instance_bank.py get / update / cache)
    for a batch of ``frames`` frames: each step moves the 600 cached anchors to the frame (get),
    merges the top 300 of the 900 new instances with them (update) and keeps the 600 most
    confident for the next frame (cache), eagerly, with the host's per-frame pose products; CUDA
    events around the timed steps."""
    from sparse4d_tt_b200.instance_bank import InstanceBank

    anchor_data, feat_data, (nf, na, nc) = bank_inputs(frames)
    bank = InstanceBank(device, anchor_data, feat_data)
    nf, na, nc = nf.to(device), na.to(device), nc.to(device)

    metas = [bank_metas(frames, k) for k in range(warmup + 1 + steps)]  # the data loader's part

    def step(k):
        bank.get(frames, metas[k])
        f, a = bank.update(nf, na, nc)
        bank.cache(f, a, nc, metas[k])

    k = 0
    for _ in range(warmup + 1):
        step(k)
        k += 1
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        step(k)
        k += 1
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    return {"workload": f"InstanceBank get + update + cache over {frames} frames: 600 cached of 900 anchors, "
                        "256 ch, 10 classes; eager, per-frame ego poses from the host",
            "ms_per_step": ms, "frames_per_s": frames / (ms / 1e3), "steps": steps,
            "launches_per_step": 3}


def decoder_leg(device, frames, steps, warmup):
    """The decoder chain around the DFA: a whole single-frame Sparse4D v3 decoder pass (6 DFA
    layers with the decoupled attention, FFN, LayerNorm, refinement and anchor re-encoding
    between them, anchors kept on the device from layer to layer) over ``frames`` frames as one
    CUDA graph (head.HeadGraph), bf16 maps, the dense layers in TF32.  Seeded synthetic
    parameters (synthetic.make_head_params) and the bench's camera ring."""
    from sparse4d_tt_b200 import synthetic as syn
    from sparse4d_tt_b200.head import HeadGraph, Sparse4DHead

    cfg = syn.DFAConfig(bs=frames)

    def run(attention):
        head = Sparse4DHead(device, syn.make_head_params(cfg, torch.Generator().manual_seed(600)),
                            dict(MODEL_CONFIG, ATTENTION_DTYPE=attention))
        g = HeadGraph(head, frames, cfg.spatial_shapes)
        dgen = torch.Generator(device=device).manual_seed(601)
        g.mc_ms_feat.copy_(torch.randn(g.mc_ms_feat.shape, device=device, generator=dgen, dtype=torch.bfloat16))
        g.projection_mat.copy_(syn.camera_ring(6, cfg.image_wh)[None].expand(frames, -1, -1, -1))
        g.image_wh.copy_(torch.tensor(cfg.image_wh, dtype=torch.float32).expand(frames, 6, 2))
        for _ in range(warmup):
            g.replay()
        ms = time_steps(g.replay, steps, lambda: None)
        out = g.output
        moved = (out["prediction"][-1][..., :3] - g.anchor[..., :3]).norm(dim=-1).mean().item()
        del g, head
        torch.cuda.empty_cache()
        return ms, moved

    ms, moved = run(torch.float32)
    ms_bf, moved_bf = run(torch.bfloat16)
    return {"workload": f"single-frame Sparse4D v3 decoder pass over {frames} frames: 6 DFA layers + 11 decoupled "
                        "attentions, 6 FFNs, 12 LayerNorms, 6 refinements and 5 anchor re-encodings; 900 anchors, "
                        "704x256 bf16 maps; one CUDA graph per pass; attention in fp32",
            "ms_per_pass": ms / steps, "frames_per_s": frames * steps / (ms / 1e3),
            "dfa_calls_per_s": 6 * frames * steps / (ms / 1e3), "steps": steps,
            "mean_anchor_move_m": moved,
            "anchors": "refined on the device by each decoder's refinement and re-encoded for the next DFA layer",
            "attention_bf16": {"ms_per_pass": ms_bf / steps, "frames_per_s": frames * steps / (ms_bf / 1e3),
                               "mean_anchor_move_m": moved_bf,
                               "note": "the same pass with the attention's softmax(QK^T)V in bf16 (flash kernels; "
                                       "ATTENTION_DTYPE), as the reference's TT-NN attention"}}


HIGHRES_FRAMES = 16  # global batch of the high-resolution stress case


def highres_leg(rank, world, device, pg, steps, warmup):
    """High-resolution stress case: one DFA layer over a global batch of 16 frames of 1600x640
    images (maps 160x400, 80x200, 40x100, 20x50; 261 MB of bf16 maps per frame), 1800 anchors,
    run two ways on the N GPUs.

    * frame-sharded: each rank takes 16 / N frames, no collective (the layer as one CUDA graph,
      and launched eagerly); the gather's roofline as in the main line;
    * camera-sharded (N >= 2): ranks form a (N / 2 frame groups) x (2 camera halves) grid; the
      two ranks of a camera group take the same 16 / (N / 2) frames, each samples 3 of the 6
      cameras with the softmax over all 6, the fp32 partial sums meet by an NCCL
      reduce-scatter over the flattened (frame, anchor) rows, and each rank projects its half
      (launched eagerly).  Rank 0 checks its shard against the same layer on one GPU;
    * camera-sharded p2p (N >= 2): the same grid and rows with no collective kernel: each
      rank's gather writes the other rank's rows straight into that GPU's memory over NVLink,
      and after a bounded flag exchange output_proj adds the two partial sums in its
      accumulator; launched eagerly and as one CUDA graph.

    Every rank runs every step; the times are device times, max over ranks."""
    import torch.distributed as dist

    from sparse4d_tt_b200 import DeformableFeatureAggregation
    from sparse4d_tt_b200 import camera_shard as cs
    from sparse4d_tt_b200 import synthetic as syn

    def barrier():
        if pg is not None:
            pg.barrier()

    def max_ms(ms):
        t = torch.tensor([ms], device=device)
        if pg is not None:
            pg.all_reduce(t, op=pg.ReduceOp.MAX)
        return float(t.item())

    peak, src = measured_hbm()
    res = {"workload": f"1 DFA layer over {HIGHRES_FRAMES} frames (global) of 1600x640 images (maps 160x400, 80x200, "
                       "40x100, 20x50), 1800 anchors x 13 pts x 6 cams x 4 levels x 256 ch, bf16 maps",
           "global_frames": HIGHRES_FRAMES, "steps": steps}
    fpr = max(1, HIGHRES_FRAMES // world)
    w = Workload(fpr, 1, device, seed=3000 + rank, cfg=syn.config_highres(fpr, 1800))
    for _ in range(warmup):
        w.step()
    eager = max_ms(time_steps(w.step, steps, barrier))
    stack = w.graph_stack()
    for _ in range(warmup):
        stack.replay()
    graph = max_ms(time_steps(stack.replay, steps, barrier))
    g_ms = stack.gather_times_ms()[0]
    alg, touched, inb = w.algorithmic_bytes_per_layer()[0]
    calls = fpr * world * steps
    res["frame_sharded"] = {
        "frames_per_gpu": fpr, "value": calls / (graph / 1e3), "unit": UNIT, "ms_per_step": graph / steps,
        "eager": {"value": calls / (eager / 1e3), "ms_per_step": eager / steps},
        "collective": None,
        "roofline": {"kernel": "dfa_gather_warp_kernel<bf16> (keypoints + projection + gather), rank 0's launch",
                     "achieved": alg / (g_ms / 1e3) / 1e9, "peak": peak, "unit": "GB/s",
                     "frac": alg / (g_ms / 1e3) / 1e9 / peak, "peak_source": src, "algorithmic_bytes": alg,
                     "unique_tap_pixels": touched, "launch_us": g_ms * 1e3},
    }
    del stack, w
    torch.cuda.empty_cache()
    if world >= 2 and world % 2 == 0:
        fgroup, cgroup = cs.make_groups(world, 2)
        fpg = HIGHRES_FRAMES // (world // 2)
        rows = fpg * 1800
        modes = {
            "camera_sharded": ("reduce_scatter", {
                "collective": "reduce_scatter",
                "combine": "NCCL reduce-scatter of the fp32 partial sums over the flattened (frame, anchor) rows, "
                           "then output_proj on this rank's rows"}),
            "camera_sharded_p2p": ("p2p", {
                "collective": None,
                "combine": "no collective kernel: each rank's gather writes the other rank's rows of its partial "
                           "sums straight into that rank's memory over NVLink (CUDA IPC mapping) as it produces "
                           "them; after a bounded flag exchange, output_proj sums this rank's own and received "
                           "partial sums, both local, in the tensor-core accumulator (s4d_dfa_output_proj_sum)"}),
        }
        for key, (reduce, extra) in modes.items():
            mc = dict(MODEL_CONFIG, CAMERA_REDUCE=reduce)
            w = Workload(fpg, 1, device, seed=4000 + fgroup, cfg=syn.config_highres(fpg, 1800), mesh_device=cgroup,
                         model_config=mc)
            for _ in range(warmup):
                w.step()
            ms = max_ms(time_steps(w.step, steps, barrier))
            graph_ms = None
            if reduce == "p2p":  # no collective kernel in the call: it can be captured in a CUDA graph
                stack = w.graph_stack()
                for _ in range(warmup):
                    stack.replay()
                graph_ms = max_ms(time_steps(stack.replay, steps, barrier))
                del stack
            # parity: this rank's shard against the same layer on this GPU alone
            out = w.step()
            b, e = w.mods[0].shard
            single = DeformableFeatureAggregation(device, w.params[0], MODEL_CONFIG).run(
                w.inst0, w.anchors[0], w.embeds[0], w.packed, w.proj, w.wh, w.cfg.spatial_shapes, fpg, 1800)
            ref = single.reshape(-1, single.shape[-1])[b:e].double()
            got = out.double()
            err = float((got - ref).abs().max())
            pcc = float(torch.corrcoef(torch.stack([got.flatten(), ref.flatten()]))[0, 1])
            peer = w.mods[0]._peer
            flag = 0 if peer is None else int(peer.error_flag.item())
            stats = torch.tensor([err, -pcc, flag], device=device)
            if pg is not None:
                pg.all_reduce(stats, op=pg.ReduceOp.MAX)
            calls = fpg * (world // 2) * steps
            res[key] = {
                "grid": f"{world // 2} frame groups x 2 camera halves (3 cameras per rank)", "frames_per_group": fpg,
                "value": calls / (ms / 1e3), "unit": UNIT, "ms_per_step": ms / steps,
                **extra, "group_size": dist.get_world_size(cgroup),
                "bytes_to_peer_per_rank": rows // 2 * 256 * 4,
                "launch": "eager (DeformableFeatureAggregation.run per step)",
                "parity": {"max_abs_err": float(stats[0]), "pcc_min": -float(stats[1]),
                           "against": "the same layer on one GPU (all 6 cameras), each rank's rows of the output; "
                                      "max over ranks"},
            }
            if graph_ms is not None:
                res[key]["graph"] = {"value": calls / (graph_ms / 1e3), "ms_per_step": graph_ms / steps,
                                     "launch": "the layer as one CUDA graph (DFAStack) per step, both exchanges and "
                                               "output_proj_sum inside it"}
            if peer is not None:
                res[key]["peer_timeout_flag"] = int(stats[2])
                peer.close()
            del w, single
            torch.cuda.empty_cache()
    return res


def cpu_baseline(seconds=12.0, max_calls=40):
    """The oracle's torch port of the reference DFA layer on the host CPU (all threads), at the
    single-frame 900-anchor shape, fp32."""
    from oracle import dfa_torch as oto
    from sparse4d_tt_b200 import synthetic as syn

    threads = len(os.sched_getaffinity(0))
    torch.set_num_threads(threads)
    cfg = syn.config_standard(1)
    ins = syn.make_inputs(cfg, 0, feature_dtype=torch.bfloat16)
    params = syn.make_params(cfg, torch.Generator().manual_seed(100))

    def call():
        with torch.no_grad():
            oto.dfa_layer(params, ins.instance_feature, ins.anchor, ins.anchor_embed, ins.feature_maps,
                          ins.projection_mat, ins.image_wh)

    for _ in range(2):
        call()
    times = []
    t_end = time.perf_counter() + seconds
    while len(times) < max_calls and (time.perf_counter() < t_end or len(times) < 5):
        t0 = time.perf_counter()
        call()
        times.append(time.perf_counter() - t0)
    med = statistics.median(times)

    # keypoints only (kps_generator + project_points + mask + nonzero), the same frame
    def kps_call():
        with torch.no_grad():
            kp = oto.key_points(ins.anchor, ins.instance_feature, params)
            uv, depth = oto.project_points_with_depth(kp, ins.projection_mat, ins.image_wh)
            _, vis = oto.visibility(uv, depth)
            return oto.visible_indices(vis)

    for _ in range(3):
        kps_call()
    k_times = []
    for _ in range(50):
        t0 = time.perf_counter()
        kps_call()
        k_times.append(time.perf_counter() - t0)
    k_med = statistics.median(k_times)

    # the InstanceBank step of the GPU leg (32 frames) on the oracle's port of the reference class
    from oracle import instance_bank_torch as oib

    anchor_data, feat_data, (nf, na, nc) = bank_inputs(32)
    bank = oib.InstanceBankOracle(anchor_data, feat_data)
    b_times = []
    metas = [bank_metas(32, k) for k in range(6)]
    for k in range(6):
        t0 = time.perf_counter()
        with torch.no_grad():
            bank.get(32, metas[k])
            f, a = bank.update(nf, na, nc)
            bank.cache(f, a, nc, metas[k])
        b_times.append(time.perf_counter() - t0)
    b_med = statistics.median(b_times[2:])
    return {"value": 1.0 / med, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"{len(times)} single-frame DFA layer calls (900 anchors, 704x256 maps as fp32, all linears "
                      f"included) after 2 warm-ups; median {med * 1e3:.1f} ms/call; torch {torch.__version__} CPU",
            "median_ms": med * 1e3, "cpu": _cpu_model(),
            "kps": {"median_ms": k_med * 1e3, "calls_per_s": 1.0 / k_med,
                    "sample": "50 keypoint-only calls (1 frame, 900 anchors, learnable_fc included) after 3 warm-ups"},
            "instance_bank": {"median_ms": b_med * 1e3, "frames_per_s": 32 / b_med,
                              "sample": "4 InstanceBank get + update + cache steps over 32 frames (the GPU leg's "
                                        "workload) after 2, on the oracle's port of the reference class"}}


def _cpu_model():
    try:
        with open("/proc/cpuinfo") as f:
            for ln in f:
                if ln.startswith("model name"):
                    return ln.split(":", 1)[1].strip()
    except Exception:
        pass
    return "unknown"


GATHER_SOURCES = ("dfa_gather.cu", "kps_math.cuh", "common.cuh")


def gather_source_sha16():
    """First 16 hex digits of the SHA-256 of the gather kernel's sources (the files the
    dfa_gather_warp_kernel is compiled from), which ties an ncu capture to the code it measured."""
    import hashlib

    h = hashlib.sha256()
    for name in GATHER_SOURCES:
        with open(os.path.join(REPO, "sparse4d-tt_b200", "csrc", name), "rb") as f:
            h.update(f.read())
    return h.hexdigest()[:16]


def read_profile_traffic():
    """(DRAM bytes, algorithmic bytes) of one captured gather launch from the committed ncu
    summary, or None when there is none or it was captured from other kernel sources than the
    ones built now (its ``kernel_source_sha16`` line differs from ``gather_source_sha16()``)."""
    path = os.path.join(REPO, "profiles", "dfa_gather_stacked_bs32.md")
    vals = {}
    try:
        with open(path) as f:
            for ln in f:
                for key in ("traffic_bytes_per_launch", "algorithmic_bytes_same_launch", "kernel_source_sha16"):
                    if ln.startswith(key + ":"):
                        vals[key] = ln.split(":", 1)[1].strip()
    except Exception:
        return None
    if len(vals) != 3 or vals["kernel_source_sha16"] != gather_source_sha16():
        return None
    return float(vals["traffic_bytes_per_launch"]), float(vals["algorithmic_bytes_same_launch"])


# ---------------------------------------------------------------------------------------------
# arms
# ---------------------------------------------------------------------------------------------
def run_reference(args):
    rank, world, _ = env_dist()
    if rank != 0:
        return
    res = cpu_baseline_steps(args.steps, args.warmup)
    cfg = workload_config(args.frames, args.layers, world)
    # The same workload, sampled: a step here is ONE DFA call of it (1 frame through 1 layer),
    # so DFA calls/s is per call on both arms.
    cfg["reference_step"] = ("1 frame through 1 DFA layer of this workload per step (bounded CPU sample); the "
                             "oracle's fp32 arithmetic on the same bf16-valued maps upcast to fp32, all linears "
                             "in fp32")
    line = {
        "impl": "reference", "metric": METRIC, "value": res["value"], "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": res["ms_per_step"], "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded camera ring, Xavier init)",
        "config": cfg,
        "cpu_baseline": {"value": res["value"], "unit": UNIT, "cores": res["cores"], "kind": "port",
                         "sample": res["sample"]},
        "e2e": {"value": res["value"], "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def cpu_baseline_steps(steps, warmup):
    from oracle import dfa_torch as oto
    from sparse4d_tt_b200 import synthetic as syn

    threads = len(os.sched_getaffinity(0))
    torch.set_num_threads(threads)
    cfg = syn.config_standard(1)
    ins = syn.make_inputs(cfg, 0, feature_dtype=torch.bfloat16)
    params = syn.make_params(cfg, torch.Generator().manual_seed(100))

    def call():
        with torch.no_grad():
            oto.dfa_layer(params, ins.instance_feature, ins.anchor, ins.anchor_embed, ins.feature_maps,
                          ins.projection_mat, ins.image_wh)

    for _ in range(warmup):
        call()
    t0 = time.perf_counter()
    for _ in range(steps):
        call()
    dt = time.perf_counter() - t0
    return {"value": steps / dt, "ms_per_step": dt / steps * 1e3, "cores": threads,
            "sample": f"each step = 1 single-frame DFA layer call (900 anchors, 704x256 maps as fp32) of the "
                      f"workload, oracle torch port of the reference DFA on {threads} host threads "
                      f"({_cpu_model()})"}


def run_ours(args):
    rank, world, local_rank = env_dist()
    if not torch.cuda.is_available():
        raise SystemExit("bench.py: no CUDA device")
    device = torch.device(f"cuda:{local_rank}")
    torch.cuda.set_device(device)
    pg = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        # NCCL prints its version banner on the process's stdout; keep stdout for the JSON
        # line by pointing fd 1 at stderr while the communicator is created and first used.
        sys.stdout.flush()
        saved = os.dup(1)
        os.dup2(2, 1)
        try:
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)
            dist.barrier()
            torch.cuda.synchronize()
        finally:
            sys.stdout.flush()
            os.dup2(saved, 1)
            os.close(saved)
        pg = dist

    def barrier():
        if pg is not None:
            pg.barrier()

    w = Workload(args.frames, args.layers, device, seed=1 + rank)
    for _ in range(args.warmup):
        w.step()
    torch.cuda.synchronize()
    bytes_per_layer = w.algorithmic_bytes_per_layer()
    # the same step launched eagerly, layer by layer (host launch cost included), timed before
    # any graph exists
    for _ in range(args.warmup):
        w.step()
    eager_ms = time_steps(w.step, args.steps, barrier)
    stack = w.graph_stack()
    for _ in range(args.warmup):
        stack.replay()
    torch.cuda.synchronize()

    # the timed step: one replay of the 6-layer graph (every kernel of every layer runs)
    clocks = ClockSampler(device)
    ms = time_steps(stack.replay, args.steps, barrier)
    clock_info = clocks.stop()
    g_ms = stack.gather_times_ms()  # the gather launches of the last timed replay

    t = torch.tensor([ms, eager_ms], device=device)
    if pg is not None:
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
    ms_max, eager_ms = (float(x) for x in t.tolist())
    calls = args.frames * args.layers * args.steps * world
    value = calls / (ms_max / 1e3)

    e2e = None
    if not args.no_e2e:
        e_steps = max(3, args.steps // 4)
        e_ms, h2d, d2h, h2d_gbs = e2e_leg(w, e_steps, 2, barrier)
        te = torch.tensor([e_ms], device=device)
        if pg is not None:
            pg.all_reduce(te, op=pg.ReduceOp.MAX)
        e_ms_max = float(te.item())
        # per-rank host-to-device rates, gathered to rank 0
        rates = torch.tensor([h2d / (e_ms / e_steps) / 1e6, h2d_gbs], device=device)
        if pg is not None:
            allr = [torch.zeros_like(rates) for _ in range(world)]
            pg.all_gather(allr, rates)
            rates_all = [r.tolist() for r in allr]
        else:
            rates_all = [rates.tolist()]
        floor_ms = h2d / (h2d_gbs * 1e6)
        e2e = {"value": args.frames * args.layers * e_steps * world / (e_ms_max / 1e3), "unit": UNIT,
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "steps": e_steps,
               "ms_per_step": e_ms_max / e_steps,
               "h2d_gbs_per_rank": [round(r[0], 2) for r in rates_all],
               "h2d_copy_gbs_per_rank": [round(r[1], 2) for r in rates_all],
               "h2d_floor_ms": floor_ms, "frac_of_h2d_floor": floor_ms / (e_ms_max / e_steps),
               "gpu_numa_node": gpu_numa_node(device),
               "path": "PipelinedDFAStack.submit (two 6-layer CUDA graphs; step k+1's uploads on a copy stream "
                       "overlap step k's replay), inputs from pinned host memory, output read back each step",
               "floor": "h2d bytes / the plain pinned host-to-device copy rate of the maps measured on this rank"}

    highres = None
    if not args.no_highres:
        highres = highres_leg(rank, world, device, pg, min(args.steps, 20), 3)

    bs1 = pack = kps = decoder = bank = None
    if rank == 0 and not args.no_bs1:
        bs1 = bs1_leg(device)
        pack = pack_leg(device)
        kps = kps_leg(device)
        bank = instance_bank_leg(device, args.frames)
        decoder = decoder_leg(device, args.frames, max(3, args.steps // 4), 2)
    barrier()

    if rank == 0:
        peak, src = measured_hbm()
        alg = statistics.mean(b for b, _, _ in bytes_per_layer)
        inb_per_call = statistics.mean(n for _, _, n in bytes_per_layer) / args.frames
        g_avg_ms = statistics.mean(g_ms)
        achieved = alg / (g_avg_ms / 1e3) / 1e9
        prof = read_profile_traffic()
        # the captured launch is layer 0; scale its DRAM bytes to the average launch by the
        # algorithmic bytes (both are proportional to the touched feature rows)
        traffic = prof[0] / prof[1] * alg if prof else None
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_max / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded camera ring, Xavier init)",
            "config": workload_config(args.frames, args.layers, world),
            "keypoint_samples_per_s": value * SAMPLES_PER_CALL,
            "inbounds_samples_per_s": value * inb_per_call,
            "inbounds_samples_per_call": inb_per_call,
            "roofline": {
                "kernel": "dfa_gather_warp_kernel<bf16> (keypoints + projection + gather)", "bound": "hbm", "achieved": achieved, "peak": peak,
                "unit": "GB/s", "frac": achieved / peak, "peak_source": f"{src} (MEASURED_PEAKS.json hbm_gbs)",
                "traffic": traffic,
                "traffic_source": ("ncu dram__bytes_read+write of the layer-0 launch (profiles/dfa_gather_stacked_bs32.md, "
                                   "captured from these kernel sources), scaled to the average launch by algorithmic "
                                   "bytes") if prof else
                                  "none: no ncu capture of the current kernel sources is committed",
                "kernel_source_sha16": gather_source_sha16(),
                "algorithmic_bytes_per_launch": alg,
                "unique_tap_pixels_per_launch": statistics.mean(t for _, t, _ in bytes_per_layer),
                "avg_launch_us": g_avg_ms * 1e3, "launches_timed": len(g_ms),
                "launch_timing": "CUDA events of the graph's event-record nodes around each layer's gather, "
                                 "last replay of the timed region",
                "share_of_step": sum(g_ms) / (ms / args.steps),
                # the L2-side tap traffic (not the roofline numerator): 4 taps x 512 B per
                # in-bounds sample, over the same average launch time
                "tap_bytes_per_launch": inb_per_call * args.frames * 4 * 512,
                "tap_gbs": inb_per_call * args.frames * 4 * 512 / (g_avg_ms / 1e3) / 1e9,
            },
            "gpu_launches": launches_per_layer(w) * args.layers * args.steps,
            "step": "one replay of the 6-layer DFAStack CUDA graph per step",
            "eager": {"ms_per_step": eager_ms / args.steps,
                      "value": args.frames * args.layers * args.steps * world / (eager_ms / 1e3),
                      "path": "DeformableFeatureAggregation.run per layer, launched from the host each step"},
            "clocks": clock_info,
            "e2e": e2e,
            "bs1": bs1,
            "pack": pack,
            "kps": kps,
            "highres": highres,
            "decoder": decoder,
            "instance_bank": bank,
        }
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline()
        print(json.dumps(line), flush=True)
    if pg is not None:
        pg.barrier()
        pg.destroy_process_group()


def run_profile_case(args):
    """A small, quiet case for ncu: the layer of bench.py's workload, run twice."""
    device = torch.device("cuda:0")
    torch.cuda.set_device(device)
    w = Workload(args.frames, 1, device, seed=1)
    w.step()
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_push("profile")
    w.step()
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    print(json.dumps({"profile_case": f"1 DFA layer x {args.frames} frames", "ok": True}), flush=True)


def main():
    args = parse_args()
    if args.profile_gather:
        run_profile_case(args)
        return
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
