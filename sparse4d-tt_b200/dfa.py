"""Drop-in ``DeformableFeatureAggregation`` for Sparse4D v3 on B200.

Same constructor arguments, parameter-dictionary keys and ``run`` signature as the reference
module (``model/deformable_feature_aggregation.py:42-57,800-811,954-995``), called the same
way by the decoder head (``model/sparse4d_head.py:405-411``).  What runs:

* the camera encoder and the per-camera term of the weight logits
  (``model/deformable_feature_aggregation.py:679-717``) on this library's fp32 kernels (with
  split logits, the default);
* ``weights_fc`` + the keypoint ``learnable_fc`` and ``output_proj`` (``:934-950``) on this
  library's tcgen05 kernels with ``MATMUL_PRECISION "tf32"``, on cuBLAS fp32 through torch with
  ``"fp32"`` (the default);
* kernel (a) ``s4d_kps_project`` replaces ``_kps_generator_pre_rotation`` +
  ``ttnn.kps_project_fused`` (``:651-677,855-860``); with the tcgen05 linears the gather
  computes the keypoints itself;
* kernel (b)+(c) ``s4d_deformable_aggregation`` replaces the softmax, the per-level
  ``ttnn.grid_sample`` + ``ttnn.transposed_s2i`` loop and ``ttnn.grouped_weighted_sum``
  (``:791-796,864-899``).

Camera sharding (the reference's ``mesh_device`` mode, ``:172-176,925-931``) is available by
passing a ``torch.distributed`` process group as ``mesh_device``: each rank samples only its
own cameras, with the softmax taken over ALL cameras (the reference softmaxes over each
device's cameras only; see ``camera_shard``).  ``model_config["CAMERA_REDUCE"]`` chooses how
the fp32 partial sums meet: ``"all_reduce"`` (default; every rank returns all ``[bs, A, 2C]``,
as the reference's ``ttnn.all_reduce``), ``"reduce_scatter"`` (NCCL reduce-scatter over the
flattened ``(frame, anchor)`` rows; the rank runs ``output_proj`` on its shard only and
returns ``[bs * A / n, 2C]``, rows ``self.shard`` of the flattened output) or ``"p2p"`` (groups
of 2 GPUs: the same shards with no collective kernel -- ``output_proj`` reads the other GPU's
partial sums over NVLink and adds them in its accumulator; see ``camera_shard``).
"""
from __future__ import annotations

import contextlib
from typing import Dict, List, Optional, Sequence, Tuple, Union

import torch
import torch.nn.functional as F

from . import ops
from .timing import TimingEvent

Tensor = torch.Tensor

X, Y, Z = 0, 1, 2
W, L, H = 3, 4, 5
SIN_YAW, COS_YAW = 6, 7

PARAM_KEYS = (
    "kps_fix_scale", "kps_learnable_fc_weight", "kps_learnable_fc_bias",
    "cam_linear1_weight", "cam_linear1_bias", "cam_ln1_weight", "cam_ln1_bias",
    "cam_linear2_weight", "cam_linear2_bias", "cam_ln2_weight", "cam_ln2_bias",
    "weights_fc_weight", "weights_fc_bias", "output_proj_weight", "output_proj_bias",
)


def preprocess_dfa_parameters(pt_model) -> Dict[str, Tensor]:
    """Parameter dictionary of a PyTorch DFA module, keyed as
    ``model/deformable_feature_aggregation.py:954-995`` keys it (works for the mmdet3d
    module and for the reference's standalone ``_PTDeformableFeatureAggregation``)."""
    p = {
        "kps_fix_scale": pt_model.kps_generator.fix_scale.data.clone(),
        "kps_learnable_fc_weight": pt_model.kps_generator.learnable_fc.weight.data.clone(),
        "kps_learnable_fc_bias": pt_model.kps_generator.learnable_fc.bias.data.clone(),
    }
    if getattr(pt_model, "camera_encoder", None) is not None:
        enc = pt_model.camera_encoder
        for idx, key in ((0, "cam_linear1"), (2, "cam_ln1"), (3, "cam_linear2"), (5, "cam_ln2")):
            p[key + "_weight"] = enc[idx].weight.data.clone()
            p[key + "_bias"] = enc[idx].bias.data.clone()
    p["weights_fc_weight"] = pt_model.weights_fc.weight.data.clone()
    p["weights_fc_bias"] = pt_model.weights_fc.bias.data.clone()
    p["output_proj_weight"] = pt_model.output_proj.weight.data.clone()
    p["output_proj_bias"] = pt_model.output_proj.bias.data.clone()
    return p


FeatureMaps = Union[List[Tensor], Tuple[Tensor, Tensor, Tensor]]

MATMUL_PRECISIONS = {"fp32": "highest", "tf32": "high"}
CAMERA_REDUCES = ("all_reduce", "reduce_scatter", "p2p")


@contextlib.contextmanager
def _matmul_precision(precision: str):
    """torch's fp32 matmul precision for the duration of the block ("highest": fp32 GEMMs;
    "high": TF32 tensor-core GEMMs with fp32 accumulation), restored afterwards."""
    old = torch.get_float32_matmul_precision()
    if old == precision:
        yield
        return
    torch.set_float32_matmul_precision(precision)
    try:
        yield
    finally:
        torch.set_float32_matmul_precision(old)


class DeformableFeatureAggregation:
    """B200 DFA layer.  ``device`` is a CUDA device (``"cuda:0"``, ``torch.device`` or index).

    ``model_config`` may carry ``"FEATURE_DTYPE"`` (``torch.bfloat16`` default, or
    ``torch.float32``): the dtype feature maps are packed to when ``run`` receives a list; and
    ``"MATMUL_PRECISION"``: ``"fp32"`` (default, cuBLAS fp32 GEMMs) or ``"tf32"`` for the
    layer's linears: TF32 operands, fp32 accumulation (the reference's TT path runs them in
    bf16).  With ``"tf32"`` and split logits they run on this library's tcgen05 kernels
    (``ops.weights_fc_into`` / ``ops.output_proj_into``), the embed add and the residual fused.
    ``split_logits=True`` (default) evaluates ``weights_fc(f + cam) = weights_fc(f) + W cam``
    as two smaller GEMMs (Ncam times fewer FLOPs) and combines the two terms inside the gather
    kernel instead of materialising the ``[bs, A, Ncam, L*P*G]`` logits (same result up to
    fp32 rounding); ``split_logits=False`` evaluates the linear exactly as the reference does."""

    # Up to this many frames per call the per-frame camera terms (encoder, per-camera logits,
    # softmax factors) run as one cluster launch; above it as three shorter launches, whose
    # short-lived CTAs leave room sooner for the concurrent tensor-core weights_fc.
    camera_terms_max_frames = 8

    def __init__(self, device, parameters: Dict[str, Tensor], model_config: Optional[Dict] = None,
                 embed_dims: int = 256, num_groups: int = 8, num_levels: int = 4, num_cams: int = 6,
                 num_pts: int = 13, num_learnable_pts: int = 6, use_camera_embed: bool = True,
                 residual_mode: str = "cat", mesh_device=None, split_logits: bool = True) -> None:
        self.device = torch.device(device if not isinstance(device, int) else f"cuda:{device}")
        if self.device.type != "cuda":
            raise ValueError("DeformableFeatureAggregation runs on a CUDA device only")
        self.embed_dims = embed_dims
        self.num_groups = num_groups
        self.group_dims = embed_dims // num_groups
        self.num_levels = num_levels
        self.num_cams = num_cams
        self.num_pts = num_pts
        self.num_learnable_pts = num_learnable_pts
        self.use_camera_embed = use_camera_embed
        self.residual_mode = residual_mode
        self.model_config = dict(model_config or {})
        self.feature_dtype = self.model_config.get("FEATURE_DTYPE", torch.bfloat16)
        prec = self.model_config.get("MATMUL_PRECISION", "fp32")
        if prec not in MATMUL_PRECISIONS:
            raise ValueError(f"MATMUL_PRECISION must be one of {sorted(MATMUL_PRECISIONS)}")
        self.matmul_precision = MATMUL_PRECISIONS[prec]
        self.split_logits = bool(split_logits and use_camera_embed and num_cams <= 8 and embed_dims == 256)
        self.process_group = mesh_device if _is_process_group(mesh_device) else None
        if mesh_device is not None and self.process_group is None:
            raise ValueError("mesh_device must be a torch.distributed ProcessGroup (camera sharding)")
        self.camera_reduce = self.model_config.get("CAMERA_REDUCE", "all_reduce")
        if self.camera_reduce not in CAMERA_REDUCES:
            raise ValueError(f"CAMERA_REDUCE must be one of {CAMERA_REDUCES}")
        # (begin, end) of the flattened (frame, anchor) rows the last run() returned
        self.shard: Optional[Tuple[int, int]] = None
        missing = [k for k in PARAM_KEYS if k not in parameters and (use_camera_embed or not k.startswith("cam_"))]
        if missing:
            raise KeyError(f"parameters missing {missing}")
        dev = self.device

        def t(k):
            return parameters[k].detach().to(dev, torch.float32).contiguous()

        self.fix_scale = t("kps_fix_scale")
        if self.fix_scale.shape[0] + num_learnable_pts != num_pts:
            raise ValueError("num_pts must equal len(kps_fix_scale) + num_learnable_pts")
        self.learnable_fc_weight = t("kps_learnable_fc_weight")
        self.learnable_fc_bias = t("kps_learnable_fc_bias")
        if use_camera_embed:
            self.cam_linear1_weight, self.cam_linear1_bias = t("cam_linear1_weight"), t("cam_linear1_bias")
            self.cam_ln1_weight, self.cam_ln1_bias = t("cam_ln1_weight"), t("cam_ln1_bias")
            self.cam_linear2_weight, self.cam_linear2_bias = t("cam_linear2_weight"), t("cam_linear2_bias")
            self.cam_ln2_weight, self.cam_ln2_bias = t("cam_ln2_weight"), t("cam_ln2_bias")
        self.weights_fc_weight = t("weights_fc_weight")
        self.weights_fc_bias = t("weights_fc_bias")
        self.output_proj_weight = t("output_proj_weight")
        self.output_proj_bias = t("output_proj_bias")
        # TF32 linears run on this library's tensor-core kernels: weights_fc + learnable_fc
        # in one pass (embed add fused) and output_proj with the residual fused.
        lpg = num_levels * num_pts * num_groups
        self._tc = (self.matmul_precision == "high" and self.split_logits
                    and ops.weights_fc_supported(lpg, 3 * num_learnable_pts, embed_dims)
                    and residual_mode in ops.RESIDUAL_MODES
                    and 1024 // (num_cams * num_pts) + 2 <= 20 and num_learnable_pts <= 10)
        # Per-frame caches, cleared by the head at the start of a frame
        # (model/sparse4d_head.py:290-296 resets the same attribute names).
        self._cached_camera_embed = None
        self._cached_camera_logits = None
        self._cached_camera_ws = None
        self._cached_camera_factors = None
        # the Sparse4D v3 shape has a kernel for the per-frame camera softmax factors
        self._factors_ok = (num_cams, num_levels, num_pts, num_groups) == (6, 4, 13, 8)
        # ... and for the gather that computes its own sample locations from the anchors
        # (s4d_deformable_aggregation_anchors): no keypoint launch, no location buffer.
        self.fused_keypoints = self._tc and self._factors_ok and num_learnable_pts > 0
        if self.camera_reduce == "p2p" and self.process_group is not None:
            import torch.distributed as dist

            if dist.get_world_size(self.process_group) != 2 or not self._tc or not self.fused_keypoints:
                raise ValueError("CAMERA_REDUCE='p2p' needs a camera group of 2 ranks, the tensor-core linears "
                                 "(MATMUL_PRECISION 'tf32', residual_mode 'cat', 'add' or 'none') and the gather "
                                 "from anchors (6 cameras, 4 levels, 13 points, 8 groups, learnable keypoints)")
        self._peer = None  # camera_shard.PeerPartialSums of the p2p mode, made at the first run
        self._side: Optional[torch.cuda.Stream] = None
        self._side_kps: Optional[torch.cuda.Stream] = None
        self._side_pending = False
        self._cached_proj_rm = None
        self._cached_wh_rm = None
        self._cam_key = None
        # When a list, every run() appends a (start, end) pair of timing events recorded on the
        # launching stream around the gather kernel (used to time that kernel in place); under
        # stream capture the two records are event-record nodes of the graph.
        self.event_log: Optional[List[Tuple[TimingEvent, TimingEvent]]] = None
        self._timing: Optional[torch.cuda.Stream] = None
        self._timing_pending = False
        # The layer that runs after this one on the same frames (set for the length of a forward
        # by DFAStack, the head and graph.chained_camera_terms): its per-frame
        # camera terms depend only on projection_mat, so run() starts them on that layer's side
        # stream just before this layer's gather, where they fill the SMs the gather's last
        # anchors leave idle instead of sharing them with the next layer's weights_fc.
        self.next_layer: Optional["DeformableFeatureAggregation"] = None

    # ---- dense parts (cuBLAS through torch) -----------------------------------------------
    def _camera_encoder(self, projection_mat: Tensor, bs: int) -> Tensor:
        """``[bs, Ncam, C]`` (``model/deformable_feature_aggregation.py:679-717``)."""
        x = projection_mat[:, :, :3].reshape(bs, self.num_cams, 12)
        C = self.embed_dims
        x = F.relu(F.linear(x, self.cam_linear1_weight, self.cam_linear1_bias))
        x = F.layer_norm(x, (C,), self.cam_ln1_weight, self.cam_ln1_bias, 1e-5)
        x = F.relu(F.linear(x, self.cam_linear2_weight, self.cam_linear2_bias))
        return F.layer_norm(x, (C,), self.cam_ln2_weight, self.cam_ln2_bias, 1e-5)

    def _camera_embed(self, projection_mat: Tensor, bs: int) -> Tensor:
        """Camera embedding, cached per frame like the reference's ``_cached_camera_embed``
        (``model/deformable_feature_aggregation.py:741-747``, cleared per frame by the head,
        ``model/sparse4d_head.py:290-296``), and re-computed when the projection tensor changes."""
        key = (projection_mat.data_ptr(), projection_mat._version, tuple(projection_mat.shape))
        if self._cached_camera_embed is None or self._cam_key != key:
            self._cached_camera_embed = self._camera_encoder(projection_mat, bs)
            self._cached_camera_logits = None
            self._cam_key = key
        return self._cached_camera_embed

    def _camera_logits(self, projection_mat: Tensor, bs: int, side: bool = False) -> Tensor:
        """Per-camera term of the split logits, ``weights_fc(camera_embed)`` with the bias:
        ``[bs, Ncam, L, P, G]``, cached per frame.  For the Sparse4D v3 shape and at most
        ``camera_terms_max_frames`` frames one launch computes the camera encoder, this term and
        the gather's per-frame softmax factors (``ops.camera_terms_into``); otherwise two kernels
        compute the encoder and this term (``ops.camera_logits_into``), followed for the v3 shape
        by the factor kernel.  With ``side=True`` they run on this
        module's side stream, forked from the current stream, so that they overlap the
        per-anchor work; ``_join_side()`` makes the current stream wait for them.  Their
        outputs and workspace stay in the per-frame cache, so no buffer the side stream writes
        is handed back to the allocator before the join."""
        key = (projection_mat.data_ptr(), projection_mat._version, tuple(projection_mat.shape))
        if self._cached_camera_logits is None or self._cam_key != key:
            lpg = (self.num_levels, self.num_pts, self.num_groups)
            wc = torch.empty(bs, self.num_cams, *lpg, device=self.device)
            emb = torch.empty(bs, self.num_cams, self.embed_dims, device=self.device)
            one_launch = self._factors_ok and bs <= self.camera_terms_max_frames
            ws = None if one_launch else torch.empty(bs * self.num_cams * self.embed_dims, device=self.device)
            ctx = contextlib.nullcontext()
            if side:
                if self._side is None:
                    self._side = torch.cuda.Stream(self.device)
                self._side.wait_stream(torch.cuda.current_stream(self.device))
                ctx = torch.cuda.stream(self._side)
                self._side_pending = True
            factors = None
            if self._factors_ok:
                factors = ops.dfa_workspace(bs, self.num_cams, self.num_levels, self.num_pts, self.num_groups,
                                            self.device)
            with ctx:
                if one_launch:  # with the softmax's per-frame camera factors, one launch
                    ops.camera_terms_into(wc, projection_mat, self.cam_linear1_weight, self.cam_linear1_bias,
                                          self.cam_ln1_weight, self.cam_ln1_bias, self.cam_linear2_weight,
                                          self.cam_linear2_bias, self.cam_ln2_weight, self.cam_ln2_bias,
                                          self.weights_fc_weight, self.weights_fc_bias, camera_embed=emb,
                                          factors=factors)
                else:
                    ops.camera_logits_into(wc, projection_mat, self.cam_linear1_weight, self.cam_linear1_bias,
                                           self.cam_ln1_weight, self.cam_ln1_bias, self.cam_linear2_weight,
                                           self.cam_linear2_bias, self.cam_ln2_weight, self.cam_ln2_bias,
                                           self.weights_fc_weight, self.weights_fc_bias, camera_embed=emb,
                                           workspace=ws)
                    if factors is not None:  # the softmax's per-frame camera factors, off the gather's path
                        ops.camera_factors_into(factors, wc)
            self._cached_camera_embed, self._cached_camera_logits, self._cam_key = emb, wc, key
            self._cached_camera_ws, self._cached_camera_factors = ws, factors
        return self._cached_camera_logits

    def _join_side(self) -> None:
        if self._side_pending:
            torch.cuda.current_stream(self.device).wait_stream(self._side)
            self._side_pending = False

    def join_timing_stream(self) -> None:
        """Makes the current stream wait for the gather-timing branch of the last call (needed
        before the end of a stream capture that logged events)."""
        if self._timing_pending:
            torch.cuda.current_stream(self.device).wait_stream(self._timing)
            self._timing_pending = False

    def reset_frame_cache(self) -> None:
        """Drops the per-frame camera caches (what the head does at the start of every frame)."""
        self._cached_camera_embed = None
        self._cached_camera_logits = None
        self._cached_camera_factors = None
        self._cam_key = None

    def _get_weights(self, instance_feature: Tensor, anchor_embed: Tensor, projection_mat: Tensor, bs: int,
                     num_anchor: int):
        """Weight logits: ``[bs, A, Ncam, L, P, G]``, or with ``split_logits`` the pair
        (``[bs, A, L, P, G]``, ``[bs, Ncam, L, P, G]``) whose sum is the same logit
        (``model/deformable_feature_aggregation.py:719-798`` before its softmax)."""
        feature = instance_feature + anchor_embed
        lpg = (self.num_levels, self.num_pts, self.num_groups)
        if not self.use_camera_embed:
            w = F.linear(feature, self.weights_fc_weight, self.weights_fc_bias)
            return w.reshape(bs, num_anchor, self.num_cams, *lpg), None
        if self.split_logits:
            wa = F.linear(feature, self.weights_fc_weight).reshape(bs, num_anchor, *lpg)
            return wa, self._camera_logits(projection_mat, bs)
        cam = self._camera_embed(projection_mat, bs)
        w = F.linear(feature[:, :, None] + cam[:, None], self.weights_fc_weight, self.weights_fc_bias)
        return w.reshape(bs, num_anchor, self.num_cams, *lpg), None

    # ---- features ---------------------------------------------------------------------------
    def _features(self, feature_maps: FeatureMaps, spatial_shapes, bs: int):
        if isinstance(feature_maps, (tuple, list)) and len(feature_maps) == 3 and feature_maps[1].dtype == torch.int32 \
                and feature_maps[1].dim() == 3:
            return feature_maps  # already packed (mc_ms_feat, spatial_shape, scale_start_index)
        maps = list(feature_maps)
        if maps[0].dim() == 5:  # [bs, Ncam, C, H, W]
            return ops.pack_feature_maps(maps, dtype=self.feature_dtype)
        # reference TT layout: per level [1, 1, bs*Ncam*H*W, C] channels-last
        cl = [m.reshape(bs, self.num_cams, h, w, self.embed_dims) for m, (h, w) in zip(maps, spatial_shapes)]
        return ops.pack_feature_maps(cl, dtype=self.feature_dtype, channels_last=True)

    # ---- forward ----------------------------------------------------------------------------
    def run(self, instance_feature: Tensor, anchor: Tensor, anchor_embed: Tensor, feature_maps: FeatureMaps,
            projection_mat: Tensor, image_wh: Tensor, spatial_shapes: Sequence[Tuple[int, int]], bs: int,
            num_anchor: int) -> Tensor:
        """``[bs, A, 2C]`` (residual ``cat``) or ``[bs, A, C]`` (``add``), fp32."""
        dev = self.device
        instance_feature = instance_feature.reshape(bs, num_anchor, self.embed_dims)
        anchor = anchor.reshape(bs, num_anchor, -1).float().contiguous()
        anchor_embed = anchor_embed.reshape(bs, num_anchor, self.embed_dims)
        projection_mat = projection_mat.reshape(bs, self.num_cams, 4, 4).float().contiguous()
        image_wh = image_wh.reshape(bs, self.num_cams, 2).float().contiguous()
        mc_ms_feat, spatial_shape, scale_start = self._features(feature_maps, spatial_shapes, bs)

        C = self.embed_dims
        rows = bs * num_anchor
        if self._tc:
            # On a side stream the camera terms overlap the next two kernels; that pays while the
            # GPU is the bottleneck (graph capture, large batches), not for small eager calls, whose
            # time is host work that the extra stream bookkeeping would lengthen.
            capturing = torch.cuda.is_current_stream_capturing()
            side = rows >= 8192 or capturing
            logits_cam = self._camera_logits(projection_mat, bs, side=side)
            inst2d, embed2d = ops.row_view(instance_feature, C), ops.row_view(anchor_embed, C)
            logits = torch.empty(bs, num_anchor, self.num_levels, self.num_pts, self.num_groups, device=dev)
            if self.fused_keypoints:
                # The gather computes the sample locations itself from the anchors (no keypoint
                # launch, no location buffer); the tensor-core pass supplies the learnable
                # keypoint logits (one N-32 MMA per K step).
                learn = torch.empty(bs, num_anchor, 3 * self.num_learnable_pts, device=dev)
                ops.weights_fc_into(logits.view(rows, -1), learn.view(rows, -1), inst2d, embed2d,
                                    self.weights_fc_weight, self.learnable_fc_weight, self.learnable_fc_bias)
                loc = None
            elif rows <= 4096:
                loc = torch.empty(bs, num_anchor, self.num_cams, self.num_pts, 2, dtype=torch.float32, device=dev)
                # Small batches are latency-bound: the keypoints compute their own learnable logits
                # and, under capture, run on a second side stream beside weights_fc (and the camera
                # terms) instead of after it.
                ctx = contextlib.nullcontext()
                if capturing:
                    if self._side_kps is None:
                        self._side_kps = torch.cuda.Stream(dev)
                    self._side_kps.wait_stream(torch.cuda.current_stream(dev))
                    ctx = torch.cuda.stream(self._side_kps)
                with ctx:
                    ops.kps_project_linear_into(anchor, inst2d, self.learnable_fc_weight, self.learnable_fc_bias,
                                                self.fix_scale, projection_mat, image_wh, sample_location=loc)
                ops.weights_fc_into(logits.view(rows, -1), None, inst2d, embed2d, self.weights_fc_weight, None,
                                    None)
                if capturing:
                    torch.cuda.current_stream(dev).wait_stream(self._side_kps)
            else:
                # Large batches: the tensor-core pass produces the learnable logits almost for free
                # (one N-32 MMA per K step), then the plain keypoint kernel runs.
                loc = torch.empty(bs, num_anchor, self.num_cams, self.num_pts, 2, dtype=torch.float32, device=dev)
                learn = torch.empty(bs, num_anchor, 3 * self.num_learnable_pts, device=dev)
                ops.weights_fc_into(logits.view(rows, -1), learn.view(rows, -1), inst2d, embed2d,
                                    self.weights_fc_weight, self.learnable_fc_weight, self.learnable_fc_bias)
                ops.kps_project_into(anchor, learn, self.fix_scale, projection_mat, image_wh, sample_location=loc)
        else:
            with _matmul_precision(self.matmul_precision):
                logits, logits_cam = self._get_weights(instance_feature, anchor_embed, projection_mat, bs, num_anchor)
                learn = F.linear(instance_feature, self.learnable_fc_weight, self.learnable_fc_bias).contiguous()
            loc = torch.empty(bs, num_anchor, self.num_cams, self.num_pts, 2, dtype=torch.float32, device=dev)
            ops.kps_project_into(anchor, learn, self.fix_scale, projection_mat, image_wh, sample_location=loc)
        self._join_side()  # the camera terms are needed from here on
        nxt = self.next_layer
        if nxt is not None and self._tc and nxt._tc and side:
            nxt._camera_logits(projection_mat, bs, side=True)  # forked after weights_fc: beside the gather

        cam_begin, cam_end = 0, self.num_cams
        if self.process_group is not None:
            from .camera_shard import rank_camera_range

            cam_begin, cam_end = rank_camera_range(self.num_cams, self.process_group)
        p2p = self.process_group is not None and self.camera_reduce == "p2p"
        if p2p:
            # the gather writes this rank's rows into its own buffer and the other rank's rows
            # straight into that rank's receive buffer over NVLink, once the other rank has
            # finished reading it (begin); the exchanges keep their epochs on the device, so the
            # call can be captured in a CUDA graph
            if self._peer is None or self._peer.closed or self._peer.capacity < rows:
                from .camera_shard import PeerPartialSums

                if torch.cuda.is_current_stream_capturing():
                    raise RuntimeError("CAMERA_REDUCE='p2p': run the module once eagerly (on both ranks, with "
                                       "this batch size or larger) before capturing it in a CUDA graph")
                if self._peer is not None:
                    self._peer.close()  # collective; a no-op when already closed
                self._peer = PeerPartialSums(rows, self.embed_dims, self.process_group, dev)
            feats = self._peer.begin(rows).view(bs, num_anchor, self.embed_dims)
        else:
            feats = torch.empty(bs, num_anchor, self.embed_dims, dtype=torch.float32, device=dev)
        logits = logits.contiguous()
        logits_cam = None if logits_cam is None else logits_cam.contiguous()
        log = self.event_log
        if log is not None:
            # The two records run on a timing branch (forked from the launching stream, joined
            # back at the next call or by join_timing_stream()), so no kernel waits on them.
            self.join_timing_stream()
            if self._timing is None:
                self._timing = torch.cuda.Stream(dev)
            cur = torch.cuda.current_stream(dev)
            ev = (TimingEvent(), TimingEvent())
            self._timing.wait_stream(cur)
            ev[0].record(self._timing)
        ws, ready = None, False
        if logits_cam is not None:
            ws, ready = self._cached_camera_factors, self._cached_camera_factors is not None
            if ws is None:
                ws = ops.dfa_workspace(bs, self.num_cams, self.num_levels, self.num_pts, self.num_groups, dev)
        if loc is None:  # the camera factors are prepared whenever the shape has the kernel for them
            if not ready:
                raise RuntimeError("DeformableFeatureAggregation: camera factors missing for the gather from anchors")
            route = {}
            if p2p:  # the other rank's rows go straight to its receive buffer
                from .camera_shard import shard_rows

                mb, me = shard_rows(rows, self.process_group)
                route = dict(out_peer=self._peer.peer_recv, peer_rows=(me, rows) if mb == 0 else (0, mb))
            ops.deformable_aggregation_anchors_into(feats, mc_ms_feat, spatial_shape, scale_start, anchor,
                                                    self.fix_scale, learn.view(rows, -1), projection_mat, image_wh,
                                                    logits, logits_cam, ws, cam_begin, cam_end, **route)
        else:
            ops.deformable_aggregation_into(feats, mc_ms_feat, spatial_shape, scale_start, loc, logits, True,
                                            logits_cam, cam_begin, cam_end, workspace=ws, factors_ready=ready)
        if log is not None:
            self._timing.wait_stream(cur)
            ev[1].record(self._timing)
            self._timing_pending = True
            log.append(ev)
        self.shard = (0, rows)
        out_shape = (bs, num_anchor)
        feats2d = feats.view(rows, C)
        inst_rows = instance_feature.reshape(rows, C)
        if p2p:
            from .camera_shard import shard_rows

            # this rank's rows of (own partial sums + the other rank's, received during its
            # gather), summed in output_proj's tensor-core accumulator
            self.shard = b, e = shard_rows(rows, self.process_group)
            recv = self._peer.exchange()
            width = 2 * C if self.residual_mode == "cat" else C
            out = torch.empty(e - b, width, device=dev)
            ops.output_proj_sum_into(out, feats2d, recv.data_ptr(), b, e - b, self.output_proj_weight,
                                     self.output_proj_bias, ops.row_view(inst_rows[b:e], C), self.residual_mode,
                                     error_flag=self._peer.error_flag)
            return out
        if self.process_group is not None:
            from .camera_shard import reduce_partial_sums, shard_rows

            if self.camera_reduce == "reduce_scatter":
                # NCCL reduce-scatter over the flattened (frame, anchor) rows: this rank keeps its
                # shard of the summed features and projects only those rows
                self.shard = shard_rows(rows, self.process_group)
                feats2d = reduce_partial_sums(feats2d, self.process_group, scatter=True)
                inst_rows = inst_rows[self.shard[0]:self.shard[1]]
                out_shape = (self.shard[1] - self.shard[0],)
            else:
                reduce_partial_sums(feats, self.process_group)
        n_out = feats2d.shape[0]

        if self._tc:
            width = 2 * C if self.residual_mode == "cat" else C
            out = torch.empty(*out_shape, width, device=dev)
            ops.output_proj_into(out.view(n_out, width), feats2d, self.output_proj_weight, self.output_proj_bias,
                                 ops.row_view(inst_rows, C), self.residual_mode)
            return out
        with _matmul_precision(self.matmul_precision):
            out = F.linear(feats2d, self.output_proj_weight, self.output_proj_bias)
        inst = inst_rows.to(out.dtype)
        if self.residual_mode == "add":
            out = out + inst
        elif self.residual_mode == "cat":
            out = torch.cat([out, inst], dim=-1)
        return out.reshape(*out_shape, out.shape[-1])

    __call__ = run


def _is_process_group(obj) -> bool:
    if obj is None:
        return False
    try:
        import torch.distributed as dist

        return isinstance(obj, dist.ProcessGroup)
    except Exception:  # pragma: no cover - torch built without distributed
        return False
