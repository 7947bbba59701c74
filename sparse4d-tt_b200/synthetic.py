"""Seeded synthetic inputs for the DFA path.

No dataset or checkpoint exists on the machines this runs on, so every input is drawn
from fixed distributions with a fixed seed:

* anchors ``[bs, A, 11]`` = (x, y, z, log w, log l, log h, sin yaw, cos yaw, vx, vy, vz),
  with x, y ~ U(-50, 50) m, z ~ U(-4, 2), w, l, h ~ U(0.5, 5), yaw ~ U(-pi, pi),
  vx, vy ~ N(0, 2), vz = 0 (anchor field order as in ``test/dfa_pcc.py:164-167``);
* instance features and anchor embeddings ~ N(0, 1);
* a 6-camera ring at yaw 0, +-55, +-110, 180 degrees, 1.5 m above the origin, with pinhole
  intrinsics fx = fy = 560, cx = 352, cy = 128 for a 704 x 256 image (scaled to the image
  size for other resolutions).  ``lidar2img = K @ [R | t]`` with camera axes x right,
  y down, z forward, the convention of ``test/sparse4d_nuscenes_val.py:474-486``;
* FPN feature maps ~ N(0, 1) at strides 4, 8, 16, 32 of the image;
* layer weights from Xavier-uniform init with zero bias, LayerNorm weight 1 / bias 0.

The parameter dictionary uses the keys of ``preprocess_dfa_parameters``
(``model/deformable_feature_aggregation.py:954-995``) so it feeds both the drop-in module and
the oracle.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Tuple

import torch

# Anchor field indices (Sparse4D box convention, test/dfa_pcc.py:164-167).
X, Y, Z = 0, 1, 2
W, L, H = 3, 4, 5
SIN_YAW, COS_YAW = 6, 7
VX, VY, VZ = 8, 9, 10

# Fixed keypoint scales of Sparse4D v3: the centre and +-0.45 of the box size on each axis
# (test/dfa_pcc.py:366-370).
FIX_SCALE = [
    [0.0, 0.0, 0.0],
    [0.45, 0.0, 0.0],
    [-0.45, 0.0, 0.0],
    [0.0, 0.45, 0.0],
    [0.0, -0.45, 0.0],
    [0.0, 0.0, 0.45],
    [0.0, 0.0, -0.45],
]

CAMERA_YAWS_DEG = [0.0, 55.0, -55.0, 110.0, -110.0, 180.0]


@dataclass
class DFAConfig:
    """Shape of one DFA layer call."""

    bs: int = 1
    num_anchor: int = 900
    num_cams: int = 6
    embed_dims: int = 256
    num_groups: int = 8
    num_learnable_pts: int = 6
    image_wh: Tuple[int, int] = (704, 256)
    strides: Tuple[int, ...] = (4, 8, 16, 32)
    fix_scale: List[List[float]] = field(default_factory=lambda: [r[:] for r in FIX_SCALE])

    @property
    def num_levels(self) -> int:
        return len(self.strides)

    @property
    def num_pts(self) -> int:
        return len(self.fix_scale) + self.num_learnable_pts

    @property
    def spatial_shapes(self) -> List[Tuple[int, int]]:
        w, h = self.image_wh
        return [(h // s, w // s) for s in self.strides]

    @property
    def pixels_per_cam(self) -> int:
        return sum(h * w for h, w in self.spatial_shapes)


def config_standard(bs: int = 1) -> DFAConfig:
    """704 x 256 image, 900 anchors: the shape of a Sparse4D v3 R50 DFA layer."""
    return DFAConfig(bs=bs)


def config_highres(bs: int = 1, num_anchor: int = 1800) -> DFAConfig:
    """1600 x 640 image (maps 160x400 ... 20x50), 1800 anchors."""
    return DFAConfig(bs=bs, num_anchor=num_anchor, image_wh=(1600, 640))


def camera_ring(num_cams: int, image_wh: Tuple[int, int], dtype=torch.float32) -> torch.Tensor:
    """lidar2img matrices ``[num_cams, 4, 4]`` of the synthetic ring."""
    w, h = image_wh
    f = 560.0 * (w / 704.0)
    K = torch.eye(4, dtype=torch.float64)
    K[0, 0], K[1, 1], K[0, 2], K[1, 2] = f, f, w / 2.0, h / 2.0
    mats = []
    centre = torch.tensor([0.0, 0.0, 1.5], dtype=torch.float64)
    for i in range(num_cams):
        yaw = math.radians(CAMERA_YAWS_DEG[i % len(CAMERA_YAWS_DEG)])
        fwd = torch.tensor([math.cos(yaw), math.sin(yaw), 0.0], dtype=torch.float64)
        right = torch.tensor([math.sin(yaw), -math.cos(yaw), 0.0], dtype=torch.float64)
        down = torch.tensor([0.0, 0.0, -1.0], dtype=torch.float64)
        R = torch.stack([right, down, fwd])
        T = torch.eye(4, dtype=torch.float64)
        T[:3, :3] = R
        T[:3, 3] = -R @ centre
        mats.append(K @ T)
    return torch.stack(mats).to(dtype)


# Every draw below is identical on every host CPU.  torch's CPU uniform sampler is scalar per
# element and float32 add / multiply are exact IEEE operations, but its normal sampler and its
# float32 log / sin / cos pick a SIMD code path per host, whose last bits differ between
# machines; so normals come from Box-Muller over float64 uniforms and every transcendental
# function is evaluated in float64 and rounded once to float32.  (A float64 result that differs
# by one ulp between hosts rounds to the same float32 unless it sits within 2^-29 of a rounding
# tie.)
_NORMAL_CHUNK = 1 << 22


def normal(shape, gen: torch.Generator) -> torch.Tensor:
    """N(0, 1) float32 draws of ``shape`` from ``gen``, reproducible across host CPUs."""
    n = math.prod(shape)
    out = torch.empty(n, dtype=torch.float32)
    for start in range(0, n, 2 * _NORMAL_CHUNK):
        m = min(2 * _NORMAL_CHUNK, n - start)
        half = (m + 1) // 2
        u = torch.rand(2, half, dtype=torch.float64, generator=gen)
        r = torch.sqrt(-2.0 * torch.log1p(-u[0]))  # 1 - u in (0, 1]
        t = (2.0 * math.pi) * u[1]
        out[start:start + m] = torch.cat([r * torch.cos(t), r * torch.sin(t)])[:m].float()
    return out.reshape(shape)


def make_anchors(bs: int, num_anchor: int, gen: torch.Generator) -> torch.Tensor:
    a = torch.zeros(bs, num_anchor, 11)
    a[..., X] = torch.rand(bs, num_anchor, generator=gen) * 100.0 - 50.0
    a[..., Y] = torch.rand(bs, num_anchor, generator=gen) * 100.0 - 50.0
    a[..., Z] = torch.rand(bs, num_anchor, generator=gen) * 6.0 - 4.0
    size = torch.rand(bs, num_anchor, 3, generator=gen) * 4.5 + 0.5
    a[..., W:H + 1] = size.double().log().float()
    yaw = torch.rand(bs, num_anchor, generator=gen) * (2 * math.pi) - math.pi
    a[..., SIN_YAW] = yaw.double().sin().float()
    a[..., COS_YAW] = yaw.double().cos().float()
    a[..., VX:VY + 1] = normal((bs, num_anchor, 2), gen) * 2.0
    return a


def refine_anchors(anchor: torch.Tensor, gen: torch.Generator, sigma: float = 0.1) -> torch.Tensor:
    """Stand-in for the decoder's box refinement between stacked DFA layers: N(0, sigma)
    offsets on centre, log-size, yaw (sin/cos, renormalised) and velocity."""
    a = anchor.clone()
    noise = normal(tuple(a.shape), gen) * sigma
    a[..., X:H + 1] += noise[..., X:H + 1]
    a[..., VX:VZ] += noise[..., VX:VZ]
    sc = (a[..., SIN_YAW:COS_YAW + 1] + noise[..., SIN_YAW:COS_YAW + 1]).double()
    a[..., SIN_YAW:COS_YAW + 1] = (sc / sc.norm(dim=-1, keepdim=True).clamp(min=1e-6)).float()
    return a


def make_params(cfg: DFAConfig, gen: torch.Generator) -> Dict[str, torch.Tensor]:
    """Xavier-uniform weights, zero biases, unit LayerNorms, keyed like
    ``preprocess_dfa_parameters`` (``model/deformable_feature_aggregation.py:954-995``)."""
    C = cfg.embed_dims

    def xavier(out_f, in_f):
        bound = math.sqrt(6.0 / (in_f + out_f))
        return torch.rand(out_f, in_f, generator=gen) * (2 * bound) - bound

    n_w = cfg.num_groups * cfg.num_levels * cfg.num_pts
    return {
        "kps_fix_scale": torch.tensor(cfg.fix_scale, dtype=torch.float32),
        "kps_learnable_fc_weight": xavier(cfg.num_learnable_pts * 3, C),
        "kps_learnable_fc_bias": torch.zeros(cfg.num_learnable_pts * 3),
        "cam_linear1_weight": xavier(C, 12),
        "cam_linear1_bias": torch.zeros(C),
        "cam_ln1_weight": torch.ones(C),
        "cam_ln1_bias": torch.zeros(C),
        "cam_linear2_weight": xavier(C, C),
        "cam_linear2_bias": torch.zeros(C),
        "cam_ln2_weight": torch.ones(C),
        "cam_ln2_bias": torch.zeros(C),
        "weights_fc_weight": xavier(n_w, C),
        "weights_fc_bias": torch.zeros(n_w),
        "output_proj_weight": xavier(C, C),
        "output_proj_bias": torch.zeros(C),
    }


@dataclass
class DFAInputs:
    instance_feature: torch.Tensor  # [bs, A, C]
    anchor: torch.Tensor  # [bs, A, 11]
    anchor_embed: torch.Tensor  # [bs, A, C]
    feature_maps: List[torch.Tensor]  # per level [bs, Ncam, C, H, W] (NCHW, as the oracle takes)
    projection_mat: torch.Tensor  # [bs, Ncam, 4, 4]
    image_wh: torch.Tensor  # [bs, Ncam, 2]


def make_inputs(
    cfg: DFAConfig,
    seed: int,
    feature_dtype: Optional[torch.dtype] = None,
    device: str = "cpu",
) -> DFAInputs:
    """All inputs of one DFA layer call.  ``feature_dtype=torch.bfloat16`` rounds the maps to
    bf16 (returned upcast to fp32, so the oracle sees exactly the values the bf16 kernel
    reads).  Small tensors are always drawn on the CPU generator so they are identical on
    every machine; with ``device='cuda'`` the maps are drawn by a CUDA generator instead
    (used for large benchmark batches, never for parity)."""
    gen = torch.Generator().manual_seed(seed)
    bs, A, C = cfg.bs, cfg.num_anchor, cfg.embed_dims
    inst = normal((bs, A, C), gen)
    anchor = make_anchors(bs, A, gen)
    embed = normal((bs, A, C), gen)
    proj = camera_ring(cfg.num_cams, cfg.image_wh).unsqueeze(0).expand(bs, -1, -1, -1).contiguous()
    wh = torch.tensor(cfg.image_wh, dtype=torch.float32).expand(bs, cfg.num_cams, 2).contiguous()
    maps = []
    if device == "cpu":
        for h, w in cfg.spatial_shapes:
            fm = normal((bs, cfg.num_cams, C, h, w), gen)
            if feature_dtype is not None and feature_dtype != torch.float32:
                fm = fm.to(feature_dtype).float()
            maps.append(fm)
    else:
        g2 = torch.Generator(device=device).manual_seed(seed + 7919)
        for h, w in cfg.spatial_shapes:
            fm = torch.randn(bs, cfg.num_cams, C, h, w, generator=g2, device=device)
            if feature_dtype is not None and feature_dtype != torch.float32:
                fm = fm.to(feature_dtype).float()
            maps.append(fm)
    return DFAInputs(inst, anchor, embed, maps, proj, wh)


def head_operation_order(num_decoder: int = 6, num_single_frame: int = 1) -> List[str]:
    """Operation order of the Sparse4D v3 decoder (``model/sparse4d_head.py``): one single-frame
    decoder ``deformable, ffn, norm, refine``, then ``temp_gnn, gnn, norm, deformable, ffn, norm,
    refine`` per temporal decoder."""
    return (["gnn", "norm", "deformable", "ffn", "norm", "refine"] * num_single_frame
            + ["temp_gnn", "gnn", "norm", "deformable", "ffn", "norm", "refine"] * (num_decoder - num_single_frame))[2:]


def make_head_params(cfg: DFAConfig, gen: torch.Generator, num_cls: int = 10, num_decoder: int = 6,
                     refine_scale: float = 0.1) -> Dict:
    """Parameters of a single-frame decoder head in the format of ``head.preprocess_head_parameters``:
    Xavier-uniform weights, zero biases, unit LayerNorms; the DFA layers from ``make_params``.
    The refinement's output scale is ``refine_scale`` (a trained head moves boxes by small
    steps; Xavier-initialised layers at scale 1 would move them by metres per layer); the
    instance bank's anchors are seeded scene anchors (``make_anchors``) and its features zeros."""
    C = cfg.embed_dims

    def xavier(out_f, in_f):
        bound = math.sqrt(6.0 / (in_f + out_f))
        return torch.rand(out_f, in_f, generator=gen) * (2 * bound) - bound

    def mlp(dims_in, dims, in_loops, out_loops):
        mods, d_in = [], dims_in
        for _ in range(out_loops):
            for _ in range(in_loops):
                mods += [("linear", xavier(dims, d_in), torch.zeros(dims)), ("relu", None, None)]
                d_in = dims
            mods.append(("ln", torch.ones(dims), torch.zeros(dims)))
        return mods

    order = head_operation_order(num_decoder)
    layers = []
    for op in order:
        if op in ("gnn", "temp_gnn"):
            layers.append({"in_proj_weight": xavier(3 * 2 * C, 2 * C), "in_proj_bias": torch.zeros(3 * 2 * C),
                           "out_proj_weight": xavier(2 * C, 2 * C), "out_proj_bias": torch.zeros(2 * C),
                           "num_heads": cfg.num_groups})
        elif op == "norm":
            layers.append({"weight": torch.ones(C), "bias": torch.zeros(C)})
        elif op == "deformable":
            layers.append(make_params(cfg, gen))
        elif op == "ffn":
            layers.append({"pre_norm": (torch.ones(2 * C), torch.zeros(2 * C)),
                           "fc1": (xavier(4 * C, 2 * C), torch.zeros(4 * C)), "fc2": (xavier(C, 4 * C), torch.zeros(C)),
                           "identity_fc": (xavier(C, 2 * C), torch.zeros(C))})
        else:  # refine
            layers.append({"layers": mlp(C, C, 2, 2) + [("linear", xavier(11, C), torch.zeros(11)),
                                                        ("scale", torch.full((11,), refine_scale), None)],
                           "cls_layers": mlp(C, C, 1, 2) + [("linear", xavier(num_cls, C), torch.zeros(num_cls))],
                           "quality_layers": mlp(C, C, 1, 2) + [("linear", xavier(2, C), torch.zeros(2))]})
    encoder = {"pos_fc": mlp(3, 128, 1, 4), "size_fc": mlp(3, 32, 1, 4), "yaw_fc": mlp(2, 32, 1, 4),
               "vel_fc": mlp(3, 64, 1, 4)}
    return {"operation_order": order, "layers": layers, "anchor_encoder": encoder,
            "anchor": make_anchors(1, cfg.num_anchor, gen)[0], "instance_feature": torch.zeros(cfg.num_anchor, C),
            "fc_before": xavier(2 * C, C), "fc_after": xavier(C, 2 * C), "num_single_frame_decoder": 1}
