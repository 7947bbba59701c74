"""Torch operators of the DFA hot path, each a thin wrapper over the C ABI.

* ``deformable_aggregation(mc_ms_feat, spatial_shape, scale_start_index, sample_location,
  weights, ...)`` -- fused softmax + multi-camera multi-scale bilinear gather + weighted sum;
  the argument meaning of upstream Sparse4D's op of the same name, and the replacement of
  ``ttnn.grid_sample`` + ``ttnn.transposed_s2i`` + ``ttnn.grouped_weighted_sum`` + softmax
  (``model/deformable_feature_aggregation.py:791-796,877-899``).
* ``kps_project(anchor, learnable_logits, fix_scale, projection_mat, image_wh, ...)`` --
  keypoints, projection, depth / frustum masks and the compacted visible indices
  (``test/dfa_pcc.py:225-247,322-333``).
* ``kps_project_fused(key_points, anchor, projection_mat, image_wh, num_cams, num_pts)`` --
  same arguments and output layout as ``ttnn.kps_project_fused``
  (``tt-metal/ops/kps_project_fused/kps_project_fused_nanobind.cpp:69-91``).
* ``weights_fc_into`` / ``output_proj_into`` -- the layer's linears on the tensor cores
  (tcgen05, TF32 operands, fp32 accumulation): ``weights_fc`` (per-anchor logits) + the
  keypoint ``learnable_fc`` in one pass with the embed add fused, and ``output_proj`` with
  the residual cat/add fused (``model/deformable_feature_aggregation.py:651-677,719-798,934-950``).
* ``pack_feature_maps(feature_maps)`` -- per-level maps to the packed channels-last
  ``mc_ms_feat`` layout.

The ``*_into`` variants write into caller-provided tensors and are what the drop-in module
uses (no allocation, CUDA-graph capturable).  All of them validate dtype, device, shape and
contiguity and raise ``ValueError`` / ``TypeError``; a non-OK status from the library raises.
There is no CPU path: CPU tensors are rejected.
"""
from __future__ import annotations

import ctypes as C
from typing import List, Optional, Sequence, Tuple, Union

import torch

from . import _lib as L

Tensor = torch.Tensor

LAYOUTS = {"cam_major": L.S4D_LAYOUT_CAM_MAJOR, "pt_major": L.S4D_LAYOUT_PT_MAJOR}


def _ptr(t: Optional[Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


# torch's current-stream handle of a device index, without building a Stream object (a
# measurable share of an eager small-batch call); the public call where it is missing
_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _stream_ptr(device: torch.device) -> int:
    if _raw_stream is not None and device.index is not None:
        return _raw_stream(device.index)
    return torch.cuda.current_stream(device).cuda_stream


def _require_cuda(name: str, *ts: Optional[Tensor]) -> torch.device:
    idx = None
    for t in ts:
        if t is None:
            continue
        i = t.get_device()
        if i < 0:
            raise ValueError(f"{name}: every tensor must be on a CUDA device (got {t.device}); no CPU path exists")
        if idx is None:
            idx = i
        elif i != idx:
            raise ValueError(f"{name}: tensors on different devices (cuda:{idx} and cuda:{i})")
    return None if idx is None else torch.device("cuda", idx)


def _require(cond: bool, msg) -> None:
    """Raise ValueError(msg) unless cond; msg may be a callable that builds the text (so that
    the checks of a successful call format nothing)."""
    if not cond:
        raise ValueError(msg() if callable(msg) else msg)


def _check_contig(name: str, **ts: Optional[Tensor]) -> None:
    for k, t in ts.items():
        if t is not None and not t.is_contiguous():
            raise ValueError(f"{name}: {k} must be contiguous")


def _check_dtype(name: str, t: Optional[Tensor], dtypes: Sequence[torch.dtype], what: str) -> None:
    if t is not None and t.dtype not in dtypes:
        raise TypeError(f"{name}: {what} must be one of {list(dtypes)}, got {t.dtype}")


# ---------------------------------------------------------------------------------------------
# dense linears on the tensor cores
# ---------------------------------------------------------------------------------------------

RESIDUAL_MODES = {"none": L.S4D_RESIDUAL_NONE, "add": L.S4D_RESIDUAL_ADD, "cat": L.S4D_RESIDUAL_CAT}


def row_view(t: Tensor, cols: int) -> Tensor:
    """``t [..., cols]`` as a 2-D ``[rows, cols]`` fp32 view the tensor-core kernels can read
    in place (unit column stride, row stride a multiple of 4 floats, 16-byte aligned base);
    a contiguous copy when the strides do not allow that."""
    _require(t.shape[-1] == cols, lambda: f"expected a last dimension of {cols}, got {tuple(t.shape)}")
    v = t.reshape(-1, cols)
    if v.stride(1) != 1 or v.stride(0) % 4 != 0 or v.stride(0) < cols or v.data_ptr() % 16 != 0:
        v = v.contiguous()
    return v


def weights_fc_supported(num_logits: int, num_learnable: int, embed_dims: int) -> bool:
    """Shapes ``weights_fc_into`` implements (the Sparse4D v3 layer: 4 x 13 x 8 logits)."""
    return num_logits == 416 and 0 <= num_learnable <= 32 and embed_dims == 256


def weights_fc_into(logits: Tensor, learnable: Optional[Tensor], instance_feature: Tensor, anchor_embed: Tensor,
                    weights_fc_weight: Tensor, learnable_fc_weight: Optional[Tensor],
                    learnable_bias: Optional[Tensor] = None, error_flag: Optional[Tensor] = None) -> None:
    """``logits [rows, n] = (instance_feature + anchor_embed) W_fc^T`` and ``learnable [rows, m]
    = instance_feature W_kps^T + learnable_bias`` in one tensor-core pass.  ``instance_feature``
    and ``anchor_embed`` are ``[rows, C]`` row views (``row_view``)."""
    name = "weights_fc"
    dev = _require_cuda(name, logits, learnable, instance_feature, anchor_embed, weights_fc_weight,
                        learnable_fc_weight, learnable_bias, error_flag)
    _check_contig(name, logits=logits, learnable=learnable, weights_fc_weight=weights_fc_weight,
                  learnable_fc_weight=learnable_fc_weight, learnable_bias=learnable_bias)
    for k, t in (("logits", logits), ("learnable", learnable), ("instance_feature", instance_feature),
                 ("anchor_embed", anchor_embed), ("weights_fc_weight", weights_fc_weight),
                 ("learnable_fc_weight", learnable_fc_weight), ("learnable_bias", learnable_bias)):
        _check_dtype(name, t, (torch.float32,), k)
    _check_dtype(name, error_flag, (torch.int32,), "error_flag")
    rows, c = instance_feature.shape
    _require(tuple(anchor_embed.shape) == (rows, c), "anchor_embed must match instance_feature")
    _require(instance_feature.stride(1) == 1 and anchor_embed.stride(1) == 1, "inputs need a unit column stride")
    n = int(weights_fc_weight.shape[0])
    _require(tuple(weights_fc_weight.shape) == (n, c), lambda: f"weights_fc_weight must be [n, {c}]")
    _require(tuple(logits.shape) == (rows, n), lambda: f"logits must be [{rows}, {n}]")
    m = 0 if learnable is None else int(learnable.shape[1])
    _require(learnable is None or tuple(learnable.shape) == (rows, m), lambda: f"learnable must be [{rows}, m]")
    _require(m == 0 or (learnable_fc_weight is not None and tuple(learnable_fc_weight.shape) == (m, c)),
             f"learnable_fc_weight must be [{m}, {c}]")
    _require(learnable_bias is None or tuple(learnable_bias.shape) == (m,), lambda: f"learnable_bias must be [{m}]")
    st = L.lib().s4d_dfa_weights_fc(instance_feature.data_ptr(), instance_feature.stride(0), anchor_embed.data_ptr(),
                                    anchor_embed.stride(0), rows, weights_fc_weight.data_ptr(),
                                    _ptr(learnable_fc_weight), _ptr(learnable_bias), n, m, c, logits.data_ptr(),
                                    _ptr(learnable), _ptr(error_flag), _stream_ptr(dev))
    L.check(name, st)


def camera_logits_into(camera_logits: Tensor, projection_mat: Tensor, cam_linear1_weight: Tensor,
                       cam_linear1_bias: Tensor, cam_ln1_weight: Tensor, cam_ln1_bias: Tensor,
                       cam_linear2_weight: Tensor, cam_linear2_bias: Tensor, cam_ln2_weight: Tensor,
                       cam_ln2_bias: Tensor, weights_fc_weight: Tensor, weights_fc_bias: Tensor,
                       camera_embed: Optional[Tensor] = None, workspace: Optional[Tensor] = None) -> Tensor:
    """Camera encoder + ``weights_fc`` on its output, one CTA per frame:
    ``camera_logits [bs, Ncam, n]`` (and optionally ``camera_embed [bs, Ncam, C]``) from
    ``projection_mat [bs, Ncam, 4, 4]`` (``model/deformable_feature_aggregation.py:679-717``)."""
    name = "camera_logits"
    ts = dict(camera_logits=camera_logits, projection_mat=projection_mat, cam_linear1_weight=cam_linear1_weight,
              cam_linear1_bias=cam_linear1_bias, cam_ln1_weight=cam_ln1_weight, cam_ln1_bias=cam_ln1_bias,
              cam_linear2_weight=cam_linear2_weight, cam_linear2_bias=cam_linear2_bias,
              cam_ln2_weight=cam_ln2_weight, cam_ln2_bias=cam_ln2_bias, weights_fc_weight=weights_fc_weight,
              weights_fc_bias=weights_fc_bias, camera_embed=camera_embed)
    dev = _require_cuda(name, *ts.values())
    _check_contig(name, **ts)
    for k, t in ts.items():
        _check_dtype(name, t, (torch.float32,), k)
    _require(projection_mat.dim() == 4 and tuple(projection_mat.shape[2:]) == (4, 4),
             "projection_mat must be [bs, Ncam, 4, 4]")
    bs, nc = int(projection_mat.shape[0]), int(projection_mat.shape[1])
    n, c = weights_fc_weight.shape
    _require(tuple(cam_linear1_weight.shape) == (c, 12) and tuple(cam_linear2_weight.shape) == (c, c),
             f"camera encoder weights must be [{c}, 12] and [{c}, {c}]")
    for k in ("cam_linear1_bias", "cam_ln1_weight", "cam_ln1_bias", "cam_linear2_bias", "cam_ln2_weight",
              "cam_ln2_bias"):
        _require(tuple(ts[k].shape) == (c,), lambda: f"{k} must be [{c}]")
    _require(tuple(weights_fc_bias.shape) == (n,), lambda: f"weights_fc_bias must be [{n}]")
    _require(camera_logits.numel() == bs * nc * n, lambda: f"camera_logits must hold [{bs}, {nc}, {n}]")
    _require(camera_embed is None or camera_embed.numel() == bs * nc * c,
             lambda: f"camera_embed must hold [{bs}, {nc}, {c}]")
    if workspace is None:
        workspace = torch.empty(bs * nc * c, dtype=torch.float32, device=dev)
    _require_cuda(name, workspace)
    ws_bytes = workspace.numel() * workspace.element_size()
    st = L.lib().s4d_dfa_camera_logits(
        projection_mat.data_ptr(), bs, nc, cam_linear1_weight.data_ptr(), cam_linear1_bias.data_ptr(),
        cam_ln1_weight.data_ptr(), cam_ln1_bias.data_ptr(), cam_linear2_weight.data_ptr(), cam_linear2_bias.data_ptr(),
        cam_ln2_weight.data_ptr(), cam_ln2_bias.data_ptr(), weights_fc_weight.data_ptr(), weights_fc_bias.data_ptr(),
        n, c, _ptr(camera_embed), camera_logits.data_ptr(), workspace.data_ptr(), ws_bytes, _stream_ptr(dev))
    L.check(name, st)
    return camera_logits


def camera_terms_into(camera_logits: Tensor, projection_mat: Tensor, cam_linear1_weight: Tensor,
                      cam_linear1_bias: Tensor, cam_ln1_weight: Tensor, cam_ln1_bias: Tensor,
                      cam_linear2_weight: Tensor, cam_linear2_bias: Tensor, cam_ln2_weight: Tensor,
                      cam_ln2_bias: Tensor, weights_fc_weight: Tensor, weights_fc_bias: Tensor,
                      camera_embed: Optional[Tensor] = None, factors: Optional[Tensor] = None) -> Tensor:
    """``camera_logits_into`` and, with ``factors`` (a workspace from ``dfa_workspace``),
    ``camera_factors_into`` in one launch of 8-CTA clusters, bitwise equal to the two calls
    (``model/deformable_feature_aggregation.py:679-805``).  Needs no scratch workspace."""
    name = "camera_terms"
    ts = dict(camera_logits=camera_logits, projection_mat=projection_mat, cam_linear1_weight=cam_linear1_weight,
              cam_linear1_bias=cam_linear1_bias, cam_ln1_weight=cam_ln1_weight, cam_ln1_bias=cam_ln1_bias,
              cam_linear2_weight=cam_linear2_weight, cam_linear2_bias=cam_linear2_bias,
              cam_ln2_weight=cam_ln2_weight, cam_ln2_bias=cam_ln2_bias, weights_fc_weight=weights_fc_weight,
              weights_fc_bias=weights_fc_bias, camera_embed=camera_embed, factors=factors)
    dev = _require_cuda(name, *ts.values())
    _check_contig(name, **ts)
    for k, t in ts.items():
        _check_dtype(name, t, (torch.float32,), k)
    _require(projection_mat.dim() == 4 and tuple(projection_mat.shape[2:]) == (4, 4),
             "projection_mat must be [bs, Ncam, 4, 4]")
    bs, nc = int(projection_mat.shape[0]), int(projection_mat.shape[1])
    n, c = weights_fc_weight.shape
    _require(tuple(cam_linear1_weight.shape) == (c, 12) and tuple(cam_linear2_weight.shape) == (c, c),
             f"camera encoder weights must be [{c}, 12] and [{c}, {c}]")
    for k in ("cam_linear1_bias", "cam_ln1_weight", "cam_ln1_bias", "cam_linear2_bias", "cam_ln2_weight",
              "cam_ln2_bias"):
        _require(tuple(ts[k].shape) == (c,), lambda: f"{k} must be [{c}]")
    _require(tuple(weights_fc_bias.shape) == (n,), lambda: f"weights_fc_bias must be [{n}]")
    _require(camera_logits.numel() == bs * nc * n, lambda: f"camera_logits must hold [{bs}, {nc}, {n}]")
    _require(camera_embed is None or camera_embed.numel() == bs * nc * c,
             lambda: f"camera_embed must hold [{bs}, {nc}, {c}]")
    fb = 0 if factors is None else factors.numel() * factors.element_size()
    st = L.lib().s4d_dfa_camera_terms(
        projection_mat.data_ptr(), bs, nc, cam_linear1_weight.data_ptr(), cam_linear1_bias.data_ptr(),
        cam_ln1_weight.data_ptr(), cam_ln1_bias.data_ptr(), cam_linear2_weight.data_ptr(), cam_linear2_bias.data_ptr(),
        cam_ln2_weight.data_ptr(), cam_ln2_bias.data_ptr(), weights_fc_weight.data_ptr(), weights_fc_bias.data_ptr(),
        n, c, _ptr(camera_embed), camera_logits.data_ptr(), _ptr(factors), fb, _stream_ptr(dev))
    L.check(name, st)
    return camera_logits


def output_proj_into(out: Tensor, features: Tensor, weight: Tensor, bias: Optional[Tensor],
                     instance_feature: Optional[Tensor] = None, residual_mode: str = "cat",
                     error_flag: Optional[Tensor] = None) -> Tensor:
    """``out[:, :C] = features W^T + bias`` with the residual fused: ``"cat"`` also writes
    ``out[:, C:2C] = instance_feature``, ``"add"`` adds it, ``"none"`` ignores it.  ``out`` is
    ``[rows, >= 2C or C]`` (row stride a multiple of 4), ``instance_feature`` a row view."""
    name = "output_proj"
    mode = RESIDUAL_MODES[residual_mode]
    dev = _require_cuda(name, out, features, weight, bias, instance_feature, error_flag)
    _check_contig(name, features=features, weight=weight, bias=bias)
    for k, t in (("out", out), ("features", features), ("weight", weight), ("bias", bias),
                 ("instance_feature", instance_feature)):
        _check_dtype(name, t, (torch.float32,), k)
    _check_dtype(name, error_flag, (torch.int32,), "error_flag")
    rows, c = features.shape
    _require(tuple(weight.shape) == (c, c), lambda: f"weight must be [{c}, {c}]")
    _require(out.dim() == 2 and out.shape[0] == rows and out.stride(1) == 1,
             lambda: f"out must be a [{rows}, n] row view")
    if mode != L.S4D_RESIDUAL_NONE:
        _require(instance_feature is not None and tuple(instance_feature.shape) == (rows, c)
                 and instance_feature.stride(1) == 1, f"instance_feature must be a [{rows}, {c}] row view")
    st = L.lib().s4d_dfa_output_proj(features.data_ptr(), rows, weight.data_ptr(), _ptr(bias), _ptr(instance_feature),
                                     0 if instance_feature is None else instance_feature.stride(0), mode,
                                     out.data_ptr(), out.stride(0), c, _ptr(error_flag), _stream_ptr(dev))
    L.check(name, st)
    return out


def output_proj_sum_into(out: Tensor, features: Tensor, features2_ptr: int, row0: int, rows: int, weight: Tensor,
                         bias: Optional[Tensor], instance_feature: Optional[Tensor] = None,
                         residual_mode: str = "cat", error_flag: Optional[Tensor] = None) -> Tensor:
    """``output_proj_into`` of ``(features + features2)[row0 : row0 + rows]``: both sources are
    ``[R, C]`` contiguous fp32; ``features2_ptr`` is the device address of the second one, which
    may be a peer GPU's buffer (``PeerPartialSums``), read by the kernel over NVLink.  ``out`` and
    ``instance_feature`` hold the ``rows`` output rows."""
    name = "output_proj_sum"
    mode = RESIDUAL_MODES[residual_mode]
    dev = _require_cuda(name, out, features, weight, bias, instance_feature, error_flag)
    _check_contig(name, features=features, weight=weight, bias=bias)
    for k, t in (("out", out), ("features", features), ("weight", weight), ("bias", bias),
                 ("instance_feature", instance_feature)):
        _check_dtype(name, t, (torch.float32,), k)
    _check_dtype(name, error_flag, (torch.int32,), "error_flag")
    total, c = features.shape
    _require(tuple(weight.shape) == (c, c), lambda: f"weight must be [{c}, {c}]")
    _require(out.dim() == 2 and out.shape[0] == rows and out.stride(1) == 1,
             lambda: f"out must be a [{rows}, n] row view")
    if mode != L.S4D_RESIDUAL_NONE:
        _require(instance_feature is not None and tuple(instance_feature.shape) == (rows, c)
                 and instance_feature.stride(1) == 1, f"instance_feature must be a [{rows}, {c}] row view")
    st = L.lib().s4d_dfa_output_proj_sum(features.data_ptr(), int(features2_ptr), total, row0, rows,
                                         weight.data_ptr(), _ptr(bias), _ptr(instance_feature),
                                         0 if instance_feature is None else instance_feature.stride(0), mode,
                                         out.data_ptr(), out.stride(0), c, _ptr(error_flag), _stream_ptr(dev))
    L.check(name, st)
    return out


LAYER_NORM_WIDTHS = (32, 64, 128, 256, 512)


def layer_norm(x: Tensor, weight: Optional[Tensor], bias: Optional[Tensor], eps: float = 1e-5,
               out: Optional[Tensor] = None) -> Tensor:
    """LayerNorm of ``x [..., width]`` (fp32, contiguous) over its last dimension on this library's
    warp-per-row kernel (``s4d_layer_norm``); ``width`` in ``LAYER_NORM_WIDTHS``."""
    name = "layer_norm"
    dev = _require_cuda(name, x, weight, bias, out)
    width = int(x.shape[-1])
    _require(width in LAYER_NORM_WIDTHS, lambda: f"{name}: width must be one of {LAYER_NORM_WIDTHS}, got {width}")
    _check_contig(name, x=x, weight=weight, bias=bias, out=out)
    for k, t in (("x", x), ("weight", weight), ("bias", bias), ("out", out)):
        _check_dtype(name, t, (torch.float32,), k)
    if out is None:
        out = torch.empty_like(x)
    _require(out.shape == x.shape, lambda: f"{name}: out must be {tuple(x.shape)}")
    st = L.lib().s4d_layer_norm(x.data_ptr(), _ptr(weight), _ptr(bias), out.data_ptr(), x.numel() // width, width,
                                float(eps), _stream_ptr(dev))
    L.check(name, st)
    return out


# ---------------------------------------------------------------------------------------------
# deformable_aggregation
# ---------------------------------------------------------------------------------------------

def _dfa_dims(sample_location: Tensor, weights: Tensor, weights_cam: Optional[Tensor], layout: int):
    if layout == L.S4D_LAYOUT_CAM_MAJOR:
        _require(sample_location.dim() == 5 and sample_location.shape[-1] == 2,
                 "sample_location must be [bs, A, Ncam, P, 2] (cam_major)")
        bs, A, nc, P = sample_location.shape[:4]
        if weights_cam is None:
            _require(weights.dim() == 6 and tuple(weights.shape[:3]) == (bs, A, nc) and weights.shape[4] == P,
                     "weights must be [bs, A, Ncam, L, P, G] (cam_major)")
            nl, G = weights.shape[3], weights.shape[5]
        else:
            _require(weights.dim() == 5 and tuple(weights.shape[:2]) == (bs, A) and weights.shape[3] == P,
                     "split weights must be [bs, A, L, P, G]")
            nl, G = weights.shape[2], weights.shape[4]
            _require(tuple(weights_cam.shape) == (bs, nc, nl, P, G), "weights_cam must be [bs, Ncam, L, P, G]")
    else:
        _require(sample_location.dim() == 5 and sample_location.shape[-1] == 2,
                 "sample_location must be [bs, A, P, Ncam, 2] (pt_major)")
        bs, A, P, nc = sample_location.shape[:4]
        _require(weights.dim() == 6 and tuple(weights.shape[:4]) == (bs, A, P, nc),
                 "weights must be [bs, A, P, Ncam, L, G] (pt_major)")
        nl, G = weights.shape[4], weights.shape[5]
    return int(bs), int(A), int(nc), int(nl), int(P), int(G)


def deformable_aggregation_into(out: Tensor, mc_ms_feat: Tensor, spatial_shape: Tensor, scale_start_index: Tensor,
                                sample_location: Tensor, weights: Tensor, weights_are_logits: bool = True,
                                weights_cam: Optional[Tensor] = None, cam_begin: int = 0, cam_end: int = -1,
                                layout: Union[int, str] = "cam_major", error_flag: Optional[Tensor] = None,
                                workspace: Optional[Tensor] = None, factors_ready: bool = False) -> Tensor:
    """Writes the fused gather into ``out [bs, A, C]`` (fp32) and returns it.  With split
    logits (``weights_cam``) an optional ``workspace`` of ``dfa_workspace_bytes(...)`` bytes
    lets the kernel factorise the softmax; ``factors_ready=True`` says ``camera_factors_into``
    already wrote the factors there (the gather call then launches no factor kernel)."""
    name = "deformable_aggregation"
    lay = LAYOUTS[layout] if isinstance(layout, str) else int(layout)
    dev = _require_cuda(name, out, mc_ms_feat, spatial_shape, scale_start_index, sample_location, weights,
                        weights_cam, error_flag)
    _check_contig(name, out=out, mc_ms_feat=mc_ms_feat, spatial_shape=spatial_shape,
                  scale_start_index=scale_start_index, sample_location=sample_location, weights=weights,
                  weights_cam=weights_cam)
    _check_dtype(name, mc_ms_feat, (torch.float32, torch.bfloat16), "mc_ms_feat")
    _check_dtype(name, spatial_shape, (torch.int32,), "spatial_shape")
    _check_dtype(name, scale_start_index, (torch.int32,), "scale_start_index")
    for k, t in (("sample_location", sample_location), ("weights", weights), ("weights_cam", weights_cam),
                 ("out", out)):
        _check_dtype(name, t, (torch.float32,), k)
    _check_dtype(name, error_flag, (torch.int32,), "error_flag")
    _require(mc_ms_feat.dim() == 3, "mc_ms_feat must be [bs, num_feat, C]")
    bs, A, nc, nl, P, G = _dfa_dims(sample_location, weights, weights_cam, lay)
    C = int(mc_ms_feat.shape[2])
    _require(int(mc_ms_feat.shape[0]) == bs, "mc_ms_feat batch must match sample_location")
    _require(tuple(spatial_shape.shape) == (nc, nl, 2), lambda: f"spatial_shape must be [{nc}, {nl}, 2]")
    _require(tuple(scale_start_index.shape) == (nc, nl), lambda: f"scale_start_index must be [{nc}, {nl}]")
    _require(tuple(out.shape) == (bs, A, C), lambda: f"out must be [{bs}, {A}, {C}]")
    ce = nc if cam_end is None or cam_end < 0 else int(cam_end)
    _require_cuda(name, workspace)
    ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
    st = L.lib().s4d_deformable_aggregation(
        mc_ms_feat.data_ptr(), L.S4D_DTYPE_BF16 if mc_ms_feat.dtype == torch.bfloat16 else L.S4D_DTYPE_F32,
        int(mc_ms_feat.shape[1]), spatial_shape.data_ptr(), scale_start_index.data_ptr(),
        sample_location.data_ptr(), weights.data_ptr(), _ptr(weights_cam),
        (2 if factors_ready else 1) if weights_are_logits else 0, lay,
        bs, A, nc, nl, P, G, C, int(cam_begin), ce, out.data_ptr(), _ptr(error_flag), _ptr(workspace), ws_bytes,
        _stream_ptr(dev))
    L.check(name, st)
    return out


def deformable_aggregation_anchors_into(out: Tensor, mc_ms_feat: Tensor, spatial_shape: Tensor,
                                        scale_start_index: Tensor, anchor: Tensor, fix_scale: Tensor,
                                        learnable: Optional[Tensor], projection_mat: Tensor, image_wh: Tensor,
                                        weights: Tensor, weights_cam: Tensor, workspace: Tensor, cam_begin: int = 0,
                                        cam_end: int = -1, error_flag: Optional[Tensor] = None,
                                        out_peer: Optional[int] = None,
                                        peer_rows: Tuple[int, int] = (0, 0)) -> Tensor:
    """``deformable_aggregation_into`` with the sample locations computed inside the gather from
    ``anchor [bs, A, D]``, ``fix_scale [num_fix, 3]``, the keypoint logits ``learnable [bs*A,
    (P - num_fix)*3]``, ``projection_mat [bs, Ncam, 4, 4]`` and ``image_wh [bs, Ncam, 2]``
    (the same (u, v) as ``kps_project_into``), for split logits whose camera factors
    ``camera_factors_into`` already wrote into ``workspace``.

    ``out_peer`` (a device address, e.g. another GPU's buffer mapped by ``PeerPartialSums``) and
    ``peer_rows = (begin, end)``: the flattened rows in ``[begin, end)`` are written to
    ``out_peer`` (``[bs*A, C]`` rows, the same indexing as ``out``) instead of ``out``."""
    name = "deformable_aggregation_anchors"
    dev = _require_cuda(name, out, mc_ms_feat, spatial_shape, scale_start_index, anchor, fix_scale, learnable,
                        projection_mat, image_wh, weights, weights_cam, workspace, error_flag)
    _check_contig(name, out=out, mc_ms_feat=mc_ms_feat, spatial_shape=spatial_shape,
                  scale_start_index=scale_start_index, anchor=anchor, fix_scale=fix_scale, learnable=learnable,
                  projection_mat=projection_mat, image_wh=image_wh, weights=weights, weights_cam=weights_cam,
                  workspace=workspace)
    _check_dtype(name, mc_ms_feat, (torch.float32, torch.bfloat16), "mc_ms_feat")
    _check_dtype(name, spatial_shape, (torch.int32,), "spatial_shape")
    _check_dtype(name, scale_start_index, (torch.int32,), "scale_start_index")
    for k, t in (("anchor", anchor), ("fix_scale", fix_scale), ("learnable", learnable),
                 ("projection_mat", projection_mat), ("image_wh", image_wh), ("weights", weights),
                 ("weights_cam", weights_cam), ("out", out)):
        _check_dtype(name, t, (torch.float32,), k)
    _check_dtype(name, error_flag, (torch.int32,), "error_flag")
    _require(mc_ms_feat.dim() == 3 and weights_cam.dim() == 5, "mc_ms_feat [bs, num_feat, C], weights_cam "
             "[bs, Ncam, L, P, G]")
    bs, nc, nl, P, G = (int(v) for v in weights_cam.shape)
    A = int(out.shape[1])
    C = int(mc_ms_feat.shape[2])
    _require(tuple(out.shape) == (bs, A, C), lambda: f"out must be [{bs}, A, {C}]")
    _require(anchor.numel() == bs * A * int(anchor.shape[-1]), "anchor must be [bs, A, D]")
    _require(tuple(projection_mat.shape[-2:]) == (4, 4) and projection_mat.numel() == bs * nc * 16,
             f"projection_mat must be [{bs}, {nc}, 4, 4]")
    _require(image_wh.numel() == bs * nc * 2, lambda: f"image_wh must be [{bs}, {nc}, 2]")
    num_fix = int(fix_scale.shape[0])
    _require(learnable is None or learnable.numel() == bs * A * (P - num_fix) * 3,
             f"learnable must hold {(P - num_fix) * 3} logits per anchor")
    ce = nc if cam_end is None or cam_end < 0 else int(cam_end)
    pb, pe = (int(v) for v in peer_rows)
    st = L.lib().s4d_deformable_aggregation_anchors_peer(
        mc_ms_feat.data_ptr(), L.S4D_DTYPE_BF16 if mc_ms_feat.dtype == torch.bfloat16 else L.S4D_DTYPE_F32,
        int(mc_ms_feat.shape[1]), spatial_shape.data_ptr(), scale_start_index.data_ptr(), anchor.data_ptr(),
        int(anchor.shape[-1]), fix_scale.data_ptr(), num_fix, _ptr(learnable), projection_mat.data_ptr(),
        image_wh.data_ptr(), weights.data_ptr(), weights_cam.data_ptr(), bs, A, nc, nl, P, G, C, int(cam_begin), ce,
        out.data_ptr(), None if out_peer is None else int(out_peer), pb, pe, _ptr(error_flag), workspace.data_ptr(),
        workspace.numel() * workspace.element_size(), _stream_ptr(dev))
    L.check(name, st)
    return out


def dfa_workspace_bytes(bs: int, num_cams: int, num_levels: int, num_pts: int, num_groups: int,
                        split_logits: bool) -> int:
    return int(L.lib().s4d_dfa_workspace_bytes(bs, num_cams, num_levels, num_pts, num_groups,
                                               1 if split_logits else 0))


def camera_factors_into(workspace: Tensor, weights_cam: Tensor) -> Tensor:
    """The per-frame camera softmax factors of split logits ``weights_cam [bs, Ncam, L, P, G]``
    into ``workspace`` (from ``dfa_workspace``), for ``deformable_aggregation_into(...,
    workspace=workspace, factors_ready=True)``."""
    name = "camera_factors"
    dev = _require_cuda(name, workspace, weights_cam)
    _check_contig(name, workspace=workspace, weights_cam=weights_cam)
    _check_dtype(name, weights_cam, (torch.float32,), "weights_cam")
    _require(weights_cam.dim() == 5, "weights_cam must be [bs, Ncam, L, P, G]")
    bs, nc, nl, npt, g = (int(v) for v in weights_cam.shape)
    st = L.lib().s4d_dfa_camera_factors(weights_cam.data_ptr(), bs, nc, nl, npt, g, workspace.data_ptr(),
                                        workspace.numel() * workspace.element_size(), _stream_ptr(dev))
    L.check(name, st)
    return workspace


def dfa_workspace(bs: int, num_cams: int, num_levels: int, num_pts: int, num_groups: int,
                  device) -> Optional[Tensor]:
    """A workspace tensor for split-logit calls (None when no workspace is needed)."""
    n = dfa_workspace_bytes(bs, num_cams, num_levels, num_pts, num_groups, True)
    return torch.empty(n // 4, dtype=torch.float32, device=device) if n else None


@torch.library.custom_op("s4d::deformable_aggregation", mutates_args=())
def deformable_aggregation(mc_ms_feat: Tensor, spatial_shape: Tensor, scale_start_index: Tensor,
                           sample_location: Tensor, weights: Tensor, weights_are_logits: bool = True,
                           weights_cam: Optional[Tensor] = None, cam_begin: int = 0, cam_end: int = -1,
                           layout: int = 0) -> Tensor:
    """Fused softmax (when ``weights_are_logits``) + bilinear gather + weighted sum.

    ``mc_ms_feat [bs, num_feat, C]`` channels-last (f32 or bf16); ``spatial_shape [Ncam, L, 2]``
    and ``scale_start_index [Ncam, L]`` int32; ``sample_location`` / ``weights`` in
    ``layout`` 0 (cam-major, native: ``[bs, A, Ncam, P, 2]`` / ``[bs, A, Ncam, L, P, G]``) or 1
    (pt-major, upstream Sparse4D: ``[bs, A, P, Ncam, 2]`` / ``[bs, A, P, Ncam, L, G]``).
    Returns ``[bs, A, C]`` fp32 summed over points."""
    bs, A = sample_location.shape[:2]
    out = torch.empty(bs, A, mc_ms_feat.shape[2], dtype=torch.float32, device=mc_ms_feat.device)
    ws = None
    if weights_cam is not None:
        nc, nl, P, G = weights_cam.shape[1:5]
        ws = dfa_workspace(bs, nc, nl, P, G, mc_ms_feat.device)
    return deformable_aggregation_into(out, mc_ms_feat, spatial_shape, scale_start_index, sample_location, weights,
                                       weights_are_logits, weights_cam, cam_begin, cam_end, layout, workspace=ws)


@deformable_aggregation.register_fake
def _(mc_ms_feat, spatial_shape, scale_start_index, sample_location, weights, weights_are_logits=True,
      weights_cam=None, cam_begin=0, cam_end=-1, layout=0):
    bs, A = sample_location.shape[:2]
    return mc_ms_feat.new_empty(bs, A, mc_ms_feat.shape[2], dtype=torch.float32)


# ---------------------------------------------------------------------------------------------
# kps_project
# ---------------------------------------------------------------------------------------------

def kps_workspace_bytes(bs: int, num_anchor: int, num_cams: int, num_pts: int) -> int:
    return int(L.lib().s4d_kps_workspace_bytes(bs, num_anchor, num_cams, num_pts))


def kps_project_into(anchor: Tensor, learnable_logits: Optional[Tensor], fix_scale: Optional[Tensor],
                     projection_mat: Tensor, image_wh: Tensor, sample_location: Optional[Tensor] = None,
                     depth_mask: Optional[Tensor] = None, visible_idx: Optional[Tensor] = None,
                     visible_count: Optional[Tensor] = None, key_points: Optional[Tensor] = None,
                     workspace: Optional[Tensor] = None, layout: Union[int, str] = "cam_major") -> None:
    """Runs the keypoint kernel into caller-provided outputs (any may be None)."""
    name = "kps_project"
    lay = LAYOUTS[layout] if isinstance(layout, str) else int(layout)
    dev = _require_cuda(name, anchor, learnable_logits, fix_scale, projection_mat, image_wh, sample_location,
                        depth_mask, visible_idx, visible_count, key_points, workspace)
    _check_contig(name, anchor=anchor, learnable_logits=learnable_logits, fix_scale=fix_scale,
                  projection_mat=projection_mat, image_wh=image_wh, sample_location=sample_location,
                  depth_mask=depth_mask, visible_idx=visible_idx, key_points=key_points)
    for k, t in (("anchor", anchor), ("learnable_logits", learnable_logits), ("fix_scale", fix_scale),
                 ("projection_mat", projection_mat), ("image_wh", image_wh), ("sample_location", sample_location),
                 ("key_points", key_points)):
        _check_dtype(name, t, (torch.float32,), k)
    _check_dtype(name, depth_mask, (torch.uint8, torch.bool), "depth_mask")
    _check_dtype(name, visible_idx, (torch.int32,), "visible_idx")
    _check_dtype(name, visible_count, (torch.int32,), "visible_count")
    _require(anchor.dim() == 3 and anchor.shape[-1] >= 8, "anchor must be [bs, A, >=8]")
    bs, A = int(anchor.shape[0]), int(anchor.shape[1])
    _require(projection_mat.dim() == 4 and projection_mat.shape[0] == bs and tuple(projection_mat.shape[2:]) == (4, 4),
             "projection_mat must be [bs, Ncam, 4, 4]")
    nc = int(projection_mat.shape[1])
    _require(tuple(image_wh.shape) == (bs, nc, 2), "image_wh must be [bs, Ncam, 2]")
    n_fix = 0 if fix_scale is None else int(fix_scale.shape[0])
    if fix_scale is not None:
        _require(fix_scale.dim() == 2 and fix_scale.shape[1] == 3, "fix_scale must be [num_fix, 3]")
    n_learn = 0
    if learnable_logits is not None:
        _require(learnable_logits.dim() == 3 and tuple(learnable_logits.shape[:2]) == (bs, A)
                 and learnable_logits.shape[2] % 3 == 0, "learnable_logits must be [bs, A, 3 * num_learnable]")
        n_learn = int(learnable_logits.shape[2]) // 3
    P = n_fix + n_learn
    if sample_location is not None:
        exp = (bs, A, nc, P, 2) if lay == L.S4D_LAYOUT_CAM_MAJOR else (bs, A, P, nc, 2)
        _require(tuple(sample_location.shape) == exp, lambda: f"sample_location must be {list(exp)}")
    if depth_mask is not None:
        _require(tuple(depth_mask.shape) == (bs, A, nc, P), lambda: f"depth_mask must be [{bs}, {A}, {nc}, {P}]")
    if key_points is not None:
        _require(tuple(key_points.shape) == (bs, A, P, 3), lambda: f"key_points must be [{bs}, {A}, {P}, 3]")
    if visible_idx is not None:
        _require(tuple(visible_idx.shape) == (bs * A * nc * P, 4), "visible_idx must be [bs*A*Ncam*P, 4]")
    ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
    st = L.lib().s4d_kps_project(
        anchor.data_ptr(), int(anchor.shape[2]), _ptr(fix_scale), n_fix, _ptr(learnable_logits), n_learn,
        projection_mat.data_ptr(), image_wh.data_ptr(), bs, A, nc, lay, _ptr(key_points), _ptr(sample_location),
        _ptr(depth_mask), _ptr(visible_idx), _ptr(visible_count), _ptr(workspace), ws_bytes, _stream_ptr(dev))
    L.check(name, st)


def kps_project_linear_into(anchor: Tensor, instance_feature: Tensor, learnable_fc_weight: Tensor,
                            learnable_fc_bias: Optional[Tensor], fix_scale: Optional[Tensor], projection_mat: Tensor,
                            image_wh: Tensor, sample_location: Optional[Tensor] = None,
                            depth_mask: Optional[Tensor] = None, key_points: Optional[Tensor] = None,
                            layout: Union[int, str] = "cam_major", visible_idx: Optional[Tensor] = None,
                            visible_count: Optional[Tensor] = None, workspace: Optional[Tensor] = None) -> None:
    """``kps_project_into`` with the learnable keypoint logits computed inside the kernel from
    ``instance_feature`` (a ``[bs*A, C]`` row view, see ``row_view``) and the keypoint
    generator's ``learnable_fc`` weight/bias (fp32), so the call needs no other linear first.
    ``visible_idx`` / ``visible_count`` (with a ``workspace`` of ``kps_workspace_bytes``) ask
    for the compacted visible indices as in ``kps_project_into``."""
    name = "kps_project_linear"
    lay = LAYOUTS[layout] if isinstance(layout, str) else int(layout)
    dev = _require_cuda(name, anchor, instance_feature, learnable_fc_weight, learnable_fc_bias, fix_scale,
                        projection_mat, image_wh, sample_location, depth_mask, key_points, visible_idx, visible_count,
                        workspace)
    _check_contig(name, anchor=anchor, learnable_fc_weight=learnable_fc_weight, learnable_fc_bias=learnable_fc_bias,
                  fix_scale=fix_scale, projection_mat=projection_mat, image_wh=image_wh,
                  sample_location=sample_location, depth_mask=depth_mask, key_points=key_points,
                  visible_idx=visible_idx)
    for k, t in (("anchor", anchor), ("instance_feature", instance_feature), ("learnable_fc_weight", learnable_fc_weight),
                 ("learnable_fc_bias", learnable_fc_bias), ("fix_scale", fix_scale), ("projection_mat", projection_mat),
                 ("image_wh", image_wh), ("sample_location", sample_location), ("key_points", key_points)):
        _check_dtype(name, t, (torch.float32,), k)
    _check_dtype(name, depth_mask, (torch.uint8, torch.bool), "depth_mask")
    _check_dtype(name, visible_idx, (torch.int32,), "visible_idx")
    _check_dtype(name, visible_count, (torch.int32,), "visible_count")
    _require(anchor.dim() == 3 and anchor.shape[-1] >= 8, "anchor must be [bs, A, >=8]")
    bs, A = int(anchor.shape[0]), int(anchor.shape[1])
    _require(projection_mat.dim() == 4 and projection_mat.shape[0] == bs and tuple(projection_mat.shape[2:]) == (4, 4),
             "projection_mat must be [bs, Ncam, 4, 4]")
    nc = int(projection_mat.shape[1])
    _require(tuple(image_wh.shape) == (bs, nc, 2), "image_wh must be [bs, Ncam, 2]")
    n_fix = 0 if fix_scale is None else int(fix_scale.shape[0])
    m3, c = (int(v) for v in learnable_fc_weight.shape)
    _require(m3 % 3 == 0, "learnable_fc_weight must be [3 * num_learnable, C]")
    _require(instance_feature.dim() == 2 and tuple(instance_feature.shape) == (bs * A, c)
             and instance_feature.stride(1) == 1, f"instance_feature must be a [{bs * A}, {c}] row view")
    P = n_fix + m3 // 3
    if sample_location is not None:
        exp = (bs, A, nc, P, 2) if lay == L.S4D_LAYOUT_CAM_MAJOR else (bs, A, P, nc, 2)
        _require(tuple(sample_location.shape) == exp, lambda: f"sample_location must be {list(exp)}")
    if depth_mask is not None:
        _require(tuple(depth_mask.shape) == (bs, A, nc, P), lambda: f"depth_mask must be [{bs}, {A}, {nc}, {P}]")
    if key_points is not None:
        _require(tuple(key_points.shape) == (bs, A, P, 3), lambda: f"key_points must be [{bs}, {A}, {P}, 3]")
    if visible_idx is not None:
        _require(tuple(visible_idx.shape) == (bs * A * nc * P, 4), "visible_idx must be [bs*A*Ncam*P, 4]")
    ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
    st = L.lib().s4d_kps_project_linear(
        anchor.data_ptr(), int(anchor.shape[2]), _ptr(fix_scale), n_fix, instance_feature.data_ptr(),
        instance_feature.stride(0), learnable_fc_weight.data_ptr(), _ptr(learnable_fc_bias), m3 // 3, c,
        projection_mat.data_ptr(), image_wh.data_ptr(), bs, A, nc, lay, _ptr(key_points), _ptr(sample_location),
        _ptr(depth_mask), _ptr(visible_idx), _ptr(visible_count), _ptr(workspace), ws_bytes, _stream_ptr(dev))
    L.check(name, st)


@torch.library.custom_op("s4d::kps_project", mutates_args=())
def kps_project(anchor: Tensor, learnable_logits: Optional[Tensor], fix_scale: Tensor, projection_mat: Tensor,
                image_wh: Tensor, layout: int = 0) -> Tuple[Tensor, Tensor, Tensor, Tensor, Tensor]:
    """Keypoints + projection + masks + compaction.

    Returns ``(sample_location, depth_mask, visible_idx, visible_count, key_points)``:
    ``sample_location [bs, A, Ncam, P, 2]`` (layout 0) or ``[bs, A, P, Ncam, 2]`` (layout 1),
    ``depth_mask [bs, A, Ncam, P]`` uint8, ``visible_idx [bs*A*Ncam*P, 4]`` int32 whose first
    ``visible_count[0]`` rows are the visible (b, a, cam, pt) in lexicographic order, and
    ``key_points [bs, A, P, 3]``."""
    bs, A = anchor.shape[:2]
    nc = projection_mat.shape[1]
    P = fix_scale.shape[0] + (0 if learnable_logits is None else learnable_logits.shape[2] // 3)
    dev = anchor.device
    loc_shape = (bs, A, nc, P, 2) if layout == L.S4D_LAYOUT_CAM_MAJOR else (bs, A, P, nc, 2)
    loc = torch.empty(loc_shape, dtype=torch.float32, device=dev)
    mask = torch.empty(bs, A, nc, P, dtype=torch.uint8, device=dev)
    idx = torch.empty(bs * A * nc * P, 4, dtype=torch.int32, device=dev)
    cnt = torch.zeros(1, dtype=torch.int32, device=dev)
    kp = torch.empty(bs, A, P, 3, dtype=torch.float32, device=dev)
    ws = torch.empty(max(kps_workspace_bytes(bs, A, nc, P), 16), dtype=torch.uint8, device=dev)
    kps_project_into(anchor, learnable_logits, fix_scale, projection_mat, image_wh, loc, mask, idx, cnt, kp, ws,
                     layout)
    return loc, mask, idx, cnt, kp


@kps_project.register_fake
def _(anchor, learnable_logits, fix_scale, projection_mat, image_wh, layout=0):
    bs, A = anchor.shape[:2]
    nc = projection_mat.shape[1]
    P = fix_scale.shape[0] + (0 if learnable_logits is None else learnable_logits.shape[2] // 3)
    loc_shape = (bs, A, nc, P, 2) if layout == 0 else (bs, A, P, nc, 2)
    return (anchor.new_empty(loc_shape), anchor.new_empty(bs, A, nc, P, dtype=torch.uint8),
            anchor.new_empty(bs * A * nc * P, 4, dtype=torch.int32), anchor.new_empty(1, dtype=torch.int32),
            anchor.new_empty(bs, A, P, 3))


def visible_indices(visible_idx: Tensor, visible_count: Tensor) -> Tensor:
    """The valid rows of ``visible_idx`` (synchronises to read the count)."""
    return visible_idx[: int(visible_count.item())]


def kps_project_fused(key_points: Tensor, anchor: Tensor, projection_mat: Tensor, image_wh: Tensor, num_cams: int,
                      num_pts: int) -> Tensor:
    """``ttnn.kps_project_fused`` standard mode: ``key_points [n, P, 3]`` pre-rotation,
    ``anchor [n, 1, 11]``, ``projection_mat [Ncam, 4, 4]``, ``image_wh [Ncam, 1, 2]`` ->
    ``[Ncam, n, 1, 2P]`` holding ``clamp(2 * uv - 1, -2, 2)``."""
    name = "kps_project_fused"
    dev = _require_cuda(name, key_points, anchor, projection_mat, image_wh)
    for k, t in (("key_points", key_points), ("anchor", anchor), ("projection_mat", projection_mat),
                 ("image_wh", image_wh)):
        _check_dtype(name, t, (torch.float32,), k)
    _require(key_points.dim() == 3 and key_points.shape[1] == num_pts and key_points.shape[2] == 3,
             "key_points must be [n, num_pts, 3]")
    n = int(key_points.shape[0])
    anchor2 = anchor.reshape(n, -1).contiguous()
    proj = projection_mat.reshape(num_cams, 4, 4).contiguous()
    wh = image_wh.reshape(num_cams, 2).contiguous()
    kp = key_points.contiguous()
    out = torch.empty(num_cams, n, 1, num_pts * 2, dtype=torch.float32, device=dev)
    st = L.lib().s4d_kps_project_fused(kp.data_ptr(), anchor2.data_ptr(), int(anchor2.shape[1]), proj.data_ptr(),
                                       wh.data_ptr(), n, int(num_cams), int(num_pts), out.data_ptr(),
                                       _stream_ptr(dev))
    L.check(name, st)
    return out


# ---------------------------------------------------------------------------------------------
# feature-map packing
# ---------------------------------------------------------------------------------------------

def level_tables(spatial_shapes: Sequence[Tuple[int, int]], num_cams: int, device=None):
    """``spatial_shape [Ncam, L, 2]`` and ``scale_start_index [Ncam, L]`` (int32) of the packed
    camera-major layout, plus ``num_feat`` (rows per batch item)."""
    hw = [int(h) * int(w) for h, w in spatial_shapes]
    per_cam = sum(hw)
    starts, acc = [], 0
    for v in hw:
        starts.append(acc)
        acc += v
    shape = torch.tensor([[list(s) for s in spatial_shapes]] * num_cams, dtype=torch.int32)
    start = torch.tensor([[c * per_cam + s for s in starts] for c in range(num_cams)], dtype=torch.int32)
    if device is not None:
        shape, start = shape.to(device), start.to(device)
    return shape, start, per_cam * num_cams


def pack_feature_maps(feature_maps: List[Tensor], dtype: Optional[torch.dtype] = None, channels_last: bool = False,
                      out: Optional[Tensor] = None):
    """Pack per-level maps into ``(mc_ms_feat [bs, Ncam*sum(HW), C], spatial_shape,
    scale_start_index)`` with one kernel launch per level (``s4d_pack_feature_maps``: a tiled
    transpose for NCHW maps, a vector copy for channels-last ones, the cast to ``dtype`` fused
    in).  Maps are NCHW ``[bs, Ncam, C, H, W]`` (the oracle's format), or with
    ``channels_last=True`` ``[bs, Ncam, H, W, C]``; fp32 or bf16.  ``out`` may be a
    preallocated ``mc_ms_feat``."""
    name = "pack_feature_maps"
    maps = [f if f.is_contiguous() else f.contiguous() for f in feature_maps]
    dev = _require_cuda(name, *maps, out)
    _require(len(maps) > 0, lambda: f"{name}: no maps")
    for f in maps:
        _check_dtype(name, f, (torch.float32, torch.bfloat16), "feature map")
        _require(f.dtype == maps[0].dtype and f.dim() == 5, lambda: f"{name}: maps must be 5-D and share one dtype")
    bs, nc = int(maps[0].shape[0]), int(maps[0].shape[1])
    if channels_last:
        shapes = [(int(f.shape[2]), int(f.shape[3])) for f in maps]
        c = int(maps[0].shape[4])
        _require(all(tuple(f.shape[:2]) == (bs, nc) and f.shape[4] == c for f in maps),
                 lambda: f"{name}: inconsistent maps")
    else:
        shapes = [(int(f.shape[3]), int(f.shape[4])) for f in maps]
        c = int(maps[0].shape[2])
        _require(all(tuple(f.shape[:3]) == (bs, nc, c) for f in maps), lambda: f"{name}: inconsistent maps")
    dtype = dtype or maps[0].dtype
    _check_dtype(name, torch.empty(0, dtype=dtype), (torch.float32, torch.bfloat16), "dtype")
    rows = nc * sum(h * w for h, w in shapes)
    if out is None:
        out = torch.empty(bs, rows, c, dtype=dtype, device=dev)
    _require(tuple(out.shape) == (bs, rows, c) and out.dtype == dtype and out.is_contiguous(),
             f"{name}: out must be a contiguous [{bs}, {rows}, {c}] {dtype} tensor")
    ptrs = (C.c_void_p * len(maps))(*[f.data_ptr() for f in maps])
    hw = (C.c_int32 * (2 * len(maps)))(*[v for s_ in shapes for v in s_])
    code = lambda t: L.S4D_DTYPE_BF16 if t == torch.bfloat16 else L.S4D_DTYPE_F32  # noqa: E731
    st = L.lib().s4d_pack_feature_maps(ptrs, L.S4D_MAPS_NHWC if channels_last else L.S4D_MAPS_NCHW,
                                       code(maps[0].dtype), bs, nc, len(maps), hw, c, code(dtype), out.data_ptr(),
                                       _stream_ptr(dev))
    L.check(name, st)
    shape, start, _ = level_tables(shapes, nc, device=dev)
    return out, shape, start
