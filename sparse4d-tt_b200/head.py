"""Sparse4D v3 decoder head around the DFA hot path, on the GPU, capturable as one CUDA graph.

The decoder of ``model/sparse4d_head.py:356-461`` (single frame: the instance bank's anchors
and zero instance features, no temporal instances) runs its operation order

    deformable, ffn, norm, refine, then 5 x (temp_gnn, gnn, norm, deformable, ffn, norm, refine)

with the anchors kept on the device from layer to layer: every ``refine`` moves them and the
anchor encoder re-embeds them for the next layer (``:419-461``).  The DFA layers are this
package's ``DeformableFeatureAggregation`` (the hand-written kernels); the dense layers around
them -- decoupled multi-head attention (``model/multihead_attention.py``), the asymmetric FFN
(``model/asymmetric_ffn.py``), LayerNorm, the refinement MLPs (``model/refinement_module.py``) and
the anchor encoder (``model/sparse_box3d_encoder.py``) -- are torch operations (cuBLAS, SDPA),
as the reference runs them through TT-NN matmuls.

``Sparse4DHead.forward`` launches only device work (no host synchronisation), so
``graph.capture`` records a whole decoder pass; ``HeadGraph`` does that over static inputs.
"""
from __future__ import annotations

import contextlib
from typing import Dict, List, Optional, Sequence, Tuple

import torch
import torch.nn.functional as F

from . import ops
from .dfa import MATMUL_PRECISIONS, DeformableFeatureAggregation, _matmul_precision, preprocess_dfa_parameters
from .graph import capture, chained_camera_terms

Tensor = torch.Tensor

X, Y, Z = 0, 1, 2
W, L, H = 3, 4, 5
SIN_YAW, COS_YAW = 6, 7
VX = 8


def _mlp_params(seq) -> List[Tuple[str, Tensor, Tensor]]:
    """(kind, weight, bias) of a Sequential of Linear / ReLU / LayerNorm / Scale modules."""
    out = []
    for m in seq:
        name = type(m).__name__
        if isinstance(m, torch.nn.Linear):
            out.append(("linear", m.weight.data.clone(), None if m.bias is None else m.bias.data.clone()))
        elif isinstance(m, torch.nn.LayerNorm):
            out.append(("ln", m.weight.data.clone(), m.bias.data.clone()))
        elif isinstance(m, torch.nn.ReLU):
            out.append(("relu", None, None))
        elif hasattr(m, "scale"):
            out.append(("scale", m.scale.data.clone(), None))
        elif name == "Dropout":
            continue
        else:
            raise TypeError(f"unexpected module {name} in an MLP")
    return out


def preprocess_head_parameters(pt_head) -> Dict:
    """Parameter dictionary of a single-frame Sparse4D head module with the structure of the
    reference's head twin (``test/sparse4d_head_pcc.py:287-330``: ``operation_order``,
    ``layers``, ``anchor_encoder``, ``anchor``, ``instance_feature``, ``fc_before`` / ``fc_after``)."""
    layers = []
    for op, m in zip(pt_head.operation_order, pt_head.layers):
        if op in ("gnn", "temp_gnn"):
            a = m.attn
            layers.append({"in_proj_weight": a.in_proj_weight.data.clone(), "in_proj_bias": a.in_proj_bias.data.clone(),
                           "out_proj_weight": a.out_proj.weight.data.clone(),
                           "out_proj_bias": a.out_proj.bias.data.clone(), "num_heads": a.num_heads})
        elif op == "norm":
            layers.append({"weight": m.weight.data.clone(), "bias": m.bias.data.clone()})
        elif op == "deformable":
            layers.append(preprocess_dfa_parameters(m))
        elif op == "ffn":
            layers.append({"pre_norm": (m.pre_norm.weight.data.clone(), m.pre_norm.bias.data.clone()),
                           "fc1": (m.layers[0][0].weight.data.clone(), m.layers[0][0].bias.data.clone()),
                           "fc2": (m.layers[1].weight.data.clone(), m.layers[1].bias.data.clone()),
                           "identity_fc": (m.identity_fc.weight.data.clone(), m.identity_fc.bias.data.clone())})
        elif op == "refine":
            layers.append({"layers": _mlp_params(m.layers), "cls_layers": _mlp_params(m.cls_layers),
                           "quality_layers": _mlp_params(m.quality_layers)})
        else:
            raise ValueError(f"unknown operation {op}")
    enc = pt_head.anchor_encoder
    encoder = {k: _mlp_params(getattr(enc, k)) for k in ("pos_fc", "size_fc", "yaw_fc", "vel_fc")}
    return {"operation_order": list(pt_head.operation_order), "layers": layers, "anchor_encoder": encoder,
            "anchor": pt_head.anchor.data.clone(), "instance_feature": pt_head.instance_feature.data.clone(),
            "fc_before": pt_head.fc_before.weight.data.clone(), "fc_after": pt_head.fc_after.weight.data.clone(),
            "num_single_frame_decoder": int(getattr(pt_head, "num_single_frame_decoder", 1))}


def _to(dev, t):
    return None if t is None else t.detach().to(dev, torch.float32).contiguous()


def _layer_norm(x: Tensor, w: Tensor, b: Tensor) -> Tensor:
    """nn.LayerNorm (eps 1e-5) over the last dimension: this library's warp-per-row kernel for
    the decoder's contiguous fp32 rows of 32 to 512 features, torch's kernel otherwise."""
    if x.dtype == torch.float32 and x.shape[-1] in ops.LAYER_NORM_WIDTHS and x.is_contiguous():
        return ops.layer_norm(x, w, b, 1e-5)
    return F.layer_norm(x, (w.shape[0],), w, b, 1e-5)


def _run_mlp(x: Tensor, mods) -> Tensor:
    for kind, w, b in mods:
        if kind == "linear":
            x = F.linear(x, w, b)
        elif kind == "relu":
            x = F.relu(x)
        elif kind == "ln":
            x = _layer_norm(x, w, b)
        else:  # scale
            x = x * w
    return x


class Sparse4DHead:
    """The single-frame decoder of ``model/sparse4d_head.py`` on ``device``, from
    ``preprocess_head_parameters``.  ``model_config`` goes to every DFA layer
    (``FEATURE_DTYPE``, ``MATMUL_PRECISION``); ``MATMUL_PRECISION`` also sets torch's fp32 matmul
    precision for the dense layers around them.  ``model_config["ATTENTION_DTYPE"]``
    (``torch.float32`` by default, or ``torch.bfloat16``) is the type the attention's softmax(QK^T)V
    runs in: bf16 (the reference's TT-NN attention runs in bf16) uses the flash kernels, about 9x
    faster than the fp32 kernel at 900 tokens, with q, k, v rounded to bf16 and the result
    returned as fp32."""

    def __init__(self, device, parameters: Dict, model_config: Optional[Dict] = None, embed_dims: int = 256,
                 num_groups: int = 8, num_levels: int = 4, num_cams: int = 6, num_learnable_pts: int = 6):
        self.device = torch.device(device if not isinstance(device, int) else f"cuda:{device}")
        self.embed_dims = embed_dims
        self.operation_order = list(parameters["operation_order"])
        self.num_single_frame_decoder = parameters.get("num_single_frame_decoder", 1)
        cfg = dict(model_config or {})
        self.matmul_precision = MATMUL_PRECISIONS[cfg.get("MATMUL_PRECISION", "fp32")]
        self.attention_dtype = cfg.get("ATTENTION_DTYPE", torch.float32)
        if self.attention_dtype not in (torch.float32, torch.bfloat16, torch.float16):
            raise ValueError("ATTENTION_DTYPE must be torch.float32, torch.bfloat16 or torch.float16")
        cfg.pop("ATTENTION_DTYPE", None)  # a head option, not a DFA one
        dev = self.device
        self.layers = []
        for op, p in zip(self.operation_order, parameters["layers"]):
            if op == "deformable":
                self.layers.append(DeformableFeatureAggregation(dev, p, cfg, embed_dims=embed_dims,
                                                                num_groups=num_groups, num_levels=num_levels,
                                                                num_cams=num_cams,
                                                                num_learnable_pts=num_learnable_pts))
            elif op in ("gnn", "temp_gnn"):
                self.layers.append({k: (_to(dev, v) if torch.is_tensor(v) else v) for k, v in p.items()})
            elif op == "norm":
                self.layers.append((_to(dev, p["weight"]), _to(dev, p["bias"])))
            elif op == "ffn":
                self.layers.append({k: (_to(dev, w), _to(dev, b)) for k, (w, b) in p.items()})
            elif op == "refine":
                self.layers.append({k: [(kind, _to(dev, w), _to(dev, b)) for kind, w, b in v] for k, v in p.items()})
        self.encoder = {k: [(kind, _to(dev, w), _to(dev, b)) for kind, w, b in v]
                        for k, v in parameters["anchor_encoder"].items()}
        self.anchor = _to(dev, parameters["anchor"])
        self.instance_feature = _to(dev, parameters["instance_feature"])
        self.fc_before = _to(dev, parameters["fc_before"])
        self.fc_after = _to(dev, parameters["fc_after"])

    # ---- dense pieces --------------------------------------------------------------------------
    def anchor_embed(self, anchor: Tensor) -> Tensor:
        """Anchor encoder (``model/sparse_box3d_encoder.py``): position, size, yaw and velocity
        MLPs, concatenated."""
        e = self.encoder
        return torch.cat([_run_mlp(anchor[..., X:Z + 1], e["pos_fc"]), _run_mlp(anchor[..., W:H + 1], e["size_fc"]),
                          _run_mlp(anchor[..., SIN_YAW:COS_YAW + 1], e["yaw_fc"]),
                          _run_mlp(anchor[..., VX:VX + 3], e["vel_fc"])], dim=-1)

    def _attention(self, p, query: Tensor, value: Optional[Tensor]) -> Tensor:
        """Decoupled self-attention (``model/sparse4d_head.py:_graph_model``): query and key are
        ``[inst, anchor_embed]`` (2C), the value ``fc_before(inst)`` (``gnn``) or the query
        itself (``temp_gnn`` without temporal instances); identity shortcut, then ``fc_after``."""
        bs, n, e = query.shape
        heads = p["num_heads"]
        wq, wk, wv = p["in_proj_weight"].chunk(3, dim=0)
        bq, bk, bv = p["in_proj_bias"].chunk(3, dim=0)
        v_in = query if value is None else value
        q = F.linear(query, wq, bq).view(bs, n, heads, e // heads).transpose(1, 2)
        k = F.linear(query, wk, bk).view(bs, n, heads, e // heads).transpose(1, 2)
        v = F.linear(v_in, wv, bv).view(bs, n, heads, e // heads).transpose(1, 2)
        dt = self.attention_dtype
        if dt == torch.float32:
            o = F.scaled_dot_product_attention(q, k, v)
        else:
            o = F.scaled_dot_product_attention(q.to(dt), k.to(dt), v.to(dt)).float()
        o = o.transpose(1, 2).reshape(bs, n, e)
        out = query + F.linear(o, p["out_proj_weight"], p["out_proj_bias"])
        return F.linear(out, self.fc_after)

    def _ffn(self, p, x: Tensor) -> Tensor:
        """Asymmetric FFN 2C -> C with pre-norm (``model/asymmetric_ffn.py``)."""
        x = _layer_norm(x, *p["pre_norm"])
        return F.linear(x, *p["identity_fc"]) + F.linear(F.relu(F.linear(x, *p["fc1"])), *p["fc2"])

    def _refine(self, p, inst: Tensor, anchor: Tensor, embed: Tensor, time_interval: Tensor, return_cls: bool):
        """Box refinement (``model/refinement_module.py``): centre, size and yaw move by the MLP
        output, velocity by output / time interval; classification and quality when asked."""
        feat = inst + embed
        out = _run_mlp(feat, p["layers"])
        moved = out[..., :VX] + anchor[..., :VX]
        vel = out[..., VX:] / time_interval.view(-1, *([1] * (out.dim() - 1))) + anchor[..., VX:]
        new_anchor = torch.cat([moved, vel], dim=-1)
        cls = _run_mlp(inst, p["cls_layers"]) if return_cls else None
        qt = _run_mlp(feat, p["quality_layers"]) if return_cls else None
        return new_anchor, cls, qt

    # ---- forward ---------------------------------------------------------------------------------
    def forward(self, feature_maps, projection_mat: Tensor, image_wh: Tensor, spatial_shapes: Sequence[Tuple[int, int]],
                bs: int, anchor: Optional[Tensor] = None, instance_feature: Optional[Tensor] = None,
                time_interval: Optional[Tensor] = None) -> Dict[str, List[Optional[Tensor]]]:
        """One decoder pass: per decoder the refined anchors ``[bs, A, 11]`` (``prediction``),
        and for the first and last decoders the class scores ``[bs, A, num_cls]`` and quality
        ``[bs, A, 2]``.  ``feature_maps`` as ``DeformableFeatureAggregation.run`` takes them
        (packed once here when given as per-level maps).  ``anchor`` / ``instance_feature``
        default to the instance bank's (expanded over ``bs``); ``time_interval [bs]`` to 0.5."""
        dev = self.device
        A = self.anchor.shape[0]
        if anchor is None:
            anchor = self.anchor[None].expand(bs, -1, -1)
        anchor = anchor.reshape(bs, A, -1).contiguous()
        inst = (self.instance_feature[None].expand(bs, -1, -1) if instance_feature is None
                else instance_feature.reshape(bs, A, self.embed_dims))
        if time_interval is None:
            time_interval = torch.full((bs,), 0.5, device=dev)
        packed = feature_maps
        if not (isinstance(feature_maps, (tuple, list)) and len(feature_maps) == 3 and torch.is_tensor(feature_maps[1])
                and feature_maps[1].dtype == torch.int32):
            packed = self.layers[self.operation_order.index("deformable")]._features(feature_maps, spatial_shapes, bs)
        for mod, op in zip(self.layers, self.operation_order):
            if op == "deformable":
                mod.reset_frame_cache()  # a new frame: the per-frame camera terms are recomputed
        preds, clss, qts = [], [], []
        last = len(self.operation_order) - 1
        dfas = [p for op, p in zip(self.operation_order, self.layers) if op == "deformable"]
        with _matmul_precision(self.matmul_precision), chained_camera_terms(dfas):
            embed = self.anchor_embed(anchor)
            for i, (op, p) in enumerate(zip(self.operation_order, self.layers)):
                if op == "temp_gnn":
                    inst = self._attention(p, torch.cat([inst, embed], dim=-1), None)
                elif op == "gnn":
                    inst = self._attention(p, torch.cat([inst, embed], dim=-1), F.linear(inst, self.fc_before))
                elif op == "norm":
                    inst = _layer_norm(inst, p[0], p[1])
                elif op == "ffn":
                    inst = self._ffn(p, inst)
                elif op == "deformable":
                    inst = p.run(inst, anchor, embed, packed, projection_mat, image_wh, spatial_shapes, bs, A)
                elif op == "refine":
                    return_cls = len(preds) == self.num_single_frame_decoder - 1 or i == last
                    anchor, cls, qt = self._refine(p, inst, anchor, embed, time_interval, return_cls)
                    preds.append(anchor)
                    clss.append(cls)
                    qts.append(qt)
                    if i != last:
                        embed = self.anchor_embed(anchor)
        return {"prediction": preds, "classification": clss, "quality": qts}

    __call__ = forward


class HeadGraph:
    """A whole decoder pass of ``Sparse4DHead`` over ``bs`` frames as one CUDA graph.  Static
    inputs: the packed maps ``mc_ms_feat [bs, num_feat, C]``, ``projection_mat [bs, Ncam, 4, 4]``,
    ``image_wh [bs, Ncam, 2]`` and the initial ``anchor [bs, A, 11]`` (the instance bank's by
    default); ``run(...)`` copies new ones in and replays, ``output`` is the replay's result dict."""

    def __init__(self, head: Sparse4DHead, bs: int, spatial_shapes: Sequence[Tuple[int, int]],
                 feature_dtype: torch.dtype = torch.bfloat16, warmup: int = 2):
        dev = head.device
        nc = 6
        self.head, self.bs, self.spatial_shapes = head, bs, [tuple(s) for s in spatial_shapes]
        self.spatial_shape, self.scale_start_index, num_feat = ops.level_tables(self.spatial_shapes, nc, device=dev)
        self.mc_ms_feat = torch.zeros(bs, num_feat, head.embed_dims, dtype=feature_dtype, device=dev)
        self.projection_mat = torch.zeros(bs, nc, 4, 4, device=dev)
        self.projection_mat[..., 2, 2] = 1.0
        self.projection_mat[..., 3, 3] = 1.0
        self.image_wh = torch.ones(bs, nc, 2, device=dev)
        self.anchor = head.anchor[None].expand(bs, -1, -1).contiguous()
        self._call = capture(self._forward, warmup=warmup)

    def _forward(self):
        packed = (self.mc_ms_feat, self.spatial_shape, self.scale_start_index)
        return self.head.forward(packed, self.projection_mat, self.image_wh, self.spatial_shapes, self.bs,
                                 anchor=self.anchor)

    @property
    def output(self):
        return self._call.output

    def replay(self):
        return self._call.replay()

    def run(self, mc_ms_feat: Optional[Tensor] = None, projection_mat: Optional[Tensor] = None,
            image_wh: Optional[Tensor] = None, anchor: Optional[Tensor] = None):
        for dst, src in ((self.mc_ms_feat, mc_ms_feat), (self.projection_mat, projection_mat),
                         (self.image_wh, image_wh), (self.anchor, anchor)):
            if src is not None:
                dst.copy_(src, non_blocking=True)
        return self.replay()
