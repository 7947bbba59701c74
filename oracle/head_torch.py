"""Torch fp32 CPU restatement of the reference's single-frame Sparse4D v3 decoder head twin.
TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``): the oracle of the decoder-chain parity
test of ``sparse4d-tt_b200/head.py``.

It follows ``_PTSparse4DHead`` and its pieces in ``test/sparse4d_head_pcc.py`` (cited per
class), built from the same torch module types in the same construction order, so that under
``torch.manual_seed(s)`` it draws the same parameters as the reference twin;
``tests/golden/make_golden.py`` runs the reference twin itself and stores checksums of every
parameter together with its outputs, which ``tests/test_oracle_head.py`` checks this
restatement against.  The DFA layers are ``oracle.dfa_torch``'s restatement of the same
algorithm (``test/sparse4d_head_pcc.py:195-254`` computes exactly what ``test/dfa_pcc.py``
computes).

Operation order of the head (``test/sparse4d_head_pcc.py:301-305``): one single-frame decoder
``deformable, ffn, norm, refine`` (the leading ``gnn, norm`` are dropped), then five temporal
decoders ``temp_gnn, gnn, norm, deformable, ffn, norm, refine``.
"""
from __future__ import annotations

from typing import Dict, List

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import dfa_torch

X, Y, Z = 0, 1, 2
W, L, H = 3, 4, 5
SIN_YAW, COS_YAW = 6, 7
VX = 8

FIX_SCALE = [[0, 0, 0], [0.45, 0, 0], [-0.45, 0, 0], [0, 0.45, 0], [0, -0.45, 0], [0, 0, 0.45], [0, 0, -0.45]]


def linear_relu_ln(embed_dims: int, in_loops: int, out_loops: int, input_dims: int = None) -> List[nn.Module]:
    """``out_loops`` x (``in_loops`` x (Linear, ReLU), LayerNorm) (``test/sparse4d_head_pcc.py:84-94``)."""
    input_dims = embed_dims if input_dims is None else input_dims
    mods: List[nn.Module] = []
    for _ in range(out_loops):
        for _ in range(in_loops):
            mods += [nn.Linear(input_dims, embed_dims), nn.ReLU(inplace=True)]
            input_dims = embed_dims
        mods.append(nn.LayerNorm(embed_dims))
    return mods


class Scale(nn.Module):
    """Learned per-channel output scale (``test/sparse4d_head_pcc.py:97-102``)."""

    def __init__(self, values):
        super().__init__()
        self.scale = nn.Parameter(torch.tensor(values, dtype=torch.float32))

    def forward(self, x):
        return x * self.scale


class Attention(nn.Module):
    """Multi-head attention with identity shortcut (``test/sparse4d_head_pcc.py:105-120``)."""

    def __init__(self, embed_dims: int, num_heads: int):
        super().__init__()
        self.attn = nn.MultiheadAttention(embed_dims, num_heads, batch_first=False)
        self.proj_drop = nn.Dropout(0.0)

    def forward(self, query, key=None, value=None):
        key = query if key is None else key
        value = key if value is None else value
        out = self.attn(query.transpose(0, 1), key.transpose(0, 1), value.transpose(0, 1))[0].transpose(0, 1)
        return query + self.proj_drop(out)


class AnchorEncoder(nn.Module):
    """Anchor -> embedding, concatenated position / size / yaw / velocity MLPs
    (``test/sparse4d_head_pcc.py:123-147``)."""

    def __init__(self, dims=(128, 32, 32, 64), vel_dims: int = 3, in_loops: int = 1, out_loops: int = 4):
        super().__init__()
        self.vel_dims = vel_dims

        def mlp(inp, out):
            return nn.Sequential(*linear_relu_ln(out, in_loops, out_loops, inp))

        self.pos_fc = mlp(3, dims[0])
        self.size_fc = mlp(3, dims[1])
        self.yaw_fc = mlp(2, dims[2])
        self.vel_fc = mlp(vel_dims, dims[3])

    def forward(self, b):
        parts = [self.pos_fc(b[..., [X, Y, Z]]), self.size_fc(b[..., [W, L, H]]),
                 self.yaw_fc(b[..., [SIN_YAW, COS_YAW]]), self.vel_fc(b[..., VX:VX + self.vel_dims])]
        return torch.cat(parts, dim=-1)


class AsymmetricFFN(nn.Module):
    """Pre-norm FFN from the 2C DFA output to C (``test/sparse4d_head_pcc.py:150-163``)."""

    def __init__(self, in_channels: int = 512, embed_dims: int = 256, ff_channels: int = 1024):
        super().__init__()
        self.pre_norm = nn.LayerNorm(in_channels)
        self.layers = nn.Sequential(
            nn.Sequential(nn.Linear(in_channels, ff_channels), nn.ReLU(inplace=True), nn.Dropout(0.0)),
            nn.Linear(ff_channels, embed_dims), nn.Dropout(0.0),
        )
        self.identity_fc = nn.Linear(in_channels, embed_dims)

    def forward(self, x):
        x = self.pre_norm(x)
        return self.identity_fc(x) + self.layers(x)


class Refinement(nn.Module):
    """Box refinement + classification + quality heads (``test/sparse4d_head_pcc.py:166-192``)."""

    def __init__(self, embed_dims: int = 256, output_dim: int = 11, num_cls: int = 10):
        super().__init__()
        self.output_dim = output_dim
        self.layers = nn.Sequential(*linear_relu_ln(embed_dims, 2, 2), nn.Linear(embed_dims, output_dim),
                                    Scale([1.0] * output_dim))
        self.cls_layers = nn.Sequential(*linear_relu_ln(embed_dims, 1, 2), nn.Linear(embed_dims, num_cls))
        self.quality_layers = nn.Sequential(*linear_relu_ln(embed_dims, 1, 2), nn.Linear(embed_dims, 2))

    def forward(self, inst, anchor, embed, time_interval, return_cls: bool):
        feat = inst + embed
        out = self.layers(feat)
        out[..., :VX] = out[..., :VX] + anchor[..., :VX]
        out[..., VX:] = (out[..., VX:].transpose(0, -1) / time_interval).transpose(0, -1) + anchor[..., VX:]
        cls = self.cls_layers(inst) if return_cls else None
        qt = self.quality_layers(feat) if return_cls else None
        return out, cls, qt


class KeypointGenerator(nn.Module):
    """The DFA's keypoint generator parameters (``test/sparse4d_head_pcc.py:257-284``)."""

    def __init__(self, embed_dims: int = 256, num_learnable_pts: int = 6):
        super().__init__()
        self.fix_scale = nn.Parameter(torch.tensor(FIX_SCALE, dtype=torch.float32), requires_grad=False)
        self.learnable_fc = nn.Linear(embed_dims, num_learnable_pts * 3)


class DFA(nn.Module):
    """The head's DFA layer (``test/sparse4d_head_pcc.py:195-224``); its forward is
    ``oracle.dfa_torch.dfa_layer`` on the parameter dictionary of ``dfa_params``."""

    def __init__(self, embed_dims: int = 256, num_groups: int = 8, num_levels: int = 4, num_cams: int = 6,
                 num_learnable_pts: int = 6):
        super().__init__()
        self.kps_generator = KeypointGenerator(embed_dims, num_learnable_pts)
        self.output_proj = nn.Linear(embed_dims, embed_dims)
        self.proj_drop = nn.Dropout(0.0)
        self.camera_encoder = nn.Sequential(
            nn.Linear(12, embed_dims), nn.ReLU(inplace=True), nn.LayerNorm(embed_dims),
            nn.Linear(embed_dims, embed_dims), nn.ReLU(inplace=True), nn.LayerNorm(embed_dims),
        )
        self.weights_fc = nn.Linear(embed_dims, num_groups * num_levels * (len(FIX_SCALE) + num_learnable_pts))

    def forward(self, inst, anchor, embed, feature_maps, projection_mat, image_wh):
        return dfa_torch.dfa_layer(dfa_params(self), inst, anchor, embed, feature_maps, projection_mat, image_wh)


def dfa_params(m) -> Dict[str, torch.Tensor]:
    """``preprocess_dfa_parameters`` keys of a DFA module of the head."""
    enc = m.camera_encoder
    return {
        "kps_fix_scale": m.kps_generator.fix_scale.data, "kps_learnable_fc_weight": m.kps_generator.learnable_fc.weight.data,
        "kps_learnable_fc_bias": m.kps_generator.learnable_fc.bias.data,
        "cam_linear1_weight": enc[0].weight.data, "cam_linear1_bias": enc[0].bias.data,
        "cam_ln1_weight": enc[2].weight.data, "cam_ln1_bias": enc[2].bias.data,
        "cam_linear2_weight": enc[3].weight.data, "cam_linear2_bias": enc[3].bias.data,
        "cam_ln2_weight": enc[5].weight.data, "cam_ln2_bias": enc[5].bias.data,
        "weights_fc_weight": m.weights_fc.weight.data, "weights_fc_bias": m.weights_fc.bias.data,
        "output_proj_weight": m.output_proj.weight.data, "output_proj_bias": m.output_proj.bias.data,
    }


def operation_order(num_decoder: int = 6, num_single_frame: int = 1) -> List[str]:
    """``test/sparse4d_head_pcc.py:301-305``."""
    return (["gnn", "norm", "deformable", "ffn", "norm", "refine"] * num_single_frame
            + ["temp_gnn", "gnn", "norm", "deformable", "ffn", "norm", "refine"] * (num_decoder - num_single_frame))[2:]


class Head(nn.Module):
    """``_PTSparse4DHead`` (``test/sparse4d_head_pcc.py:287-408``), single frame, no temporal
    instances: ``temp_gnn`` attends over the query itself."""

    def __init__(self, embed_dims: int = 256, num_decoder: int = 6, num_single_frame: int = 1, num_anchor: int = 900,
                 num_cls: int = 10, num_groups: int = 8):
        super().__init__()
        self.embed_dims = embed_dims
        self.num_single_frame_decoder = num_single_frame
        self.operation_order = operation_order(num_decoder, num_single_frame)
        mods = []
        for op in self.operation_order:
            if op in ("gnn", "temp_gnn"):
                mods.append(Attention(2 * embed_dims, num_groups))
            elif op == "norm":
                mods.append(nn.LayerNorm(embed_dims))
            elif op == "deformable":
                mods.append(DFA(embed_dims, num_groups))
            elif op == "ffn":
                mods.append(AsymmetricFFN(2 * embed_dims, embed_dims, 4 * embed_dims))
            elif op == "refine":
                mods.append(Refinement(embed_dims, 11, num_cls))
        self.layers = nn.ModuleList(mods)
        self.anchor_encoder = AnchorEncoder((128, 32, 32, 64))
        self.anchor = nn.Parameter(torch.randn(num_anchor, 11) * 0.1)
        self.instance_feature = nn.Parameter(torch.zeros(num_anchor, embed_dims))
        self.fc_before = nn.Linear(embed_dims, 2 * embed_dims, bias=False)
        self.fc_after = nn.Linear(2 * embed_dims, embed_dims, bias=False)

    def graph_model(self, i, query, value, query_pos):
        """Decoupled attention (``test/sparse4d_head_pcc.py:332-340``)."""
        query = torch.cat([query, query_pos], dim=-1)
        if value is not None:
            value = self.fc_before(value)
        return self.fc_after(self.layers[i](query, None, value))

    @torch.no_grad()
    def forward(self, feature_maps, projection_mat, image_wh, bs: int = 1, anchor=None, time_interval=0.5):
        """Predictions, classifications and qualities of every decoder
        (``test/sparse4d_head_pcc.py:342-408``); ``anchor [bs, A, 11]`` replaces the instance
        bank's anchors when given."""
        inst = self.instance_feature[None].expand(bs, -1, -1).clone()
        anchor = self.anchor[None].expand(bs, -1, -1).clone() if anchor is None else anchor.clone()
        ti = torch.tensor([time_interval] * bs, dtype=torch.float32)
        embed = self.anchor_encoder(anchor)
        preds, clss, qts = [], [], []
        last = len(self.operation_order) - 1
        for i, op in enumerate(self.operation_order):
            if op == "temp_gnn":
                inst = self.graph_model(i, inst, None, embed)
            elif op == "gnn":
                inst = self.graph_model(i, inst, inst, embed)
            elif op in ("norm", "ffn"):
                inst = self.layers[i](inst)
            elif op == "deformable":
                inst = self.layers[i](inst, anchor, embed, feature_maps, projection_mat, image_wh)
            elif op == "refine":
                return_cls = len(preds) == self.num_single_frame_decoder - 1 or i == last
                anchor, cls, qt = self.layers[i](inst, anchor, embed, ti, return_cls)
                preds.append(anchor)
                clss.append(cls)
                qts.append(qt)
                if i != last:
                    embed = self.anchor_encoder(anchor)
        return {"prediction": preds, "classification": clss, "quality": qts}


def build_head(seed: int = 42, num_anchor: int = 900) -> Head:
    """The head under ``torch.manual_seed(seed)``, as the reference's test builds its twin
    (``test/sparse4d_head_pcc.py:530-547``)."""
    torch.manual_seed(seed)
    return Head(num_anchor=num_anchor).eval()


def head_inputs(bs: int = 1, num_cams: int = 6, embed_dims: int = 256,
                spatial_shapes=((64, 176), (32, 88), (16, 44), (8, 22))):
    """Inputs drawn right after the head, from the same global generator, as the reference's
    test draws them (``test/sparse4d_head_pcc.py:549-558``): maps x0.1, projections x0.1."""
    maps = [torch.randn(bs, num_cams, embed_dims, h, w) * 0.1 for h, w in spatial_shapes]
    proj = torch.randn(bs, num_cams, 4, 4) * 0.1
    wh = torch.tensor([[704.0, 256.0]]).unsqueeze(0).expand(bs, num_cams, 2).contiguous()
    return maps, proj, wh
