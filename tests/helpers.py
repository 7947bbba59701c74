"""Shared pieces of the parity tests: the reference's comparison metrics and seeded inputs."""
from __future__ import annotations

import numpy as np
import torch

import fixtures as fx
from oracle import dfa_torch as oto
from sparse4d_tt_b200 import synthetic as syn


def pcc(a, b) -> float:
    """Pearson correlation, as ``compute_pcc`` (``test/dfa_pcc.py:49-58``)."""
    a = torch.as_tensor(a).double().flatten()
    b = torch.as_tensor(b).double().flatten()
    a = a - a.mean()
    b = b - b.mean()
    d = a.norm() * b.norm()
    if d == 0:
        return 1.0 if a.norm() == 0 and b.norm() == 0 else 0.0
    return float(torch.dot(a, b) / d)


def mean_rel_err(a, b, eps: float = 1e-6) -> float:
    """``compute_relative_error`` (``test/dfa_pcc.py:61-66``): mean(|a-b| / max(|a|, |b|, eps))."""
    a = torch.as_tensor(a).float().flatten()
    b = torch.as_tensor(b).float().flatten()
    return float(((a - b).abs() / torch.max(a.abs(), b.abs()).clamp(min=eps)).mean())


def max_rel_err(a, b) -> float:
    """Largest absolute error relative to the largest reference magnitude."""
    a = torch.as_tensor(a).double()
    b = torch.as_tensor(b).double()
    return float((a - b).abs().max() / b.abs().max().clamp(min=1e-30))


def cfg_from_fixture(g, name):
    if name.startswith("standard"):
        return syn.config_standard(int(g["bs"]))
    if name.startswith("highres"):
        return syn.config_highres(int(g["bs"]), int(g["num_anchor"]))
    return syn.DFAConfig(bs=int(g["bs"]), num_anchor=int(g["num_anchor"]), num_cams=int(g["num_cams"]),
                         image_wh=tuple(int(v) for v in g["image_wh"]), strides=tuple(int(v) for v in g["strides"]))


def regen(name):
    """Fixture + regenerated inputs and parameters of a synthetic golden case."""
    g = fx.load(name)
    cfg = cfg_from_fixture(g, name)
    dt = torch.bfloat16 if bool(g["bf16_maps"]) else None
    ins = syn.make_inputs(cfg, int(g["seed"]), feature_dtype=dt)
    params = syn.make_params(cfg, torch.Generator().manual_seed(int(g["param_seed"])))
    np.testing.assert_allclose(fx.checksum(ins.anchor), g["ck_anchor"], rtol=1e-12)
    return g, cfg, ins, params


def oracle_uv_bacp(uv_bcap2: torch.Tensor) -> torch.Tensor:
    """``[bs, Ncam, A, P, 2]`` -> ``[bs, A, Ncam, P, 2]`` (the operator's cam-major layout)."""
    return uv_bcap2.permute(0, 2, 1, 3, 4).contiguous()


def oracle_gather_inputs(cfg, ins, params):
    """Sample locations and logits computed by the oracle, on the CPU."""
    kps = oto.key_points(ins.anchor, ins.instance_feature, params)
    uv, depth = oto.project_points_with_depth(kps, ins.projection_mat, ins.image_wh)
    logits = oto.weight_logits(ins.instance_feature, ins.anchor_embed, ins.projection_mat, params,
                               cfg.num_levels, cfg.num_pts, cfg.num_groups)
    return uv, depth, logits
