"""The drop-in DeformableFeatureAggregation module end to end on the GPU, against the
reference's own outputs (fixtures) and the oracle."""
import numpy as np
import pytest
import torch

import fixtures as fx
from helpers import max_rel_err, mean_rel_err, pcc, regen
from oracle import dfa_torch as oto
from sparse4d_tt_b200 import DeformableFeatureAggregation, ops
from sparse4d_tt_b200 import synthetic as syn

pytestmark = pytest.mark.gpu

FP32_ATOL = 1e-4
BF16_PCC = 0.9999
BF16_REL = 1e-2


@pytest.fixture(autouse=True)
def _fp32_matmul():
    assert torch.get_float32_matmul_precision() == "highest"
    assert not torch.backends.cuda.matmul.allow_tf32


def _module(params, cfg, dtype=torch.float32, split=False, matmul="fp32"):
    return DeformableFeatureAggregation("cuda:0", params, {"FEATURE_DTYPE": dtype, "MATMUL_PRECISION": matmul},
                                        embed_dims=cfg.embed_dims,
                                        num_groups=cfg.num_groups, num_levels=cfg.num_levels,
                                        num_cams=cfg.num_cams, num_pts=cfg.num_pts,
                                        num_learnable_pts=cfg.num_learnable_pts, split_logits=split)


def _run(mod, ins, cfg, maps=None):
    d = torch.device("cuda:0")
    out = mod.run(ins.instance_feature.to(d), ins.anchor.to(d), ins.anchor_embed.to(d),
                  maps if maps is not None else [m.to(d) for m in ins.feature_maps], ins.projection_mat.to(d),
                  ins.image_wh.to(d), cfg.spatial_shapes, cfg.bs, cfg.num_anchor)
    torch.cuda.synchronize()
    return out.cpu()


@pytest.mark.parametrize("split", [False, True])
def test_layer_fp32_against_reference(cuda_device, split):
    g, cfg, ins, params = regen("standard_s0_fp32")
    out = _run(_module(params, cfg, split=split), ins, cfg)
    assert out.shape == (1, 900, 512)
    rows = g["rows"]
    np.testing.assert_allclose(out[..., :256].reshape(900, 256).numpy()[rows], g["out_rows"], rtol=0, atol=FP32_ATOL)
    np.testing.assert_allclose(out[..., :256].reshape(900, 256).double().sum(1).numpy(), g["out_row_ck"][:, 0],
                               rtol=0, atol=1e-3)
    assert torch.equal(out[..., 256:], ins.instance_feature)
    ref = oto.dfa_layer(params, ins.instance_feature, ins.anchor, ins.anchor_embed, ins.feature_maps,
                        ins.projection_mat, ins.image_wh)
    err = (out - ref).abs().max().item()
    print(f"layer fp32 split={split}: max abs err vs oracle {err:.3e}")
    assert err <= FP32_ATOL


@pytest.mark.parametrize("split", [False, True])
def test_layer_bf16_against_reference(cuda_device, split):
    g, cfg, ins, params = regen("standard_s1_bf16")
    out = _run(_module(params, cfg, torch.bfloat16, split), ins, cfg)
    sel = out[..., :256].reshape(900, 256).numpy()[g["rows"]]
    p, mre, xre = pcc(sel, g["out_rows"]), mean_rel_err(sel, g["out_rows"]), max_rel_err(sel, g["out_rows"])
    print(f"layer bf16 split={split}: pcc={p:.7f} mean_rel={mre:.2e} max_rel={xre:.2e}")
    assert p >= BF16_PCC and mre <= BF16_REL and xre <= BF16_REL
    ref = oto.dfa_layer(params, ins.instance_feature, ins.anchor, ins.anchor_embed, ins.feature_maps,
                        ins.projection_mat, ins.image_wh)
    assert pcc(out, ref) >= BF16_PCC and max_rel_err(out, ref) <= BF16_REL


def test_layer_bf16_tf32_linears(cuda_device):
    """The benchmark's configuration: bf16 maps, split logits, TF32 linears; against the
    reference's rows and the fp32 oracle at the bf16 tolerance."""
    g, cfg, ins, params = regen("standard_s1_bf16")
    mod = _module(params, cfg, torch.bfloat16, True, "tf32")
    assert mod._tc  # the linears run on the library's tensor-core kernels
    out = _run(mod, ins, cfg)
    assert torch.get_float32_matmul_precision() == "highest"  # restored after the layer
    sel = out[..., :256].reshape(900, 256).numpy()[g["rows"]]
    p, mre, xre = pcc(sel, g["out_rows"]), mean_rel_err(sel, g["out_rows"]), max_rel_err(sel, g["out_rows"])
    print(f"layer bf16 + tf32 linears: pcc={p:.7f} mean_rel={mre:.2e} max_rel={xre:.2e}")
    assert p >= BF16_PCC and mre <= BF16_REL and xre <= BF16_REL
    ref = oto.dfa_layer(params, ins.instance_feature, ins.anchor, ins.anchor_embed, ins.feature_maps,
                        ins.projection_mat, ins.image_wh)
    assert pcc(out, ref) >= BF16_PCC and max_rel_err(out, ref) <= BF16_REL


def test_layer_highres_1800_anchors(cuda_device):
    g, cfg, ins, params = regen("highres_s2_bf16")
    out = _run(_module(params, cfg, torch.bfloat16), ins, cfg)
    sel = out[..., :256].reshape(1800, 256).numpy()[g["rows"]]
    assert pcc(sel, g["out_rows"]) >= BF16_PCC and max_rel_err(sel, g["out_rows"]) <= BF16_REL
    np.testing.assert_allclose(sel, g["out_rows"], rtol=0, atol=FP32_ATOL)


@pytest.mark.parametrize("bs", [1, 2])
def test_layer_reference_dummy_case(cuda_device, bs):
    """The reference's own e2e test (seed 42, default init, random projections, bs 1 and 2)."""
    g = fx.load(f"refdummy_bs{bs}")
    (inst, anchor, embed, maps, proj, wh), params = fx.reference_dummy_case(bs)
    cfg = syn.DFAConfig(bs=bs)
    ins = syn.DFAInputs(inst, anchor, embed, maps, proj, wh)
    out = _run(_module(params, cfg), ins, cfg)
    rows = g["rows"]
    np.testing.assert_allclose(out[..., :256].reshape(bs * 900, 256).numpy()[rows], g["out_rows"], rtol=0,
                               atol=FP32_ATOL)


def test_layer_feature_map_formats_agree(cuda_device):
    """List of NCHW maps, the reference's TT layout ([1, 1, bs*Ncam*H*W, C] per level) and a
    pre-packed (mc_ms_feat, spatial_shape, scale_start_index) give identical results."""
    cfg = syn.DFAConfig(bs=2, num_anchor=128)
    ins = syn.make_inputs(cfg, 13, feature_dtype=torch.bfloat16)
    params = syn.make_params(cfg, torch.Generator().manual_seed(31))
    mod = _module(params, cfg, torch.bfloat16)
    d = torch.device("cuda:0")
    a = _run(mod, ins, cfg)
    tt = [m.permute(0, 1, 3, 4, 2).reshape(1, 1, -1, 256).contiguous().to(d) for m in ins.feature_maps]
    b = _run(mod, ins, cfg, maps=tt)
    packed = ops.pack_feature_maps([m.to(d) for m in ins.feature_maps], dtype=torch.bfloat16)
    c = _run(mod, ins, cfg, maps=packed)
    assert torch.equal(a, b) and torch.equal(a, c)


def test_stacked_layers_small_batch(cuda_device):
    """Six stacked layers (different weights, anchors refined between layers) at bs=2."""
    cfg = syn.DFAConfig(bs=2, num_anchor=900)
    ins = syn.make_inputs(cfg, 17)
    gen = torch.Generator().manual_seed(99)
    d = torch.device("cuda:0")
    packed = ops.pack_feature_maps([m.to(d) for m in ins.feature_maps], dtype=torch.float32)
    anchor, inst = ins.anchor, ins.instance_feature
    for layer in range(6):
        params = syn.make_params(cfg, torch.Generator().manual_seed(500 + layer))
        mod = _module(params, cfg, split=True)
        step = syn.DFAInputs(inst, anchor, ins.anchor_embed, ins.feature_maps, ins.projection_mat, ins.image_wh)
        out = _run(mod, step, cfg, maps=packed)
        ref = oto.dfa_layer(params, inst, anchor, ins.anchor_embed, ins.feature_maps, ins.projection_mat,
                            ins.image_wh)
        assert (out - ref).abs().max().item() <= FP32_ATOL, layer
        inst = ref[..., :256].contiguous()
        anchor = syn.refine_anchors(anchor, gen)


@pytest.mark.parametrize("mode", ["cat", "add"])
def test_stacked_layers_tf32_strided_instance(cuda_device, mode):
    """Six stacked layers with the tensor-core linears, each fed the previous layer's output as
    a strided [.., :256] view of a [.., 512] buffer (read in place by TMA), against the oracle
    fed the same values.  Residual "add" writes [.., 256]."""
    cfg = syn.DFAConfig(bs=2, num_anchor=900)
    ins = syn.make_inputs(cfg, 23, feature_dtype=torch.bfloat16)
    gen = torch.Generator().manual_seed(77)
    d = torch.device("cuda:0")
    packed = ops.pack_feature_maps([m.to(d) for m in ins.feature_maps], dtype=torch.bfloat16)
    anchor, inst = ins.anchor, ins.instance_feature
    for layer in range(6):
        params = syn.make_params(cfg, torch.Generator().manual_seed(700 + layer))
        mod = DeformableFeatureAggregation("cuda:0", params, {"FEATURE_DTYPE": torch.bfloat16,
                                                              "MATMUL_PRECISION": "tf32"}, residual_mode=mode)
        assert mod._tc
        buf = torch.full((cfg.bs, cfg.num_anchor, 512), float("nan"), device=d)
        buf[..., :256] = inst.to(d)
        out = mod.run(buf[..., :256], anchor.to(d), ins.anchor_embed.to(d), packed, ins.projection_mat.to(d),
                      ins.image_wh.to(d), cfg.spatial_shapes, cfg.bs, cfg.num_anchor)
        torch.cuda.synchronize()
        out = out.cpu()
        ref = oto.dfa_layer(params, inst, anchor, ins.anchor_embed, ins.feature_maps, ins.projection_mat,
                            ins.image_wh, residual_mode=mode)
        assert out.shape == ref.shape
        p_, xre = pcc(out, ref), max_rel_err(out, ref)
        print(f"layer {layer} {mode}: pcc={p_:.7f} max_rel={xre:.2e}")
        assert p_ >= BF16_PCC and xre <= BF16_REL, layer
        inst = ref[..., :256].contiguous()
        anchor = syn.refine_anchors(anchor, gen)


def test_layer_tf32_large_batch_path(cuda_device):
    """Above 4096 anchor rows the tensor-core pass also produces the learnable logits and the plain
    keypoint kernel follows (below it, the keypoint kernel computes them itself): 5 frames x 900
    anchors through the module against the oracle, at the bf16 tolerance."""
    cfg = syn.DFAConfig(bs=5, num_anchor=900)
    ins = syn.make_inputs(cfg, 41, feature_dtype=torch.bfloat16)
    params = syn.make_params(cfg, torch.Generator().manual_seed(141))
    mod = _module(params, cfg, torch.bfloat16, True, "tf32")
    assert mod._tc
    out = _run(mod, ins, cfg)
    ref = oto.dfa_layer(params, ins.instance_feature, ins.anchor, ins.anchor_embed, ins.feature_maps,
                        ins.projection_mat, ins.image_wh)
    p_, xre = pcc(out, ref), max_rel_err(out, ref)
    print(f"5 x 900 tf32 layer: pcc={p_:.7f} max_rel={xre:.2e}")
    assert p_ >= BF16_PCC and xre <= BF16_REL
