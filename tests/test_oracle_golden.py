"""Pin the CPU oracle against fixtures produced by running the reference's own PyTorch DFA
(``tests/golden/make_golden.py``), and cross-check the two oracle restatements (torch and
numpy) against each other."""
import numpy as np
import pytest
import torch

import fixtures as fx
from oracle import dfa_numpy as onp
from oracle import dfa_torch as oto
from sparse4d_tt_b200 import synthetic as syn


def _cfg_from(meta, name):
    if name.startswith("standard"):
        return syn.config_standard(int(meta["bs"]))
    if name.startswith("highres"):
        return syn.config_highres(int(meta["bs"]), int(meta["num_anchor"]))
    return syn.DFAConfig(bs=int(meta["bs"]), num_anchor=int(meta["num_anchor"]), num_cams=int(meta["num_cams"]),
                         image_wh=tuple(int(v) for v in meta["image_wh"]),
                         strides=tuple(int(v) for v in meta["strides"]))


def _regen(name):
    g = fx.load(name)
    cfg = _cfg_from(g, name)
    dt = torch.bfloat16 if bool(g["bf16_maps"]) else None
    ins = syn.make_inputs(cfg, int(g["seed"]), feature_dtype=dt)
    params = syn.make_params(cfg, torch.Generator().manual_seed(int(g["param_seed"])))
    return g, cfg, ins, params


def _check_inputs(g, tensors, maps, params):
    for name, t in zip(("instance_feature", "anchor", "anchor_embed", "projection_mat", "image_wh"), tensors):
        np.testing.assert_allclose(fx.checksum(t), g[f"ck_{name}"], rtol=1e-12, err_msg=name)
    for i, fm in enumerate(maps):
        np.testing.assert_allclose(fx.checksum(fm), g[f"ck_map{i}"], rtol=1e-12, err_msg=f"map{i}")
    for k, v in params.items():
        np.testing.assert_allclose(fx.checksum(v), g[f"ck_param_{k}"], rtol=1e-12, atol=1e-12, err_msg=k)


def _masks(uv, depth):
    return oto.visibility(uv, depth)


@pytest.mark.parametrize("name", ["small_b2_s3", "small_b1_s4_cam3"])
def test_small_cases_all_intermediates(name):
    g, cfg, ins, params = _regen(name)
    _check_inputs(g, (ins.instance_feature, ins.anchor, ins.anchor_embed, ins.projection_mat, ins.image_wh),
                  ins.feature_maps, params)
    out, im = oto.dfa_layer(params, ins.instance_feature, ins.anchor, ins.anchor_embed, ins.feature_maps,
                            ins.projection_mat, ins.image_wh, return_intermediates=True)
    np.testing.assert_allclose(im["key_points"].numpy(), g["key_points"], rtol=0, atol=1e-5)
    np.testing.assert_allclose(im["uv"].numpy(), g["uv"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(im["weights"][0, :4].numpy(), g["weights_b0a0_3"], rtol=1e-5, atol=1e-7)
    np.testing.assert_allclose(im["fused"].numpy(), g["fused"], rtol=0, atol=1e-5)
    np.testing.assert_allclose(out[..., : cfg.embed_dims].numpy(), g["out"], rtol=0, atol=1e-5)
    mask, vis = _masks(im["uv"], im["depth"])
    assert np.array_equal(fx.pack_bits(mask), g["mask_bits"])
    assert np.array_equal(fx.pack_bits(vis), g["vis_bits"])
    assert np.array_equal(torch.nonzero(vis).numpy(), g["vis_idx"])


@pytest.mark.parametrize("name", ["standard_s0_fp32", "standard_s1_bf16", "highres_s2_bf16"])
def test_full_size_cases(name):
    g, cfg, ins, params = _regen(name)
    _check_inputs(g, (ins.instance_feature, ins.anchor, ins.anchor_embed, ins.projection_mat, ins.image_wh),
                  ins.feature_maps, params)
    out, im = oto.dfa_layer(params, ins.instance_feature, ins.anchor, ins.anchor_embed, ins.feature_maps,
                            ins.projection_mat, ins.image_wh, return_intermediates=True)
    bs, A = cfg.bs, cfg.num_anchor
    rows = g["rows"]
    fused = im["fused"].reshape(bs * A, -1)
    np.testing.assert_allclose(fused[rows].numpy(), g["fused_rows"], rtol=0, atol=1e-5)
    np.testing.assert_allclose(out[..., : cfg.embed_dims].reshape(bs * A, -1)[rows].numpy(), g["out_rows"],
                               rtol=0, atol=1e-5)
    np.testing.assert_allclose(fused.double().sum(1).numpy(), g["fused_row_ck"][:, 0], rtol=0, atol=1e-4)
    mask, vis = _masks(im["uv"], im["depth"])
    assert np.array_equal(fx.pack_bits(mask), g["mask_bits"])
    assert np.array_equal(fx.pack_bits(vis), g["vis_bits"])
    assert int(vis.sum()) == int(g["n_visible"])


@pytest.mark.parametrize("name,bs", [("refdummy_bs1", 1), ("refdummy_bs2", 2)])
def test_reference_dummy_case(name, bs):
    """The reference's own e2e test inputs (seed 42, random projection matrices, default
    Linear init), replayed here and checked against the reference's outputs."""
    g = fx.load(name)
    (inst, anchor, embed, maps, proj, wh), params = fx.reference_dummy_case(bs)
    _check_inputs(g, (inst, anchor, embed, proj, wh), maps, params)
    out, im = oto.dfa_layer(params, inst, anchor, embed, maps, proj, wh, return_intermediates=True)
    rows = g["rows"]
    fused = im["fused"].reshape(bs * 900, -1)
    np.testing.assert_allclose(fused[rows].numpy(), g["fused_rows"], rtol=0, atol=1e-5)
    np.testing.assert_allclose(out[..., :256].reshape(bs * 900, -1)[rows].numpy(), g["out_rows"], rtol=0, atol=1e-5)
    mask, vis = _masks(im["uv"], im["depth"])
    assert np.array_equal(fx.pack_bits(vis), g["vis_bits"])


@pytest.mark.parametrize("name", ["small_b2_s3", "small_b1_s4_cam3"])
def test_numpy_oracle_matches_reference(name):
    """The numpy restatement (explicit taps, packed channels-last layout, fixed projection
    order) against the reference's keypoints, projection, masks and fused features."""
    g, cfg, ins, params = _regen(name)
    logits_l = oto.learnable_logits(ins.instance_feature, params).numpy()
    kp = onp.key_points(ins.anchor.numpy(), logits_l, params["kps_fix_scale"].numpy())
    np.testing.assert_allclose(kp, g["key_points"], rtol=0, atol=2e-5)
    uv, mask, vis = onp.project(kp, ins.projection_mat.numpy(), ins.image_wh.numpy())
    np.testing.assert_allclose(uv.transpose(0, 2, 1, 3, 4), g["uv"], rtol=1e-4, atol=1e-5)
    assert np.array_equal(fx.pack_bits(mask), g["mask_bits"])
    assert np.array_equal(fx.pack_bits(vis), g["vis_bits"])
    assert np.array_equal(np.argwhere(vis).astype(np.int32), g["vis_idx"])
    logits = oto.weight_logits(ins.instance_feature, ins.anchor_embed, ins.projection_mat, params,
                               cfg.num_levels, cfg.num_pts, cfg.num_groups).numpy()
    feat, spatial, start = onp.pack_feature_maps([m.numpy() for m in ins.feature_maps])
    # sample at the reference's own projected points so only the gather is compared
    fused = onp.deformable_aggregation(feat, spatial, start, g["uv"].transpose(0, 2, 1, 3, 4), logits)
    np.testing.assert_allclose(fused, g["fused"], rtol=0, atol=2e-5)


def test_numpy_oracle_full_size_masks():
    """Bit-exact depth and frustum masks of the numpy oracle at the full 900-anchor size."""
    g, cfg, ins, params = _regen("standard_s0_fp32")
    logits_l = oto.learnable_logits(ins.instance_feature, params).numpy()
    kp = onp.key_points(ins.anchor.numpy(), logits_l, params["kps_fix_scale"].numpy())
    uv, mask, vis = onp.project(kp, ins.projection_mat.numpy(), ins.image_wh.numpy())
    assert np.array_equal(fx.pack_bits(mask), g["mask_bits"])
    assert np.array_equal(fx.pack_bits(vis), g["vis_bits"])


def test_numpy_gather_edge_cases():
    """Border, corner and out-of-image sample locations: the numpy gather against
    ``F.grid_sample`` through the torch oracle."""
    rng = np.random.default_rng(0)
    bs, A, nc, P, G, C = 1, 5, 2, 4, 8, 256
    shapes = [(3, 5), (1, 1)]
    maps = [rng.standard_normal((bs, nc, C, h, w)).astype(np.float32) for h, w in shapes]
    uv = np.array([
        [0.0, 0.0], [1.0, 1.0], [0.5, 0.5], [1e-7, 1 - 1e-7],
    ], dtype=np.float32)
    uv = np.tile(uv[None, None, None], (bs, A, nc, 1, 1))
    uv[0, 1] += 0.37
    uv[0, 2] -= 0.41
    uv[0, 3, :, :, 0] = -0.2
    uv[0, 4, :, :] = 5.0
    logits = rng.standard_normal((bs, A, nc, len(shapes), P, G)).astype(np.float32) * 3
    feat, spatial, start = onp.pack_feature_maps(maps)
    got = onp.deformable_aggregation(feat, spatial, start, uv, logits)
    ref = oto.deformable_aggregation([torch.from_numpy(m) for m in maps],
                                     torch.from_numpy(uv).permute(0, 2, 1, 3, 4), torch.from_numpy(logits))
    np.testing.assert_allclose(got, ref.numpy(), rtol=0, atol=1e-5)
    assert np.all(got[0, 4] == 0)


@pytest.mark.parametrize("bs", [1, 2])
def test_reference_dummy_kps_inputs_pin_the_masks(bs):
    """The stored input bits of the reference's seed-42 case reproduce the fixture's input
    checksums, and the numpy oracle's fixed-order projection of them gives the reference's
    depth and visibility masks bit for bit (the GPU keypoint test feeds these same bits)."""
    g = fx.load(f"refdummy_bs{bs}")
    anchor, learn, fix, proj, wh = fx.reference_dummy_kps_inputs(bs)
    assert fx.same_inputs(g, anchor=anchor, projection_mat=proj, image_wh=wh)
    assert np.allclose(fx.checksum(fix), g["ck_param_kps_fix_scale"], rtol=1e-12, atol=0)
    kp = onp.key_points(anchor.numpy(), learn.numpy(), fix.numpy())
    _, mask, vis = onp.project(kp, proj.numpy(), wh.numpy())
    assert np.array_equal(fx.pack_bits(mask), g["mask_bits"])
    assert np.array_equal(fx.pack_bits(vis), g["vis_bits"])
    assert int(vis.sum()) == int(g["n_visible"])
