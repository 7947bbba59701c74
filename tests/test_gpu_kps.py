"""Kernel (a) on the GPU against the oracle and the reference's fixtures: projected points
within float tolerance, depth mask / frustum mask / compacted (b, a, cam, pt) indices bit-exact."""
import numpy as np
import pytest
import torch

import fixtures as fx
from helpers import regen
from oracle import dfa_numpy as onp
from oracle import dfa_torch as oto
from sparse4d_tt_b200 import ops
from sparse4d_tt_b200 import synthetic as syn

pytestmark = pytest.mark.gpu


def _run(anchor, learn, fix, proj, wh, layout=0):
    d = torch.device("cuda:0")
    out = ops.kps_project(anchor.to(d), None if learn is None else learn.to(d), fix.to(d), proj.to(d), wh.to(d),
                          layout)
    torch.cuda.synchronize()
    loc, mask, idx, cnt, kp = [t.cpu() for t in out]
    return loc, mask, idx[: int(cnt[0])], int(cnt[0]), kp


def _margins(uv, depth):
    """Distance of the nearest sample to a mask threshold (explains any flip)."""
    u, v = uv[..., 0].abs(), uv[..., 1].abs()
    return {
        "depth": float((depth - 1e-5).abs().min()),
        "u0": float(u.min()), "u1": float((1 - uv[..., 0]).abs().min()),
        "v0": float(v.min()), "v1": float((1 - uv[..., 1]).abs().min()),
    }


def _term_scale(kp, proj, wh):
    """(|P_r0 px| + |P_r1 py| + |P_r2 pz| + |P_r3|) / max(z, 1e-5) / (w or h), r = 0, 1:
    the size of the terms whose sum is u * z * w, i.e. how far rounding can move u."""
    P = proj.astype(np.float64)[:, None, :, None]
    p = kp.astype(np.float64)[:, :, None, :, :]
    z = ((P[..., 2, 0] * p[..., 0] + P[..., 2, 1] * p[..., 1]) + P[..., 2, 2] * p[..., 2]) + P[..., 2, 3]
    zc = np.maximum(z, 1e-5)
    out = []
    for r in (0, 1):
        t = (np.abs(P[..., r, 0] * p[..., 0]) + np.abs(P[..., r, 1] * p[..., 1]) + np.abs(P[..., r, 2] * p[..., 2])
             + np.abs(P[..., r, 3]))
        out.append(t / zc / wh.astype(np.float64)[:, None, :, None, r])
    return np.stack(out, axis=-1)


@pytest.mark.parametrize("name", ["standard_s0_fp32", "highres_s2_bf16", "small_b2_s3", "small_b1_s4_cam3"])
def test_kps_bit_exact_masks_and_indices(cuda_device, name):
    g, cfg, ins, params = regen(name)
    learn = oto.learnable_logits(ins.instance_feature, params)  # the oracle's own fp32 logits
    loc, mask, idx, cnt, kp = _run(ins.anchor, learn, params["kps_fix_scale"], ins.projection_mat, ins.image_wh)
    bs, A, nc, P = cfg.bs, cfg.num_anchor, cfg.num_cams, cfg.num_pts
    ref_mask = fx.unpack_bits(g["mask_bits"], (bs, A, nc, P))
    ref_vis = fx.unpack_bits(g["vis_bits"], (bs, A, nc, P))
    assert np.array_equal(mask.numpy().astype(bool), ref_mask)
    assert cnt == int(ref_vis.sum())
    assert np.array_equal(idx.numpy(), np.argwhere(ref_vis).astype(np.int32))
    # the numpy oracle evaluates the same fixed order: identical masks
    kp_np = onp.key_points(ins.anchor.numpy(), learn.numpy(), params["kps_fix_scale"].numpy())
    uv_np, mask_np, vis_np = onp.project(kp_np, ins.projection_mat.numpy(), ins.image_wh.numpy())
    assert np.array_equal(mask.numpy().astype(bool), mask_np)
    np.testing.assert_allclose(kp.numpy(), kp_np, rtol=1e-5, atol=1e-5)
    kps_t = oto.key_points(ins.anchor, ins.instance_feature, params)
    uv_t, depth_t = oto.project_points_with_depth(kps_t, ins.projection_mat, ins.image_wh)
    # u = X / z is ill-conditioned next to the camera plane (a 1-ulp keypoint difference from
    # exp() moves z by ~1e-6 m), and X = sum_j P_j p_j cancels (terms of 1e4 summing to ~1):
    # where |z| > 0.5 m, allow 1e-4 relative plus 1e-5 of the summed term magnitudes
    # (about 100 ulps of the largest term) divided by z * w; masks and indices are bit-exact.
    well = (depth_t.permute(0, 2, 1, 3).abs() > 0.5).numpy()[..., None].repeat(2, -1)
    scale = _term_scale(kp_np, ins.projection_mat.numpy(), ins.image_wh.numpy())
    err = np.abs(loc.numpy() - uv_np)
    tol = 1e-4 * np.abs(uv_np) + 1e-4 + 1e-5 * scale
    assert np.all(err[well] <= tol[well]), float((err - tol)[well].max())
    m = _margins(uv_t, depth_t)
    print(f"{name}: visible={cnt} margins={m}")


@pytest.mark.parametrize("bs", [1, 2])
def test_kps_reference_dummy_inputs(cuda_device, bs):
    """The reference's own e2e inputs (random N(0,1) projection matrices)."""
    g = fx.load(f"refdummy_bs{bs}")
    # the exact input bits the reference computed the fixture's masks from (stored, so that a
    # host whose CPU rounds sin/cos or the linear differently tests the same case)
    anchor, learn, fix, proj, wh = fx.reference_dummy_kps_inputs(bs)
    assert fx.same_inputs(g, anchor=anchor, projection_mat=proj)
    loc, mask, idx, cnt, kp = _run(anchor, learn, fix, proj, wh)
    ref_vis = fx.unpack_bits(g["vis_bits"], (bs, 900, 6, 13))
    assert cnt == int(ref_vis.sum()) == int(g["n_visible"])
    assert np.array_equal(idx.numpy(), np.argwhere(ref_vis).astype(np.int32))
    rows = g["rows"]
    np.testing.assert_allclose(kp.reshape(bs * 900, 13, 3).numpy()[rows], g["kp_rows"], rtol=1e-5, atol=1e-5)


def test_kps_layouts_agree(cuda_device):
    cfg = syn.DFAConfig(bs=2, num_anchor=77)
    ins = syn.make_inputs(cfg, 11)
    params = syn.make_params(cfg, torch.Generator().manual_seed(5))
    learn = oto.learnable_logits(ins.instance_feature, params)
    a = _run(ins.anchor, learn, params["kps_fix_scale"], ins.projection_mat, ins.image_wh, 0)
    b = _run(ins.anchor, learn, params["kps_fix_scale"], ins.projection_mat, ins.image_wh, 1)
    assert torch.equal(a[0], b[0].permute(0, 1, 3, 2, 4))
    assert torch.equal(a[1], b[1]) and torch.equal(a[2], b[2])


def test_kps_edge_cases(cuda_device):
    d = torch.device("cuda:0")
    fix = torch.tensor(syn.FIX_SCALE)
    proj = syn.camera_ring(6, (704, 256))[None]
    wh = torch.tensor([[704.0, 256.0]]).expand(1, 6, 2).contiguous()
    # no anchors: count is 0
    loc, mask, idx, cnt, kp = _run(torch.zeros(1, 0, 11), torch.zeros(1, 0, 18), fix, proj, wh)
    assert cnt == 0 and loc.numel() == 0
    # one anchor straight ahead of camera 0 at 20 m: its centre is visible in camera 0
    a = torch.zeros(1, 1, 11)
    a[0, 0, 0] = 20.0
    a[0, 0, 2] = 1.5
    a[0, 0, 7] = 1.0
    loc, mask, idx, cnt, kp = _run(a, torch.zeros(1, 1, 18), fix, proj, wh)
    assert cnt > 0 and idx[0].tolist() == [0, 0, 0, 0]
    np.testing.assert_allclose(loc[0, 0, 0, 0].numpy(), [0.5, 0.5], atol=1e-6)
    # anchors behind every camera plane of a forward-only rig: nothing in front
    proj1 = proj[:, :1].contiguous()
    a2 = a.clone()
    a2[0, 0, 0] = -20.0
    loc, mask, idx, cnt, kp = _run(a2, torch.zeros(1, 1, 18), fix, proj1, wh[:, :1].contiguous())
    assert cnt == 0 and int(mask.sum()) == 0
    # no learnable points; extra anchor fields beyond the 11 are ignored
    cfg = syn.DFAConfig(bs=1, num_anchor=50)
    ins = syn.make_inputs(cfg, 3)
    wide = torch.cat([ins.anchor, torch.randn(1, 50, 5)], dim=-1).contiguous()
    r1 = _run(ins.anchor, None, fix, ins.projection_mat, ins.image_wh)
    r2 = _run(wide, None, fix, ins.projection_mat, ins.image_wh)
    assert torch.equal(r1[0], r2[0]) and torch.equal(r1[2], r2[2])
    assert r1[0].shape == (1, 50, 6, 7, 2)


def test_kps_project_fused_dropin(cuda_device):
    """``ttnn.kps_project_fused`` arguments and output: grid = clamp(2 uv - 1, -2, 2)."""
    cfg = syn.DFAConfig(bs=1, num_anchor=64)
    ins = syn.make_inputs(cfg, 21)
    params = syn.make_params(cfg, torch.Generator().manual_seed(2))
    learn = oto.learnable_logits(ins.instance_feature, params)
    n = 64
    size = ins.anchor[0, :, 3:6].exp()[:, None]
    pre = torch.cat([params["kps_fix_scale"][None] * size,
                     (learn[0].reshape(n, 6, 3).sigmoid() - 0.5) * size], dim=1).contiguous()
    d = torch.device("cuda:0")
    grid = ops.kps_project_fused(pre.to(d), ins.anchor[0].reshape(n, 1, 11).to(d),
                                 ins.projection_mat[0].to(d), ins.image_wh[0].reshape(6, 1, 2).to(d), 6, 13)
    torch.cuda.synchronize()
    assert grid.shape == (6, n, 1, 26)
    kps = oto.key_points(ins.anchor, ins.instance_feature, params)
    uv, _ = oto.project_points_with_depth(kps, ins.projection_mat, ins.image_wh)
    ref = (uv[0] * 2 - 1).clamp(-2, 2).reshape(6, n, 1, 26)
    np.testing.assert_allclose(grid.cpu().numpy(), ref.numpy(), rtol=1e-4, atol=1e-5)


def test_kps_deterministic(cuda_device):
    g, cfg, ins, params = regen("standard_s0_fp32")
    learn = oto.learnable_logits(ins.instance_feature, params)
    a = _run(ins.anchor, learn, params["kps_fix_scale"], ins.projection_mat, ins.image_wh)
    b = _run(ins.anchor, learn, params["kps_fix_scale"], ins.projection_mat, ins.image_wh)
    for x, y in zip(a, b):
        if isinstance(x, torch.Tensor):
            assert torch.equal(x, y)


@pytest.mark.parametrize("strided", [False, True])
def test_kps_linear_matches_given_logits(cuda_device, strided):
    """s4d_kps_project_linear (learnable logits computed in the kernel, fp32) against
    s4d_kps_project fed float64-accurate logits of the same linear: keypoints within fp32
    rounding, sample locations within the projection tolerance where the depth is not tiny."""
    cfg = syn.config_standard(2)
    ins = syn.make_inputs(cfg, 31)
    params = syn.make_params(cfg, torch.Generator().manual_seed(131))
    params["kps_learnable_fc_bias"] = torch.randn(18, generator=torch.Generator().manual_seed(2)) * 0.1
    d = torch.device("cuda:0")
    inst = ins.instance_feature.reshape(-1, 256)
    if strided:
        wide = torch.zeros(inst.shape[0], 512)
        wide[:, :256] = inst
        inst_d = wide.to(d)[:, :256]
    else:
        inst_d = inst.to(d)
    w, b = params["kps_learnable_fc_weight"].to(d), params["kps_learnable_fc_bias"].to(d)
    bs, A = cfg.bs, cfg.num_anchor
    loc = torch.empty(bs, A, 6, 13, 2, device=d)
    kp = torch.empty(bs, A, 13, 3, device=d)
    ops.kps_project_linear_into(ins.anchor.to(d), inst_d, w, b, params["kps_fix_scale"].to(d), ins.projection_mat.to(d),
                                ins.image_wh.to(d), sample_location=loc, key_points=kp)
    learn = (inst.double() @ params["kps_learnable_fc_weight"].double().T
             + params["kps_learnable_fc_bias"].double()).float().reshape(bs, A, 18)
    ref_loc, _, _, _, ref_kp = ops.kps_project(ins.anchor.to(d), learn.to(d), params["kps_fix_scale"].to(d),
                                               ins.projection_mat.to(d), ins.image_wh.to(d))
    torch.cuda.synchronize()
    np.testing.assert_allclose(kp.cpu().numpy(), ref_kp.cpu().numpy(), rtol=1e-5, atol=1e-4)
    Pm = ins.projection_mat
    depth = torch.einsum("bck,bapk->bacp", Pm[:, :, 2, :3], ref_kp.cpu()) + Pm[:, None, :, 2, 3, None]
    well = (depth.abs() > 0.5).numpy()[..., None].repeat(2, -1)
    err = (loc.cpu() - ref_loc.cpu()).abs().numpy()
    assert np.all(err[well] <= 1e-3 * np.abs(ref_loc.cpu().numpy()[well]) + 1e-4)


def test_kps_linear_compaction_is_consistent(cuda_device):
    """s4d_kps_project_linear with the compaction (the keypoint leg of the benchmark): the
    compacted indices are exactly the (b, anchor, cam, pt) whose written depth mask is set and
    whose written (u, v) lie in [0, 1], in lexicographic order."""
    cfg = syn.config_standard(2)
    ins = syn.make_inputs(cfg, 32)
    params = syn.make_params(cfg, torch.Generator().manual_seed(132))
    d = torch.device("cuda:0")
    bs, A, nc, P = cfg.bs, cfg.num_anchor, cfg.num_cams, cfg.num_pts
    loc = torch.empty(bs, A, nc, P, 2, device=d)
    mask = torch.empty(bs, A, nc, P, dtype=torch.uint8, device=d)
    idx = torch.empty(bs * A * nc * P, 4, dtype=torch.int32, device=d)
    cnt = torch.zeros(1, dtype=torch.int32, device=d)
    ws = torch.empty(max(ops.kps_workspace_bytes(bs, A, nc, P), 16), dtype=torch.uint8, device=d)
    ops.kps_project_linear_into(ins.anchor.to(d), ins.instance_feature.reshape(-1, 256).to(d),
                                params["kps_learnable_fc_weight"].to(d), params["kps_learnable_fc_bias"].to(d),
                                params["kps_fix_scale"].to(d), ins.projection_mat.to(d), ins.image_wh.to(d),
                                sample_location=loc, depth_mask=mask, visible_idx=idx, visible_count=cnt,
                                workspace=ws)
    torch.cuda.synchronize()
    u, v = loc[..., 0].cpu(), loc[..., 1].cpu()
    vis = mask.cpu().bool() & (u >= 0) & (u <= 1) & (v >= 0) & (v <= 1)
    n = int(cnt.item())
    assert n == int(vis.sum()) > 0
    assert torch.equal(idx[:n].cpu(), torch.nonzero(vis).to(torch.int32))
