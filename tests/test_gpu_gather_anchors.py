"""The gather that computes its own sample locations (s4d_deformable_aggregation_anchors)
against the two-step path it replaces: the keypoint kernel writing the locations, then the
gather reading them.  Both evaluate the same keypoint and projection arithmetic, so the results
must be identical bit for bit, for both feature types, camera sub-ranges and anchors whose
points fall behind or outside the cameras."""
import pytest
import torch

from sparse4d_tt_b200 import ops
from sparse4d_tt_b200 import synthetic as syn

pytestmark = pytest.mark.gpu


def _case(bs, seed, scale_anchor=1.0):
    cfg = syn.config_standard(bs)
    ins = syn.make_inputs(cfg, seed)
    params = syn.make_params(cfg, torch.Generator().manual_seed(seed + 1))
    gen = torch.Generator().manual_seed(seed + 2)
    d = torch.device("cuda:0")
    anchor = ins.anchor.clone()
    anchor[..., 3:6] += torch.log(torch.tensor(scale_anchor))
    learn = torch.randn(bs * cfg.num_anchor, 18, generator=gen) * 2
    wa = torch.randn(bs, cfg.num_anchor, 4, 13, 8, generator=gen) * 2
    wc = torch.randn(bs, 6, 4, 13, 8, generator=gen) * 2
    feat32, shape, start = ops.pack_feature_maps([m.to(d) for m in ins.feature_maps], dtype=torch.float32)
    t = {k: v.contiguous().to(d) for k, v in dict(anchor=anchor, learn=learn, wa=wa, wc=wc, proj=ins.projection_mat,
                                                  wh=ins.image_wh, fix=params["kps_fix_scale"]).items()}
    return cfg, t, feat32, shape, start


def _both(cfg, t, feat, shape, start, cam_range=(0, 6)):
    d = torch.device("cuda:0")
    bs, A = cfg.bs, cfg.num_anchor
    ws = ops.camera_factors_into(ops.dfa_workspace(bs, 6, 4, 13, 8, d), t["wc"])
    loc = torch.empty(bs, A, 6, 13, 2, device=d)
    ops.kps_project_into(t["anchor"], t["learn"].view(bs, A, 18), t["fix"], t["proj"], t["wh"], sample_location=loc)
    two_step = torch.empty(bs, A, 256, device=d)
    ops.deformable_aggregation_into(two_step, feat, shape, start, loc, t["wa"], True, t["wc"], *cam_range,
                                    workspace=ws, factors_ready=True)
    fused = torch.full((bs, A, 256), float("nan"), device=d)
    flag = torch.zeros(1, dtype=torch.int32, device=d)
    ops.deformable_aggregation_anchors_into(fused, feat, shape, start, t["anchor"], t["fix"], t["learn"], t["proj"],
                                            t["wh"], t["wa"], t["wc"], ws, *cam_range, error_flag=flag)
    torch.cuda.synchronize()
    assert flag.item() == 0
    return two_step, fused, loc


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("bs", [1, 3])
def test_gather_from_anchors_equals_two_step(cuda_device, dtype, bs):
    cfg, t, feat32, shape, start = _case(bs, 40 + bs)
    feat = feat32.to(dtype)
    two_step, fused, loc = _both(cfg, t, feat, shape, start)
    inb = ((loc >= 0) & (loc <= 1)).all(-1).float().mean().item()
    print(f"bs={bs} {dtype}: in-image sample fraction {inb:.3f}")
    assert 0.05 < inb < 0.95  # the case has both visible and invisible points
    assert torch.equal(two_step, fused), (two_step - fused).abs().max().item()


def test_gather_from_anchors_camera_range(cuda_device):
    cfg, t, feat32, shape, start = _case(2, 50)
    two_step, fused, _ = _both(cfg, t, feat32.to(torch.bfloat16), shape, start, cam_range=(2, 5))
    assert torch.equal(two_step, fused)


@pytest.mark.parametrize("scale", [0.05, 30.0])
def test_gather_from_anchors_extreme_boxes(cuda_device, scale):
    """Tiny boxes (every keypoint near the centre) and huge ones (points behind the cameras and
    far outside the images)."""
    cfg, t, feat32, shape, start = _case(2, 60, scale_anchor=scale)
    two_step, fused, _ = _both(cfg, t, feat32, shape, start)
    assert torch.equal(two_step, fused)


def test_gather_from_anchors_empty(cuda_device):
    d = torch.device("cuda:0")
    feat = torch.zeros(1, 100, 256, device=d)
    shape = torch.ones(6, 4, 2, dtype=torch.int32, device=d)
    start = torch.zeros(6, 4, dtype=torch.int32, device=d)
    out = torch.empty(1, 0, 256, device=d)
    ws = ops.dfa_workspace(1, 6, 4, 13, 8, d)
    ops.deformable_aggregation_anchors_into(out, feat, shape, start, torch.empty(1, 0, 11, device=d),
                                            torch.zeros(7, 3, device=d), torch.empty(0, 18, device=d),
                                            torch.eye(4, device=d).repeat(1, 6, 1, 1), torch.ones(1, 6, 2, device=d),
                                            torch.empty(1, 0, 4, 13, 8, device=d), torch.zeros(1, 6, 4, 13, 8, device=d),
                                            ws)
    torch.cuda.synchronize()


def _anchors_gather(cfg, t, feat, shape, start):
    d = torch.device("cuda:0")
    ws = ops.camera_factors_into(ops.dfa_workspace(cfg.bs, 6, 4, 13, 8, d), t["wc"])
    out = torch.full((cfg.bs, cfg.num_anchor, 256), float("nan"), device=d)
    ops.deformable_aggregation_anchors_into(out, feat, shape, start, t["anchor"], t["fix"], t["learn"], t["proj"],
                                            t["wh"], t["wa"], t["wc"], ws)
    torch.cuda.synchronize()
    return out


@pytest.mark.parametrize("A", [100, 900, 1800])
def test_split_anchor_blocks_match_one_warp_per_anchor(cuda_device, A):
    """Launches of few anchors share each anchor between 8 (100 anchors), 4 (900) or 2 (1800)
    warps of a block; the same frame repeated in a batch of at least 4,800 anchors (one warp per
    anchor on a 148-SM B200) must give the same sums up to the order of the fp32 additions."""
    cfg1 = syn.DFAConfig(bs=1, num_anchor=A)
    ins = syn.make_inputs(cfg1, 70)
    params = syn.make_params(cfg1, torch.Generator().manual_seed(71))
    gen = torch.Generator().manual_seed(72)
    d = torch.device("cuda:0")
    learn = torch.randn(A, 18, generator=gen) * 2
    wa = torch.randn(1, A, 4, 13, 8, generator=gen) * 2
    wc = torch.randn(1, 6, 4, 13, 8, generator=gen) * 2
    feat, shape, start = ops.pack_feature_maps([m.to(d) for m in ins.feature_maps], dtype=torch.bfloat16)
    t1 = {k: v.contiguous().to(d) for k, v in dict(anchor=ins.anchor, learn=learn, wa=wa, wc=wc,
                                                   proj=ins.projection_mat, wh=ins.image_wh,
                                                   fix=params["kps_fix_scale"]).items()}
    one = _anchors_gather(cfg1, t1, feat, shape, start)
    n = max(3, -(-4800 // A))
    cfgn = syn.DFAConfig(bs=n, num_anchor=A)
    tn = dict(t1)
    for k in ("anchor", "wa", "wc", "proj", "wh"):
        tn[k] = t1[k].expand(n, *t1[k].shape[1:]).contiguous()
    tn["learn"] = t1["learn"].repeat(n, 1)
    many = _anchors_gather(cfgn, tn, feat.expand(n, -1, -1).contiguous(), shape, start)
    assert torch.isfinite(one).all()
    ref = many[0]
    err = (one[0] - ref).abs().max().item()
    assert err <= 1e-5 * max(1.0, ref.abs().max().item()), err
    assert torch.equal(many[0], many[n - 1])  # deterministic


def test_split_anchor_blocks_bs1_against_reference_rows(cuda_device):
    """The module's bs = 1 gather (900 anchors, 4 warps per anchor) fed the oracle's keypoint
    logits and split weight logits, against the reference's fused rows of the bf16 fixture and
    the oracle, at the bf16 tolerance."""
    from helpers import max_rel_err, mean_rel_err, pcc, regen
    from oracle import dfa_torch as oto

    g, cfg, ins, params = regen("standard_s1_bf16")
    d = torch.device("cuda:0")
    W, b = params["weights_fc_weight"].double(), params["weights_fc_bias"].double()
    wa = ((ins.instance_feature + ins.anchor_embed).double() @ W.T).float().reshape(1, 900, 4, 13, 8)
    cam = oto.camera_embed(ins.projection_mat, params).double()
    wc = (cam @ W.T + b).float().reshape(1, 6, 4, 13, 8)
    learn = oto.learnable_logits(ins.instance_feature, params).reshape(900, 18)
    feat, shape, start = ops.pack_feature_maps([m.to(d) for m in ins.feature_maps], dtype=torch.bfloat16)
    t = {k: v.contiguous().to(d) for k, v in dict(anchor=ins.anchor, learn=learn, wa=wa, wc=wc,
                                                  proj=ins.projection_mat, wh=ins.image_wh,
                                                  fix=params["kps_fix_scale"]).items()}
    got = _anchors_gather(cfg, t, feat, shape, start).cpu().reshape(900, 256)
    sel = got.numpy()[g["rows"]]
    p, mre, xre = pcc(sel, g["fused_rows"]), mean_rel_err(sel, g["fused_rows"]), max_rel_err(sel, g["fused_rows"])
    print(f"bs1 split gather vs reference rows: pcc={p:.7f} mean_rel={mre:.2e} max_rel={xre:.2e}")
    assert p >= 0.9999 and mre <= 1e-2 and xre <= 1e-2
    kps = oto.key_points(ins.anchor, ins.instance_feature, params)
    uv, _ = oto.project_points_with_depth(kps, ins.projection_mat, ins.image_wh)
    logits = oto.weight_logits(ins.instance_feature, ins.anchor_embed, ins.projection_mat, params, 4, 13, 8)
    ref = oto.deformable_aggregation(ins.feature_maps, uv, logits).reshape(900, 256)
    assert pcc(got, ref) >= 0.9999 and max_rel_err(got, ref) <= 1e-2


@pytest.mark.parametrize("bs,rows", [(1, (450, 900)), (1, (0, 450)), (3, (900, 2700)), (3, (0, 0))])
def test_gather_output_routing(cuda_device, bs, rows):
    """s4d_deformable_aggregation_anchors_peer: rows [begin, end) go to out_peer (here a second
    buffer on the same GPU), the others to out, each bit for bit the unrouted result; neither
    buffer is written outside its rows (the cooperative kernel at bs = 1, the warp kernel at
    bs = 3)."""
    cfg, t, feat32, shape, start = _case(bs, 90 + bs)
    feat = feat32.to(torch.bfloat16)
    d = torch.device("cuda:0")
    A = cfg.num_anchor
    ws = ops.camera_factors_into(ops.dfa_workspace(bs, 6, 4, 13, 8, d), t["wc"])
    args = (feat, shape, start, t["anchor"], t["fix"], t["learn"], t["proj"], t["wh"], t["wa"], t["wc"], ws)
    ref = torch.empty(bs, A, 256, device=d)
    ops.deformable_aggregation_anchors_into(ref, *args)
    out = torch.full((bs, A, 256), float("nan"), device=d)
    peer = torch.full((bs * A, 256), float("nan"), device=d)
    flag = torch.zeros(1, dtype=torch.int32, device=d)
    ops.deformable_aggregation_anchors_into(out, *args, error_flag=flag, out_peer=peer.data_ptr(), peer_rows=rows)
    torch.cuda.synchronize()
    assert flag.item() == 0
    b, e = rows
    ref2, out2 = ref.view(-1, 256), out.view(-1, 256)
    inside = torch.zeros(bs * A, dtype=torch.bool, device=d)
    inside[b:e] = True
    assert torch.equal(peer[inside], ref2[inside])
    assert torch.equal(out2[~inside], ref2[~inside])
    assert torch.isnan(out2[inside]).all() and torch.isnan(peer[~inside]).all()


@pytest.mark.parametrize("bs", [1, 3])
def test_prepared_workspace_serves_repeated_calls(cuda_device, bs):
    """The gather takes anchors from a counter in the workspace: s4d_dfa_camera_factors zeroes it
    (here over memory filled with garbage first) and every gather launch leaves it at zero, so one
    prepared workspace serves call after call with no reset in between, for the cooperative
    kernel (bs = 1) and the warp kernel (bs = 3), from anchors and from locations alike."""
    cfg, t, feat32, shape, start = _case(bs, 120 + bs)
    feat = feat32.to(torch.bfloat16)
    d = torch.device("cuda:0")
    A = cfg.num_anchor
    ws = ops.dfa_workspace(bs, 6, 4, 13, 8, d)
    ws.view(torch.int32).fill_(-12345)  # whatever the allocator handed out
    ops.camera_factors_into(ws, t["wc"])
    loc = torch.empty(bs, A, 6, 13, 2, device=d)
    ops.kps_project_into(t["anchor"], t["learn"].view(bs, A, 18), t["fix"], t["proj"], t["wh"], sample_location=loc)
    outs = []
    for i in range(5):
        out = torch.full((bs, A, 256), float("nan"), device=d)
        if i % 2 == 0:
            ops.deformable_aggregation_anchors_into(out, feat, shape, start, t["anchor"], t["fix"], t["learn"],
                                                    t["proj"], t["wh"], t["wa"], t["wc"], ws)
        else:
            ops.deformable_aggregation_into(out, feat, shape, start, loc, t["wa"], True, t["wc"], workspace=ws,
                                            factors_ready=True)
        outs.append(out)
    torch.cuda.synchronize()
    assert not torch.isnan(outs[0]).any()
    for o in outs[1:]:
        assert torch.equal(o, outs[0])
    # the counter pair is back at zero after the last call
    tail = ws.view(torch.int32)[-4:]
    assert tail[0].item() == 0 and tail[1].item() == 0
