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
