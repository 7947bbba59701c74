"""The fused camera-encoder kernel (camera embedding + per-camera logit term) against a float64
restatement of the reference's camera encoder (test/dfa_pcc.py:272-279,309-316)."""
import pytest
import torch
import torch.nn.functional as F

from sparse4d_tt_b200 import ops
from sparse4d_tt_b200 import synthetic as syn

pytestmark = pytest.mark.gpu


def _reference(params, proj):
    p = {k: v.double() for k, v in params.items()}
    bs, nc = proj.shape[:2]
    x = proj.double()[:, :, :3].reshape(bs, nc, 12)
    x = F.relu(F.linear(x, p["cam_linear1_weight"], p["cam_linear1_bias"]))
    x = F.layer_norm(x, (256,), p["cam_ln1_weight"], p["cam_ln1_bias"], 1e-5)
    x = F.relu(F.linear(x, p["cam_linear2_weight"], p["cam_linear2_bias"]))
    emb = F.layer_norm(x, (256,), p["cam_ln2_weight"], p["cam_ln2_bias"], 1e-5)
    return emb, F.linear(emb, p["weights_fc_weight"], p["weights_fc_bias"])


@pytest.mark.parametrize("bs,nc", [(1, 6), (3, 6), (32, 6), (2, 1), (2, 8)])
def test_camera_logits_matches_float64(cuda_device, bs, nc):
    dev = torch.device("cuda:0")
    cfg = syn.DFAConfig(bs=bs, num_cams=nc)
    params = syn.make_params(cfg, torch.Generator().manual_seed(40 + nc))
    gen = torch.Generator().manual_seed(bs)
    # LayerNorm affine parameters away from their (1, 0) init, so that the test sees them.
    for k in ("cam_ln1_weight", "cam_ln2_weight"):
        params[k] = 1 + 0.2 * torch.randn(256, generator=gen)
    for k in ("cam_ln1_bias", "cam_ln2_bias", "cam_linear1_bias", "cam_linear2_bias", "weights_fc_bias"):
        params[k] = 0.1 * torch.randn(params[k].shape, generator=gen)
    ring = syn.camera_ring(6, (704, 256))
    proj = torch.stack([ring[i % 6] * (1 + 0.01 * i) for i in range(nc)])[None].repeat(bs, 1, 1, 1)
    proj = proj * (1 + 0.05 * torch.randn(bs, nc, 1, 1, generator=gen))
    d = {k: v.to(dev).contiguous() for k, v in params.items()}
    logits = torch.empty(bs, nc, 416, device=dev)
    emb = torch.empty(bs, nc, 256, device=dev)
    ops.camera_logits_into(logits, proj.to(dev).contiguous(), d["cam_linear1_weight"], d["cam_linear1_bias"],
                           d["cam_ln1_weight"], d["cam_ln1_bias"], d["cam_linear2_weight"], d["cam_linear2_bias"],
                           d["cam_ln2_weight"], d["cam_ln2_bias"], d["weights_fc_weight"], d["weights_fc_bias"],
                           camera_embed=emb)
    torch.cuda.synchronize()
    ref_emb, ref_logits = _reference(params, proj)
    e_err = (emb.cpu().double() - ref_emb).abs().max().item()
    l_err = (logits.cpu().double() - ref_logits).abs().max().item()
    print(f"bs={bs} nc={nc}: camera_embed max err {e_err:.2e}, logits max err {l_err:.2e}")
    assert e_err <= 2e-5 * max(1.0, ref_emb.abs().max().item())
    assert l_err <= 2e-5 * max(1.0, ref_logits.abs().max().item())


def test_layer_uses_per_frame_camera_cache(cuda_device):
    """The module computes the camera terms once per projection tensor and again after
    reset_frame_cache() or when the projection changes."""
    from sparse4d_tt_b200 import DeformableFeatureAggregation

    dev = torch.device("cuda:0")
    cfg = syn.DFAConfig(bs=2, num_anchor=64)
    params = syn.make_params(cfg, torch.Generator().manual_seed(5))
    mod = DeformableFeatureAggregation(dev, params, {"FEATURE_DTYPE": torch.float32})
    proj = syn.camera_ring(6, (704, 256))[None].repeat(2, 1, 1, 1).to(dev)
    a = mod._camera_logits(proj, 2)
    assert mod._camera_logits(proj, 2) is a
    mod.reset_frame_cache()
    b = mod._camera_logits(proj, 2)
    assert b is not a and torch.equal(a, b)
    proj.mul_(1.01)  # in-place change of the projection: recomputed
    c = mod._camera_logits(proj, 2)
    assert c is not b and not torch.equal(b, c)
