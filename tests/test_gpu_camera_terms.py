"""The one-launch camera terms (camera encoder, per-camera logits and the gather's per-frame
softmax factors in one cluster launch) against the two-launch camera encoder plus the factor
kernel: bitwise equal, since both compute every value with the same operations in the same
order.  Shapes the factor kernel does not cover are checked against exp(wc - max) in float64."""
import numpy as np
import pytest
import torch

from sparse4d_tt_b200 import _lib as L
from sparse4d_tt_b200 import ops
from sparse4d_tt_b200 import synthetic as syn

pytestmark = pytest.mark.gpu


def _inputs(bs, nc, n, seed):
    dev = torch.device("cuda:0")
    cfg = syn.DFAConfig(bs=bs, num_cams=nc)
    params = syn.make_params(cfg, torch.Generator().manual_seed(60 + seed))
    gen = torch.Generator().manual_seed(seed)
    for k in ("cam_ln1_weight", "cam_ln2_weight"):
        params[k] = 1 + 0.2 * torch.randn(256, generator=gen)
    for k in ("cam_ln1_bias", "cam_ln2_bias", "cam_linear1_bias", "cam_linear2_bias"):
        params[k] = 0.1 * torch.randn(params[k].shape, generator=gen)
    params["weights_fc_weight"] = 0.05 * torch.randn(n, 256, generator=gen)
    params["weights_fc_bias"] = 0.1 * torch.randn(n, generator=gen)
    ring = syn.camera_ring(6, (704, 256))
    proj = torch.stack([ring[i % 6] * (1 + 0.01 * i) for i in range(nc)])[None].repeat(bs, 1, 1, 1)
    proj = proj * (1 + 0.05 * torch.randn(bs, nc, 1, 1, generator=gen))
    d = {k: v.to(dev).contiguous() for k, v in params.items()}
    weights = [d[k] for k in ("cam_linear1_weight", "cam_linear1_bias", "cam_ln1_weight", "cam_ln1_bias",
                              "cam_linear2_weight", "cam_linear2_bias", "cam_ln2_weight", "cam_ln2_bias",
                              "weights_fc_weight", "weights_fc_bias")]
    return proj.to(dev).contiguous(), weights


def _factor_words(bs, nc, n):
    return bs * (nc + 1) * n


@pytest.mark.parametrize("bs", [1, 3, 32])
def test_camera_terms_bitwise_equal_to_two_launches_and_factors(cuda_device, bs):
    dev = torch.device("cuda:0")
    proj, w = _inputs(bs, 6, 416, bs)
    logits_a = torch.empty(bs, 6, 4, 13, 8, device=dev)
    emb_a = torch.empty(bs, 6, 256, device=dev)
    ws_a = ops.dfa_workspace(bs, 6, 4, 13, 8, dev)
    ops.camera_logits_into(logits_a, proj, *w, camera_embed=emb_a)
    ops.camera_factors_into(ws_a, logits_a)

    logits_b = torch.full_like(logits_a, float("nan"))
    emb_b = torch.full_like(emb_a, float("nan"))
    ws_b = ops.dfa_workspace(bs, 6, 4, 13, 8, dev)
    ws_b.view(torch.int32).fill_(-1)  # the anchor counter pair must come back zero
    ops.camera_terms_into(logits_b, proj, *w, camera_embed=emb_b, factors=ws_b)
    torch.cuda.synchronize()
    assert torch.equal(logits_a.view(torch.int32), logits_b.view(torch.int32))
    assert torch.equal(emb_a.view(torch.int32), emb_b.view(torch.int32))
    k = _factor_words(bs, 6, 416)
    assert torch.equal(ws_a[:k].view(torch.int32), ws_b[:k].view(torch.int32))
    counter = ws_b.view(torch.int32)[ws_b.numel() - 4: ws_b.numel() - 2]
    assert counter.tolist() == [0, 0]


@pytest.mark.parametrize("nc,n", [(1, 416), (8, 416), (6, 200), (3, 512)])
def test_camera_terms_without_factors_equal_camera_logits(cuda_device, nc, n):
    """No workspace: logits and embedding only, any 1..8 cameras and up to 512 logit columns."""
    dev = torch.device("cuda:0")
    bs = 2
    proj, w = _inputs(bs, nc, n, 7 + nc)
    logits_a = torch.empty(bs, nc, n, device=dev)
    emb_a = torch.empty(bs, nc, 256, device=dev)
    ops.camera_logits_into(logits_a, proj, *w, camera_embed=emb_a)
    logits_b = torch.full_like(logits_a, float("nan"))
    ops.camera_terms_into(logits_b, proj, *w)
    emb_b = torch.full_like(emb_a, float("nan"))
    logits_c = torch.full_like(logits_a, float("nan"))
    ops.camera_terms_into(logits_c, proj, *w, camera_embed=emb_b)
    torch.cuda.synchronize()
    assert torch.equal(logits_a.view(torch.int32), logits_b.view(torch.int32))
    assert torch.equal(logits_a.view(torch.int32), logits_c.view(torch.int32))
    assert torch.equal(emb_a.view(torch.int32), emb_b.view(torch.int32))


@pytest.mark.parametrize("nc,n", [(4, 96), (8, 512), (2, 8)])
def test_camera_terms_factors_other_shapes(cuda_device, nc, n):
    """Factors of shapes the factor kernel does not take (ragged column shares: 96 columns leave
    two of the eight CTAs without columns, 8 columns leave seven): exp(wc - M2[group]) per camera
    and their sum, M2 the frame's maximum of its group (column j is group j % 8), against float64
    on the kernel's own logits; ex2.approx is within 2 ulp."""
    dev = torch.device("cuda:0")
    bs = 3
    proj, w = _inputs(bs, nc, n, 30 + n)
    logits = torch.empty(bs, nc, n, device=dev)
    nbytes = int(L.lib().s4d_dfa_workspace_bytes(bs, nc, 1, n // 8, 8, 1))
    ws = torch.full((nbytes // 4,), float("nan"), device=dev)
    ops.camera_terms_into(logits, proj, *w, factors=ws)
    torch.cuda.synchronize()
    wc = logits.cpu().double().view(bs, nc, n // 8, 8)
    m2 = wc.amax(dim=(1, 2), keepdim=True)
    ec = torch.exp(wc - m2).view(bs, nc, n)
    want = torch.cat([ec, ec.sum(1, keepdim=True)], 1)
    got = ws[: _factor_words(bs, nc, n)].cpu().double().view(bs, nc + 1, n)
    err = ((got - want).abs() / want.abs().clamp_min(1e-30)).max().item()
    print(f"nc={nc} n={n}: factors max rel err {err:.2e}")
    assert err <= 4e-6
    assert np.array_equal(ws.view(torch.int32)[ws.numel() - 4: ws.numel() - 2].cpu().numpy(), [0, 0])


def test_camera_terms_in_the_layer(cuda_device):
    """The DFA module uses the one-launch camera terms for the Sparse4D v3 shape and few frames;
    its cached logits, embedding and factors equal the two-launch path's."""
    from sparse4d_tt_b200 import DeformableFeatureAggregation

    dev = torch.device("cuda:0")
    cfg = syn.DFAConfig(bs=2, num_anchor=64)
    params = syn.make_params(cfg, torch.Generator().manual_seed(9))
    mod = DeformableFeatureAggregation(dev, params, {"FEATURE_DTYPE": torch.float32})
    assert mod._factors_ok and mod.camera_terms_max_frames >= 2
    proj = syn.camera_ring(6, (704, 256))[None].repeat(2, 1, 1, 1).to(dev)
    wc = mod._camera_logits(proj, 2)
    assert mod._cached_camera_ws is None  # the one-launch path needs no scratch
    ref = torch.empty_like(wc)
    emb = torch.empty(2, 6, 256, device=dev)
    w = [getattr(mod, k) for k in ("cam_linear1_weight", "cam_linear1_bias", "cam_ln1_weight", "cam_ln1_bias",
                                   "cam_linear2_weight", "cam_linear2_bias", "cam_ln2_weight", "cam_ln2_bias",
                                   "weights_fc_weight", "weights_fc_bias")]
    ops.camera_logits_into(ref, proj, *w, camera_embed=emb)
    ws = ops.camera_factors_into(ops.dfa_workspace(2, 6, 4, 13, 8, dev), ref)
    torch.cuda.synchronize()
    assert torch.equal(wc, ref) and torch.equal(mod._cached_camera_embed, emb)
    k = _factor_words(2, 6, 416)
    assert torch.equal(mod._cached_camera_factors[:k], ws[:k])
