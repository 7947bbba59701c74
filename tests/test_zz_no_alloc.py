"""s4d_kps_project_noalloc, the keypoint projection + compaction entry point for callers that
cannot allocate device memory (FFI hosts without a CUDA allocator, fixed memory budgets, loops
that must not allocate): called through the C ABI and checked against s4d_kps_project with a
caller-allocated workspace, on two calls in a row with different inputs (the built-in scratch
keeps the previous call's contents, which must not leak into the next result).  Named to be
collected last."""
import pytest
import torch

from oracle import dfa_torch as oto
from sparse4d_tt_b200 import _lib as L
from sparse4d_tt_b200 import ops
from sparse4d_tt_b200 import synthetic as syn

pytestmark = pytest.mark.gpu


def _inputs(seed, bs, A):
    cfg = syn.DFAConfig(bs=bs, num_anchor=A)
    ins = syn.make_inputs(cfg, seed)
    params = syn.make_params(cfg, torch.Generator().manual_seed(seed + 1))
    d = torch.device("cuda:0")
    learn = oto.learnable_logits(ins.instance_feature, params)
    return [t.to(d).contiguous() for t in (ins.anchor, learn, params["kps_fix_scale"], ins.projection_mat,
                                           ins.image_wh)]


def _noalloc(anchor, learn, fix, proj, wh):
    bs, A = anchor.shape[:2]
    nc, P = proj.shape[1], fix.shape[0] + learn.shape[2] // 3
    d = anchor.device
    loc = torch.empty(bs, A, nc, P, 2, device=d)
    mask = torch.empty(bs, A, nc, P, dtype=torch.uint8, device=d)
    idx = torch.empty(bs * A * nc * P, 4, dtype=torch.int32, device=d)
    cnt = torch.empty(1, dtype=torch.int32, device=d)
    kp = torch.empty(bs, A, P, 3, device=d)
    st = L.lib().s4d_kps_project_noalloc(
        anchor.data_ptr(), anchor.shape[2], fix.data_ptr(), fix.shape[0], learn.data_ptr(), learn.shape[2] // 3,
        proj.data_ptr(), wh.data_ptr(), bs, A, nc, 0, kp.data_ptr(), loc.data_ptr(), mask.data_ptr(), idx.data_ptr(),
        cnt.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert st == L.S4D_OK, L.lib().s4d_last_error().decode()
    return loc, mask, idx, cnt, kp


def test_noalloc_matches_workspace_entry_point_twice(cuda_device):
    for seed, bs, A in ((30, 2, 900), (31, 1, 333)):
        ins = _inputs(seed, bs, A)
        got = _noalloc(*ins)
        ref = ops.kps_project(*ins)
        torch.cuda.synchronize()
        n = int(ref[3].item())
        assert int(got[3].item()) == n > 0
        assert torch.equal(got[0], ref[0]) and torch.equal(got[1], ref[1]) and torch.equal(got[4], ref[4])
        assert torch.equal(got[2][:n], ref[2][:n])


def test_noalloc_rejects_sizes_beyond_its_scratch(cuda_device):
    anchor, learn, fix, proj, wh = _inputs(32, 1, 8)
    st = L.lib().s4d_kps_project_noalloc(
        anchor.data_ptr(), 11, fix.data_ptr(), 7, learn.data_ptr(), 6, proj.data_ptr(), wh.data_ptr(), 64, 6000, 6,
        0, None, None, None, None, None, None)
    assert st == L.S4D_ERR_UNSUPPORTED_SHAPE
    assert "scratch limit" in L.lib().s4d_last_error().decode()


def _boundary_inputs(A, nc, nfix, nlearn, seed=33):
    """One frame of A anchors seen by nc ring cameras, with nfix fixed and nlearn learnable
    keypoints (random fixed scales and logits)."""
    gen = torch.Generator().manual_seed(seed)
    d = torch.device("cuda:0")
    anchor = syn.make_anchors(1, A, gen)
    learn = torch.randn(1, A, 3 * nlearn, generator=gen)
    fix = torch.rand(nfix, 3, generator=gen) - 0.5
    proj = syn.camera_ring(nc, (704, 256))[None]
    wh = torch.tensor([704.0, 256.0]).expand(1, nc, 2)
    return [t.to(d).contiguous() for t in (anchor, learn, fix, proj, wh)]


def test_noalloc_accepts_exactly_its_limit(cuda_device):
    """bs*A*Ncam*P of exactly 4,194,304 elements (the documented maximum) is accepted and
    matches the workspace entry point, whose workspace at that size is what the built-in
    scratch holds; one element more is rejected."""
    ins = _boundary_inputs(65536, 4, 8, 8)  # 1 x 65,536 x 4 x 16 = 2^22
    got = _noalloc(*ins)
    ref = ops.kps_project(*ins)
    torch.cuda.synchronize()
    n = int(ref[3].item())
    assert int(got[3].item()) == n > 0
    assert torch.equal(got[0], ref[0]) and torch.equal(got[1], ref[1]) and torch.equal(got[4], ref[4])
    assert torch.equal(got[2][:n], ref[2][:n])
    anchor, learn, fix, proj, wh = _boundary_inputs(8, 1, 5, 0)
    st = L.lib().s4d_kps_project_noalloc(
        anchor.data_ptr(), 11, fix.data_ptr(), 5, None, 0, proj.data_ptr(), wh.data_ptr(), 1, 838861, 1, 0, None,
        None, None, None, None, None)  # 1 x 838,861 x 1 x 5 = 2^22 + 1
    assert st == L.S4D_ERR_UNSUPPORTED_SHAPE
    assert "scratch limit" in L.lib().s4d_last_error().decode()
