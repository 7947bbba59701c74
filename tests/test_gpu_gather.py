"""Kernel (b)+(c) on the GPU against the oracle: fp32 features within max-abs 1e-4; bf16
features (fp32 accumulation) with PCC >= 0.9999 and relative error <= 1e-2; layouts, split
logits, camera ranges and edge cases."""
import numpy as np
import pytest
import torch

from helpers import max_rel_err, mean_rel_err, oracle_gather_inputs, oracle_uv_bacp, pcc, regen
from oracle import dfa_numpy as onp
from oracle import dfa_torch as oto
from sparse4d_tt_b200 import ops
from sparse4d_tt_b200 import synthetic as syn

pytestmark = pytest.mark.gpu

FP32_ATOL = 1e-4  # fp32 features: max abs error
BF16_PCC = 0.9999  # bf16 features, fp32 accumulation
BF16_REL = 1e-2


def _gpu_gather(maps, uv_bacp, logits, dtype=torch.float32, logits_flag=True, layout=0, cam_range=None,
                weights_cam=None):
    d = torch.device("cuda:0")
    feat, shape, start = ops.pack_feature_maps([m.to(d) for m in maps], dtype=dtype)
    nc = shape.shape[0]
    cb, ce = (0, nc) if cam_range is None else cam_range
    out = ops.deformable_aggregation(feat, shape, start, uv_bacp.contiguous().to(d), logits.contiguous().to(d),
                                     logits_flag, None if weights_cam is None else weights_cam.contiguous().to(d),
                                     cb, ce, layout)
    torch.cuda.synchronize()
    return out.cpu()


@pytest.mark.parametrize("name", ["standard_s0_fp32", "small_b2_s3", "small_b1_s4_cam3"])
def test_gather_fp32_matches_oracle(cuda_device, name):
    g, cfg, ins, params = regen(name)
    uv, depth, logits = oracle_gather_inputs(cfg, ins, params)
    ref = oto.deformable_aggregation(ins.feature_maps, uv, logits)
    got = _gpu_gather(ins.feature_maps, oracle_uv_bacp(uv), logits)
    err = (got - ref).abs().max().item()
    print(f"{name}: fp32 max abs err {err:.3e}")
    assert err <= FP32_ATOL
    # and against the reference's own fused features in the fixture
    if "fused" in g:
        np.testing.assert_allclose(got.numpy(), g["fused"], rtol=0, atol=FP32_ATOL)
    else:
        rows = g["rows"]
        np.testing.assert_allclose(got.reshape(-1, 256).numpy()[rows], g["fused_rows"], rtol=0, atol=FP32_ATOL)


@pytest.mark.parametrize("name", ["standard_s1_bf16", "highres_s2_bf16"])
def test_gather_bf16_matches_oracle(cuda_device, name):
    """bf16 maps (the oracle sees the same bf16-rounded values in fp32)."""
    g, cfg, ins, params = regen(name)
    uv, depth, logits = oracle_gather_inputs(cfg, ins, params)
    got = _gpu_gather(ins.feature_maps, oracle_uv_bacp(uv), logits, dtype=torch.bfloat16)
    rows = g["rows"]
    sel = got.reshape(-1, 256).numpy()[rows]
    p, mre, xre = pcc(sel, g["fused_rows"]), mean_rel_err(sel, g["fused_rows"]), max_rel_err(sel, g["fused_rows"])
    print(f"{name}: vs reference rows pcc={p:.7f} mean_rel={mre:.2e} max_rel={xre:.2e}")
    assert p >= BF16_PCC and mre <= BF16_REL and xre <= BF16_REL
    np.testing.assert_allclose(got.reshape(-1, 256).double().sum(1).numpy(), g["fused_row_ck"][:, 0],
                               rtol=0, atol=1e-3)
    if name.startswith("standard"):
        ref = oto.deformable_aggregation(ins.feature_maps, uv, logits)
        p = pcc(got, ref)
        assert p >= BF16_PCC and mean_rel_err(got, ref) <= BF16_REL and max_rel_err(got, ref) <= BF16_REL
        assert (got - ref).abs().max().item() <= FP32_ATOL


def test_gather_bf16_storage_against_fp32_oracle(cuda_device):
    """bf16 storage error alone: bf16 kernel on rounded maps vs the fp32 oracle on the unrounded maps."""
    cfg = syn.config_standard(1)
    ins = syn.make_inputs(cfg, 7)
    params = syn.make_params(cfg, torch.Generator().manual_seed(70))
    uv, depth, logits = oracle_gather_inputs(cfg, ins, params)
    ref = oto.deformable_aggregation(ins.feature_maps, uv, logits)
    got = _gpu_gather(ins.feature_maps, oracle_uv_bacp(uv), logits, dtype=torch.bfloat16)
    p, mre, xre = pcc(got, ref), mean_rel_err(got, ref), max_rel_err(got, ref)
    print(f"bf16 storage: pcc={p:.7f} mean_rel={mre:.2e} max_rel={xre:.2e}")
    assert p >= BF16_PCC and mre <= BF16_REL and xre <= BF16_REL


def _small_case(seed=0, bs=2, A=33, nc=6, P=13, shapes=((16, 40), (8, 20), (4, 10), (2, 5)), G=8, spread=1.3):
    gen = torch.Generator().manual_seed(seed)
    maps = [torch.randn(bs, nc, 256, h, w, generator=gen) for h, w in shapes]
    uv = torch.rand(bs, A, nc, P, 2, generator=gen) * spread - (spread - 1) / 2
    logits = torch.randn(bs, A, nc, len(shapes), P, G, generator=gen) * 2
    return maps, uv, logits


def _oracle(maps, uv_bacp, logits, logits_flag=True, cam_range=None):
    if cam_range is None and logits_flag:
        return oto.deformable_aggregation(maps, uv_bacp.permute(0, 2, 1, 3, 4), logits)
    feat, shape, start = onp.pack_feature_maps([m.numpy() for m in maps])
    return torch.from_numpy(onp.deformable_aggregation(feat, shape, start, uv_bacp.numpy(), logits.numpy(),
                                                       logits=logits_flag, cam_range=cam_range))


def test_gather_pt_major_layout(cuda_device):
    """Upstream (pt-major) layout.  At the Sparse4D shape cam-major runs the shape-specialised
    kernel and pt-major the generic one: both against the oracle and against each other."""
    maps, uv, logits = _small_case(1)
    a = _gpu_gather(maps, uv, logits)
    b = _gpu_gather(maps, uv.permute(0, 1, 3, 2, 4), logits.permute(0, 1, 4, 2, 3, 5), layout=1)
    ref = _oracle(maps, uv, logits)
    assert (a - ref).abs().max().item() <= FP32_ATOL
    assert (b - ref).abs().max().item() <= FP32_ATOL
    assert (a - b).abs().max().item() <= 1e-5


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_fast_and_generic_kernels_agree(cuda_device, dtype):
    """Force the generic kernel at the Sparse4D shape by misaligning the logits by one float
    (the fast kernel needs 16-byte aligned rows) and compare with the fast kernel."""
    d = torch.device("cuda:0")
    maps, uv, logits = _small_case(11, bs=2, A=65)
    feat, shape, start = ops.pack_feature_maps([m.to(d) for m in maps], dtype=dtype)
    uv_d = uv.to(d).contiguous()
    w = logits.to(d).contiguous()
    store = torch.empty(w.numel() + 1, device=d)
    w_mis = store[1:].view_as(w)
    w_mis.copy_(w)
    fast = ops.deformable_aggregation(feat, shape, start, uv_d, w)
    generic = ops.deformable_aggregation(feat, shape, start, uv_d, w_mis)
    torch.cuda.synchronize()
    assert (fast - generic).abs().max().item() <= 1e-5
    if dtype == torch.float32:
        assert (fast.cpu() - _oracle(maps, uv, logits)).abs().max().item() <= FP32_ATOL


def test_gather_split_logits(cuda_device):
    maps, uv, _ = _small_case(2)
    gen = torch.Generator().manual_seed(9)
    wa = torch.randn(2, 33, 4, 13, 8, generator=gen)
    wc = torch.randn(2, 6, 4, 13, 8, generator=gen)
    full = wa[:, :, None] + wc[:, None]
    a = _gpu_gather(maps, uv, wa, weights_cam=wc)
    b = _gpu_gather(maps, uv, full)
    assert (a - b).abs().max().item() <= 1e-6
    assert (a - _oracle(maps, uv, full)).abs().max().item() <= FP32_ATOL


def _split_gather(maps, uv, wa, wc, dtype=torch.float32, with_ws=True, cam_range=None):
    d = torch.device("cuda:0")
    feat, shape, start = ops.pack_feature_maps([m.to(d) for m in maps], dtype=dtype)
    bs, A = uv.shape[:2]
    nc = shape.shape[0]
    cb, ce = (0, nc) if cam_range is None else cam_range
    out = torch.empty(bs, A, 256, device=d)
    ws = ops.dfa_workspace(bs, *wc.shape[1:5], d) if with_ws else None
    ops.deformable_aggregation_into(out, feat, shape, start, uv.contiguous().to(d), wa.contiguous().to(d), True,
                                    wc.contiguous().to(d), cb, ce, workspace=ws)
    torch.cuda.synchronize()
    return out.cpu()


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_gather_split_factorised_softmax(cuda_device, dtype):
    """Split logits with a workspace (per-frame camera factors, factorised softmax) against
    the same call without a workspace and against the oracle."""
    maps, uv, _ = _small_case(12, bs=3, A=70)
    gen = torch.Generator().manual_seed(19)
    wa = torch.randn(3, 70, 4, 13, 8, generator=gen) * 2
    wc = torch.randn(3, 6, 4, 13, 8, generator=gen) * 2
    a = _split_gather(maps, uv, wa, wc, dtype, True)
    b = _split_gather(maps, uv, wa, wc, dtype, False)
    assert (a - b).abs().max().item() <= 1e-5
    if dtype == torch.float32:
        ref = _oracle(maps, uv, wa[:, :, None] + wc[:, None])
        assert (a - ref).abs().max().item() <= FP32_ATOL
    parts = [_split_gather(maps, uv, wa, wc, dtype, True, r) for r in ((0, 2), (2, 6))]
    assert (parts[0] + parts[1] - a).abs().max().item() <= 1e-5


def test_gather_split_exact_fallback(cuda_device):
    """Logits whose largest sum sits far below max(wa) + max(wc): the factorised sum
    underflows and the kernel switches to the exact softmax."""
    maps, uv, _ = _small_case(13, bs=1, A=8)
    wa = torch.zeros(1, 8, 4, 13, 8)
    wc = torch.zeros(1, 6, 4, 13, 8)
    wa[:, :, 1, 3] = 100.0  # max(wa) at (level 1, point 3) ...
    wc[:, :, 1, 3] = -200.0  # ... where every camera term is very negative
    wa[:, 5] += torch.randn(4, 13, 8, generator=torch.Generator().manual_seed(3))
    a = _split_gather(maps, uv, wa, wc, torch.float32, True)
    ref = _oracle(maps, uv, wa[:, :, None] + wc[:, None])
    assert torch.isfinite(a).all()
    assert (a - ref).abs().max().item() <= FP32_ATOL


def test_gather_given_weights(cuda_device):
    """weights_are_logits=False: plain weighted sum (upstream op semantics)."""
    maps, uv, logits = _small_case(3)
    w = oto.softmax_weights(logits) * 1.7
    got = _gpu_gather(maps, uv, w, logits_flag=False)
    ref = _oracle(maps, uv, w, logits_flag=False)
    assert (got - ref).abs().max().item() <= FP32_ATOL


def test_gather_camera_ranges_sum_to_full(cuda_device):
    maps, uv, logits = _small_case(4)
    full = _gpu_gather(maps, uv, logits)
    parts = [_gpu_gather(maps, uv, logits, cam_range=r) for r in ((0, 3), (3, 6))]
    assert (parts[0] + parts[1] - full).abs().max().item() <= 1e-5
    ref0 = _oracle(maps, uv, logits, cam_range=(0, 3))
    assert (parts[0] - ref0).abs().max().item() <= FP32_ATOL
    empty = _gpu_gather(maps, uv, logits, cam_range=(2, 2))
    assert torch.count_nonzero(empty) == 0


@pytest.mark.parametrize("G", [1, 4, 32])
def test_gather_group_counts(cuda_device, G):
    maps, uv, logits = _small_case(5, G=G)
    got = _gpu_gather(maps, uv, logits)
    assert (got - _oracle(maps, uv, logits)).abs().max().item() <= FP32_ATOL


def test_gather_edge_locations(cuda_device):
    """Borders, corners, 1x1 maps, all-outside anchors, huge logits."""
    maps, uv, logits = _small_case(6, shapes=((5, 7), (1, 1), (3, 2)), P=5)
    uv[0, 0] = 0.0
    uv[0, 1] = 1.0
    uv[0, 2, :, :, 0] = 1.0
    uv[0, 2, :, :, 1] = 0.0
    uv[0, 3] = 5.0  # every sample outside the maps
    uv[0, 4] = -1e7
    uv[1, 5] = 0.5 / 7  # exactly on pixel centres of level 0 in x
    logits[1, 6] *= 1e4  # near one-hot softmax
    got = _gpu_gather(maps, uv, logits)
    ref = _oracle(maps, uv, logits)
    assert (got - ref).abs().max().item() <= FP32_ATOL
    assert torch.count_nonzero(got[0, 3]) == 0 and torch.count_nonzero(got[0, 4]) == 0


def test_gather_bad_level_sets_flag(cuda_device):
    """A (camera, level) whose rows lie outside mc_ms_feat is skipped and flagged; the other
    samples are unaffected (the result equals the oracle with that level's map zeroed)."""
    d = torch.device("cuda:0")
    maps, uv, logits = _small_case(7, bs=1, A=4)
    feat, shape, start = ops.pack_feature_maps([m.to(d) for m in maps])
    bad_start = start.clone()
    bad_start[5, 3] = feat.shape[1]  # level 3 of camera 5 begins past the end of mc_ms_feat
    flag = torch.zeros(1, dtype=torch.int32, device=d)
    out = torch.empty(1, 4, 256, device=d)
    ops.deformable_aggregation_into(out, feat, shape, bad_start, uv.to(d), logits.to(d), error_flag=flag)
    torch.cuda.synchronize()
    assert int(flag.item()) & 1
    zeroed = [m.clone() for m in maps]
    zeroed[3][:, 5] = 0
    ref = _oracle(zeroed, uv, logits)
    assert (out.cpu() - ref).abs().max().item() <= FP32_ATOL


def test_gather_deterministic(cuda_device):
    maps, uv, logits = _small_case(8)
    a = _gpu_gather(maps, uv, logits, dtype=torch.bfloat16)
    b = _gpu_gather(maps, uv, logits, dtype=torch.bfloat16)
    assert torch.equal(a, b)


def test_gather_linearity_full_size(cuda_device):
    """Size-independent property at the 1800-anchor 1600x640 shape: the operator is linear in
    the features (f -> 2f doubles the output exactly in fp32) and the bf16 result tracks the
    fp32 result."""
    d = torch.device("cuda:0")
    cfg = syn.config_highres(1, 1800)
    gen = torch.Generator(device=d).manual_seed(3)
    nc = 6
    shape, start, nf = ops.level_tables(cfg.spatial_shapes, nc, device=d)
    feat = torch.randn(1, nf, 256, device=d, generator=gen)
    uv = torch.rand(1, 1800, nc, 13, 2, device=d, generator=gen) * 1.4 - 0.2
    logits = torch.randn(1, 1800, nc, 4, 13, 8, device=d, generator=gen)
    o1 = ops.deformable_aggregation(feat, shape, start, uv, logits)
    o2 = ops.deformable_aggregation(feat * 2, shape, start, uv, logits)
    ob = ops.deformable_aggregation(feat.to(torch.bfloat16), shape, start, uv, logits)
    torch.cuda.synchronize()
    assert torch.equal(o2, o1 * 2)
    assert pcc(ob.cpu(), o1.cpu()) >= BF16_PCC


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_gather_prepared_camera_factors(cuda_device, dtype):
    """Factors written by camera_factors_into (as the module does on its camera stream) and read
    with factors_ready=True give exactly the result of the gather call computing them itself."""
    maps, uv, _ = _small_case(21, bs=2, A=90)
    gen = torch.Generator().manual_seed(23)
    wa = (torch.randn(2, 90, 4, 13, 8, generator=gen) * 2).cuda()
    wc = (torch.randn(2, 6, 4, 13, 8, generator=gen) * 2).cuda()
    d = torch.device("cuda:0")
    feat, shape, start = ops.pack_feature_maps([m.to(d) for m in maps], dtype=dtype)
    loc = uv.contiguous().to(d)
    ws_a = ops.dfa_workspace(2, 6, 4, 13, 8, d)
    a = torch.empty(2, 90, 256, device=d)
    ops.deformable_aggregation_into(a, feat, shape, start, loc, wa, True, wc, workspace=ws_a)
    ws_b = ops.camera_factors_into(ops.dfa_workspace(2, 6, 4, 13, 8, d), wc)
    b = torch.empty(2, 90, 256, device=d)
    ops.deformable_aggregation_into(b, feat, shape, start, loc, wa, True, wc, workspace=ws_b, factors_ready=True)
    torch.cuda.synchronize()
    n = 2 * 7 * 416  # the factors (the workspace ends with the gather's anchor counter)
    assert torch.equal(a, b) and torch.equal(ws_a[:n], ws_b[:n])
