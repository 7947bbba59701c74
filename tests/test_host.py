"""Host-side logic that needs no GPU: synthetic inputs, packing, level tables, parameter
extraction and the drop-in module's argument checks."""
import numpy as np
import pytest
import torch

from oracle import dfa_numpy as onp
from sparse4d_tt_b200 import DeformableFeatureAggregation, ops, preprocess_dfa_parameters
from sparse4d_tt_b200 import synthetic as syn


def test_synthetic_inputs_are_deterministic():
    cfg = syn.DFAConfig(bs=2, num_anchor=16)
    a, b = syn.make_inputs(cfg, 5), syn.make_inputs(cfg, 5)
    for x, y in zip((a.instance_feature, a.anchor, a.projection_mat), (b.instance_feature, b.anchor, b.projection_mat)):
        assert torch.equal(x, y)
    assert not torch.equal(a.anchor, syn.make_inputs(cfg, 6).anchor)


def test_camera_ring_projects_forward_points_to_image_centre():
    proj = syn.camera_ring(6, (704, 256))
    for c, yaw in enumerate(syn.CAMERA_YAWS_DEG):
        r = np.radians(yaw)
        p = torch.tensor([20 * np.cos(r), 20 * np.sin(r), 1.5, 1.0], dtype=torch.float32)
        q = proj[c] @ p
        assert q[2] > 0
        np.testing.assert_allclose((q[:2] / q[2]).numpy(), [352, 128], atol=1e-3)


def test_synthetic_visibility_fraction():
    """About 15 % of the point samples land in front of a camera and inside its image."""
    from oracle import dfa_torch as oto

    cfg = syn.config_standard(1)
    ins = syn.make_inputs(cfg, 0)
    params = syn.make_params(cfg, torch.Generator().manual_seed(100))
    kps = oto.key_points(ins.anchor, ins.instance_feature, params)
    uv, depth = oto.project_points_with_depth(kps, ins.projection_mat, ins.image_wh)
    _, vis = oto.visibility(uv, depth)
    assert 0.10 < vis.float().mean().item() < 0.22


def test_pack_feature_maps_has_no_cpu_path():
    """Packing runs on the GPU only (s4d_pack_feature_maps); CPU tensors are rejected loudly."""
    maps = [torch.zeros(1, 2, 64, 4, 6), torch.zeros(1, 2, 64, 2, 3)]
    with pytest.raises(ValueError, match="no CPU path"):
        ops.pack_feature_maps(maps)


def test_level_tables():
    shape, start, nf = ops.level_tables([(64, 176), (32, 88), (16, 44), (8, 22)], 6)
    assert nf == 6 * 14960
    assert start[1, 0].item() == 14960 and start[0, 3].item() == 64 * 176 + 32 * 88 + 16 * 44
    assert shape.dtype == torch.int32 and tuple(shape.shape) == (6, 4, 2)


def test_preprocess_parameters_matches_reference_keys():
    """The keys of model/deformable_feature_aggregation.py:954-995, from a module with the
    reference DFA's attribute structure."""
    cfg = syn.DFAConfig()
    p = syn.make_params(cfg, torch.Generator().manual_seed(0))

    class Lin(torch.nn.Module):
        def __init__(self, w, b):
            super().__init__()
            self.weight = torch.nn.Parameter(w)
            self.bias = torch.nn.Parameter(b)

    class KPS(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.fix_scale = torch.nn.Parameter(p["kps_fix_scale"], requires_grad=False)
            self.learnable_fc = Lin(p["kps_learnable_fc_weight"], p["kps_learnable_fc_bias"])

    class M(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.kps_generator = KPS()
            self.camera_encoder = torch.nn.Sequential(
                Lin(p["cam_linear1_weight"], p["cam_linear1_bias"]), torch.nn.ReLU(),
                Lin(p["cam_ln1_weight"], p["cam_ln1_bias"]),
                Lin(p["cam_linear2_weight"], p["cam_linear2_bias"]), torch.nn.ReLU(),
                Lin(p["cam_ln2_weight"], p["cam_ln2_bias"]))
            self.weights_fc = Lin(p["weights_fc_weight"], p["weights_fc_bias"])
            self.output_proj = Lin(p["output_proj_weight"], p["output_proj_bias"])

    got = preprocess_dfa_parameters(M())
    assert set(got) == set(p)
    for k in p:
        assert torch.equal(got[k], p[k]), k


def test_module_rejects_cpu_device_and_missing_params():
    p = syn.make_params(syn.DFAConfig(), torch.Generator().manual_seed(0))
    with pytest.raises(ValueError, match="CUDA"):
        DeformableFeatureAggregation("cpu", p)
    bad = dict(p)
    del bad["weights_fc_bias"]
    with pytest.raises(KeyError):
        DeformableFeatureAggregation("cuda:0", bad)


def test_refine_anchors_keeps_unit_yaw():
    gen = torch.Generator().manual_seed(0)
    a = syn.make_anchors(1, 100, gen)
    r = syn.refine_anchors(a, gen)
    n = r[..., 6:8].norm(dim=-1)
    np.testing.assert_allclose(n.numpy(), 1.0, atol=1e-5)
    assert (r[..., 0:3] - a[..., 0:3]).abs().max() < 1.0


def _fastdiv(d):
    """Python replica of FastDiv (csrc/common.cuh): l = ceil(log2 d), m = floor(2^32 (2^l - d) / d) + 1."""
    l = 0
    while (1 << l) < d:
        l += 1
    m = ((1 << 32) * ((1 << l) - d)) // d + 1
    m &= 0xFFFFFFFF
    return lambda n: ((((n * m) >> 32) + n) & 0xFFFFFFFF) >> l


@pytest.mark.parametrize("d", [1, 2, 3, 6, 7, 13, 78, 900, 1800, 3600, 65537, 1 << 20, (1 << 31) - 1])
def test_fastdiv_is_exact_below_2_31(d):
    import random

    q = _fastdiv(d)
    rng = random.Random(d)
    ns = [0, 1, d - 1, d, d + 1, (1 << 31) - 1, (1 << 31) - 2, (1 << 30)]
    ns += [rng.randrange(1 << 31) for _ in range(20000)]
    ns += [k * d + r for k in (1, 2, 1000, ((1 << 31) - 1) // d) for r in (-1, 0, 1) if 0 <= k * d + r < (1 << 31)]
    for n in ns:
        assert q(n) == n // d, (n, d)


def test_chained_camera_terms_links_and_unlinks():
    """Within the block each layer points at the one after it (the last at nothing); the links
    are removed on exit, also when the block raises."""
    from types import SimpleNamespace

    from sparse4d_tt_b200 import chained_camera_terms

    layers = [SimpleNamespace(next_layer=None) for _ in range(4)]
    with chained_camera_terms(layers):
        assert [m.next_layer for m in layers] == layers[1:] + [None]
    assert all(m.next_layer is None for m in layers)
    with pytest.raises(RuntimeError):
        with chained_camera_terms(layers):
            raise RuntimeError("a layer failed")
    assert all(m.next_layer is None for m in layers)
    with chained_camera_terms([]):
        pass


def test_camera_operators_have_no_cpu_path():
    """The camera encoder operators (two launches, and the one-launch camera terms with the
    softmax factors) run on the GPU only; CPU tensors are rejected before any library call."""
    cfg = syn.DFAConfig(bs=1)
    params = syn.make_params(cfg, torch.Generator().manual_seed(3))
    w = [params[k] for k in ("cam_linear1_weight", "cam_linear1_bias", "cam_ln1_weight", "cam_ln1_bias",
                             "cam_linear2_weight", "cam_linear2_bias", "cam_ln2_weight", "cam_ln2_bias",
                             "weights_fc_weight", "weights_fc_bias")]
    proj = torch.eye(4).expand(1, 6, 4, 4).contiguous()
    logits = torch.empty(1, 6, 416)
    with pytest.raises(ValueError, match="no CPU path"):
        ops.camera_logits_into(logits, proj, *w)
    with pytest.raises(ValueError, match="no CPU path"):
        ops.camera_terms_into(logits, proj, *w, factors=torch.empty(16))
