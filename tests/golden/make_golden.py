"""Generate the golden fixtures by running the REFERENCE's own PyTorch DFA.

Run where the reference checkout is present, with ``REF_ROOT`` set to its root, from the
repository root:

    REF_ROOT=<reference checkout> python tests/golden/make_golden.py [fixture name ...]

It imports ``test/dfa_pcc.py`` of the reference with a stand-in ``ttnn`` module (the
reference imports ttnn at module top, ``test/dfa_pcc.py:37``, but its PyTorch DFA never
calls it), loads the seeded parameters into ``_PTDeformableFeatureAggregation``
(``test/dfa_pcc.py:250-358``), runs it on seeded inputs and writes ``tests/golden/*.npz``:
checksums of every input and parameter, intermediate tensors (keypoints, projected
points, depth, weights) and outputs, whole for the small cases and as per-row checksums
plus a fixed sample of full rows for the full-size ones.  The tests regenerate the inputs
from the seeds and compare the oracle, and on a GPU the CUDA path, against these files.
"""
from __future__ import annotations

import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
REF_ROOT = os.environ.get("REF_ROOT", "")
sys.path.insert(0, REPO)
sys.path.insert(0, HERE)

import fixtures as fx  # noqa: E402
from sparse4d_tt_b200 import synthetic as syn  # noqa: E402


def import_reference():
    if not REF_ROOT or not os.path.isdir(os.path.join(REF_ROOT, "test")):
        raise SystemExit("make_golden.py: set REF_ROOT to the root of the reference checkout")
    stub = types.ModuleType("ttnn")

    class _Any:
        def __init__(self, *a, **k):
            pass

        def __getattr__(self, n):
            if n.startswith("__"):
                raise AttributeError(n)
            return _Any()

        def __call__(self, *a, **k):
            return _Any()

    def _mod_getattr(n):
        if n.startswith("__"):
            raise AttributeError(n)
        return _Any()

    stub.__getattr__ = _mod_getattr
    sys.modules["ttnn"] = stub
    sys.path.insert(0, REF_ROOT)
    sys.path.insert(0, os.path.join(REF_ROOT, "test"))
    import dfa_pcc  # noqa: E402

    return dfa_pcc


def build_reference_module(ref, cfg: syn.DFAConfig, params):
    m = ref._PTDeformableFeatureAggregation(
        embed_dims=cfg.embed_dims, num_groups=cfg.num_groups, num_levels=cfg.num_levels,
        num_cams=cfg.num_cams, num_learnable_pts=cfg.num_learnable_pts, use_camera_embed=True,
        residual_mode="cat", fix_scale=cfg.fix_scale,
    )
    enc = m.camera_encoder
    with torch.no_grad():
        m.kps_generator.fix_scale.copy_(params["kps_fix_scale"])
        m.kps_generator.learnable_fc.weight.copy_(params["kps_learnable_fc_weight"])
        m.kps_generator.learnable_fc.bias.copy_(params["kps_learnable_fc_bias"])
        for idx, key in ((0, "cam_linear1"), (3, "cam_linear2")):
            enc[idx].weight.copy_(params[key + "_weight"])
            enc[idx].bias.copy_(params[key + "_bias"])
        for idx, key in ((2, "cam_ln1"), (5, "cam_ln2")):
            enc[idx].weight.copy_(params[key + "_weight"])
            enc[idx].bias.copy_(params[key + "_bias"])
        m.weights_fc.weight.copy_(params["weights_fc_weight"])
        m.weights_fc.bias.copy_(params["weights_fc_bias"])
        m.output_proj.weight.copy_(params["output_proj_weight"])
        m.output_proj.bias.copy_(params["output_proj_bias"])
    return m.eval()


def run_reference(m, inst, anchor, embed, maps, proj, wh):
    """Reference forward plus its intermediates, each from the reference's own methods."""
    metas = {"projection_mat": proj, "image_wh": wh}
    with torch.no_grad():
        kps = m.kps_generator(anchor, inst)
        weights = m._get_weights(inst, embed, metas)
        pts2d = m.project_points(kps, proj, wh)  # [bs, Ncam, A, P, 2]
        # depth is not returned by the reference; the same matmul gives it
        ext = torch.cat([kps, torch.ones_like(kps[..., :1])], dim=-1)
        depth = torch.matmul(proj[:, :, None, None], ext[:, None, ..., None]).squeeze(-1)[..., 2]
        feats = m.feature_sampling(maps, kps, proj, wh)
        fused = m.multi_view_level_fusion(feats, weights).sum(dim=2)
        out = m(instance_feature=inst, anchor=anchor, anchor_embed=embed, feature_maps=maps, metas=metas)
    return {"key_points": kps, "weights": weights, "uv": pts2d, "depth": depth, "fused": fused, "out": out}


def input_checksums(prefix, tensors, params):
    d = {}
    for name, t in zip(("instance_feature", "anchor", "anchor_embed", "projection_mat", "image_wh"), tensors):
        d[f"ck_{name}"] = fx.checksum(t)
    for i, fm in enumerate(tensors[5]):
        d[f"ck_map{i}"] = fx.checksum(fm)
    for k, v in params.items():
        d[f"ck_param_{k}"] = fx.checksum(v)
    return d


def masks(res):
    uv, depth = res["uv"], res["depth"]
    mask = depth > 1e-5
    vis = mask & (uv[..., 0] >= 0) & (uv[..., 0] <= 1) & (uv[..., 1] >= 0) & (uv[..., 1] <= 1)
    return mask.permute(0, 2, 1, 3), vis.permute(0, 2, 1, 3)


def save_small(path, cfg, seed, pseed, feature_dtype, res, ins, params, meta):
    mask, vis = masks(res)
    d = dict(meta)
    d.update(input_checksums("", (ins.instance_feature, ins.anchor, ins.anchor_embed, ins.projection_mat,
                                  ins.image_wh, ins.feature_maps), params))
    d.update({
        "key_points": res["key_points"].numpy(), "uv": res["uv"].numpy(), "depth": res["depth"].numpy(),
        "weights_b0a0_3": res["weights"][0, :4].numpy(), "fused": res["fused"].numpy(),
        "out": res["out"][..., : cfg.embed_dims].numpy(),
        "mask_bits": fx.pack_bits(mask), "vis_bits": fx.pack_bits(vis),
        "vis_idx": torch.nonzero(vis).numpy().astype(np.int32),
    })
    np.savez_compressed(path, **d)


def save_large(path, cfg, res, ck_inputs, meta):
    mask, vis = masks(res)
    bs, A = res["fused"].shape[:2]
    rows = fx.sample_rows(bs * A)
    fused = res["fused"].reshape(bs * A, -1)
    out = res["out"][..., : cfg.embed_dims].reshape(bs * A, -1)
    d = dict(meta)
    d.update(ck_inputs)
    d.update({
        "rows": rows, "fused_rows": fused[rows].numpy(), "out_rows": out[rows].numpy(),
        "fused_row_ck": np.stack([fused.double().sum(1).numpy(), (fused.double() ** 2).sum(1).numpy()], 1),
        "out_row_ck": np.stack([out.double().sum(1).numpy(), (out.double() ** 2).sum(1).numpy()], 1),
        "kp_rows": res["key_points"].reshape(bs * A, -1, 3)[rows].numpy(),
        "uv_rows": res["uv"].permute(0, 2, 1, 3, 4).reshape(bs * A, -1)[rows].numpy(),
        "mask_bits": fx.pack_bits(mask), "vis_bits": fx.pack_bits(vis),
        "n_visible": np.array(int(vis.sum())),
    })
    np.savez_compressed(path, **d)


def synthetic_case(ref, name, cfg, seed, pseed, feature_dtype=None, large=False):
    ins = syn.make_inputs(cfg, seed, feature_dtype=feature_dtype)
    params = syn.make_params(cfg, torch.Generator().manual_seed(pseed))
    m = build_reference_module(ref, cfg, params)
    res = run_reference(m, ins.instance_feature, ins.anchor, ins.anchor_embed, ins.feature_maps,
                        ins.projection_mat, ins.image_wh)
    meta = {
        "seed": np.array(seed), "param_seed": np.array(pseed),
        "bs": np.array(cfg.bs), "num_anchor": np.array(cfg.num_anchor), "num_cams": np.array(cfg.num_cams),
        "image_wh": np.array(cfg.image_wh), "strides": np.array(cfg.strides),
        "bf16_maps": np.array(feature_dtype == torch.bfloat16), "torch_version": np.array(torch.__version__),
    }
    path = os.path.join(HERE, name + ".npz")
    if large:
        ck = input_checksums("", (ins.instance_feature, ins.anchor, ins.anchor_embed, ins.projection_mat,
                                  ins.image_wh, ins.feature_maps), params)
        save_large(path, cfg, res, ck, meta)
    else:
        save_small(path, cfg, seed, pseed, feature_dtype, res, ins, params, meta)
    print(f"{name}: visible={int(masks(res)[1].sum())} -> {os.path.getsize(path)} bytes")


def reference_dummy(ref, name, bs):
    """The reference's own e2e case: ``create_dummy_inputs(bs)`` then ``build_pt_dfa()``
    under the global RNG, exactly as ``test_e2e_pcc`` (``test/dfa_pcc.py:496-519``)."""
    inst, anchor, embed, maps, metas = ref.create_dummy_inputs(bs, 900, 6, 256)
    m = ref.build_pt_dfa().eval()
    params = ref.preprocess_dfa_parameters_from_pt(m)
    for k in ("cam_ln1_weight", "cam_ln1_bias", "cam_ln2_weight", "cam_ln2_bias"):
        params[k] = params[k].clone()
    res = run_reference(m, inst, anchor, embed, maps, metas["projection_mat"], metas["image_wh"])
    cfg = syn.DFAConfig(bs=bs)
    ck = input_checksums("", (inst, anchor, embed, metas["projection_mat"], metas["image_wh"], maps), params)
    meta = {"bs": np.array(bs), "torch_version": np.array(torch.__version__)}
    path = os.path.join(HERE, name + ".npz")
    save_large(path, cfg, res, ck, meta)
    print(f"{name}: visible={int(masks(res)[1].sum())} -> {os.path.getsize(path)} bytes")


def reference_dummy_kps_inputs(ref, name, batches=(1, 2)):
    """Exact input bits of the reference's own e2e case (``create_dummy_inputs`` + ``build_pt_dfa``,
    seed 42) for the keypoint path: anchors, the learnable-keypoint logits of the reference
    module's own ``learnable_fc``, projection matrices and image sizes.  These are the inputs the
    ``refdummy_bs*`` masks and indices were computed from; a host whose CPU rounds ``sin``/``cos``
    or the linear differently in the last bit still feeds the GPU exactly these."""
    out = {}
    for bs in batches:
        inst, anchor, embed, maps, metas = ref.create_dummy_inputs(bs, 900, 6, 256)
        m = ref.build_pt_dfa().eval()
        with torch.no_grad():
            learn = m.kps_generator.learnable_fc(inst)
        out[f"anchor_bs{bs}"] = anchor.numpy()
        out[f"learn_bs{bs}"] = learn.numpy()
        out[f"proj_bs{bs}"] = metas["projection_mat"].numpy()
        out[f"wh_bs{bs}"] = metas["image_wh"].numpy()
        out[f"fix_scale_bs{bs}"] = m.kps_generator.fix_scale.detach().numpy()
    path = os.path.join(HERE, name + ".npz")
    np.savez_compressed(path, **out)
    print(f"{name}: {sorted(out)} -> {os.path.getsize(path)} bytes")


def import_reference_head():
    """The reference's head twin module ``test/sparse4d_head_pcc.py`` (its ttnn and TT model imports
    stand in through the same stub as ``import_reference``)."""
    import_reference()
    import sparse4d_head_pcc  # noqa: E402

    return sparse4d_head_pcc


def head_twin(name, seed=42, bs=1):
    """The reference's own single-frame head test case (``test/sparse4d_head_pcc.py:530-565``):
    ``_PTSparse4DHead`` built under ``torch.manual_seed(42)``, maps and projections x0.1, the
    forward with debug intermediates.  Stores checksums of every parameter (state-dict order) and
    input, every decoder's prediction whole, the classification and quality of the decoders that
    return them, and the instance feature after each step."""
    hp = import_reference_head()
    torch.manual_seed(seed)
    head = hp._PTSparse4DHead(embed_dims=256, num_decoder=6, num_single_frame=1, num_anchor=900, num_temp=600,
                              num_cls=10, num_groups=8, decouple_attn=True).eval()
    maps = [torch.randn(bs, 6, 256, h, w) * 0.1 for h, w in ((64, 176), (32, 88), (16, 44), (8, 22))]
    metas = {"projection_mat": torch.randn(bs, 6, 4, 4) * 0.1,
             "image_wh": torch.tensor([[704.0, 256.0]]).unsqueeze(0).expand(bs, 6, 2).contiguous(),
             "timestamp": torch.zeros(bs)}
    with torch.no_grad():
        out = head(maps, metas, bs=bs, debug=True)
    d = {"seed": np.array(seed), "bs": np.array(bs), "torch_version": np.array(torch.__version__),
         "operation_order": np.array(head.operation_order)}
    d["param_names"] = np.array(list(head.state_dict().keys()))
    d["param_ck"] = np.stack([fx.checksum(v) for v in head.state_dict().values()])
    for i, m in enumerate(maps):
        d[f"ck_map{i}"] = fx.checksum(m)
    d["ck_projection_mat"] = fx.checksum(metas["projection_mat"])
    for i, pr in enumerate(out["prediction"]):
        d[f"prediction{i}"] = pr.numpy()
    for i, c in enumerate(out["classification"]):
        if c is not None:
            d[f"classification{i}"] = c.numpy()
    for i, q in enumerate(out["quality"]):
        if q is not None:
            d[f"quality{i}"] = q.numpy()
    for k, v in out["debug"].items():
        if k.startswith("step_") and not k.endswith("_anchor"):
            d["ck_" + k] = fx.checksum(v)
    path = os.path.join(HERE, name + ".npz")
    np.savez_compressed(path, **d)
    print(f"{name}: {len(d['param_names'])} parameters, {len(out['prediction'])} decoders -> "
          f"{os.path.getsize(path)} bytes")


def instance_bank_projection(name, seed=7, bs=2, num=600):
    """The reference's own InstanceBank._anchor_projection (model/instance_bank.py:322-369, plain
    torch) on seeded cached anchors, ego transforms and time gaps; inputs and outputs stored
    whole (small)."""
    import importlib

    if not REF_ROOT:
        raise SystemExit("make_golden.py: set REF_ROOT to the root of the reference checkout")
    sys.path.insert(0, REF_ROOT)
    ib = importlib.import_module("model.instance_bank")
    gen = torch.Generator().manual_seed(seed)
    anchor = syn.make_anchors(bs, num, gen)
    T = torch.zeros(bs, 4, 4)
    for b in range(bs):
        yaw = float(torch.rand(1, generator=gen)) * 0.4 - 0.2
        c, s_ = np.cos(yaw), np.sin(yaw)
        T[b, :3, :3] = torch.tensor([[c, -s_, 0.0], [s_, c, 0.0], [0.0, 0.0, 1.0]], dtype=torch.float32)
        T[b, :3, 3] = torch.rand(3, generator=gen) * 4.0 - 2.0
        T[b, 3, 3] = 1.0
    ti = -(torch.rand(bs, generator=gen) * 0.6)  # get() passes -(t_now - t_cached)
    out = ib.InstanceBank._anchor_projection(anchor, T, ti)
    path = os.path.join(HERE, name + ".npz")
    np.savez_compressed(path, anchor=anchor.numpy(), T=T.numpy(), time_interval=ti.numpy(), out=out.numpy())
    print(f"{name}: {bs}x{num} anchors -> {os.path.getsize(path)} bytes")


def main():
    torch.set_num_threads(os.cpu_count() or 1)
    ref = import_reference()
    small = syn.DFAConfig(bs=2, num_anchor=40, image_wh=(128, 64))
    jobs = {
        "small_b2_s3": lambda: synthetic_case(ref, "small_b2_s3", small, seed=3, pseed=103),
        "small_b1_s4_cam3": lambda: synthetic_case(
            ref, "small_b1_s4_cam3", syn.DFAConfig(bs=1, num_anchor=24, num_cams=3, image_wh=(96, 64)), seed=4,
            pseed=104),
        "standard_s0_fp32": lambda: synthetic_case(ref, "standard_s0_fp32", syn.config_standard(1), seed=0,
                                                   pseed=100, large=True),
        "standard_s1_bf16": lambda: synthetic_case(ref, "standard_s1_bf16", syn.config_standard(1), seed=1,
                                                   pseed=101, feature_dtype=torch.bfloat16, large=True),
        "highres_s2_bf16": lambda: synthetic_case(ref, "highres_s2_bf16", syn.config_highres(1, 1800), seed=2,
                                                  pseed=102, feature_dtype=torch.bfloat16, large=True),
        "refdummy_bs1": lambda: reference_dummy(ref, "refdummy_bs1", 1),
        "refdummy_bs2": lambda: reference_dummy(ref, "refdummy_bs2", 2),
        "refdummy_kps_inputs": lambda: reference_dummy_kps_inputs(ref, "refdummy_kps_inputs"),
        "head_twin_s42": lambda: head_twin("head_twin_s42"),
        "instance_bank_projection": lambda: instance_bank_projection("instance_bank_projection"),
    }
    names = sys.argv[1:] or list(jobs)
    for n in names:
        jobs[n]()


if __name__ == "__main__":
    main()
