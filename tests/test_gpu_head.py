"""The decoder chain around the DFA (sparse4d-tt_b200/head.py) on the GPU: refinement -> anchor
re-encoding between the stacked DFA layers, with the dense layers around them, checked against
the reference's single-frame head twin (fixture head_twin_s42, written by running the reference
itself; the oracle restatement rebuilds the same parameters under seed 42) and replayed as one
CUDA graph."""
import numpy as np
import pytest
import torch

import fixtures as fx
from helpers import pcc
from oracle import head_torch as oh
from sparse4d_tt_b200 import synthetic as syn
from sparse4d_tt_b200.head import HeadGraph, Sparse4DHead, preprocess_head_parameters

pytestmark = pytest.mark.gpu

SHAPES = [(64, 176), (32, 88), (16, 44), (8, 22)]


@pytest.fixture(scope="module")
def twin():
    g = fx.load("head_twin_s42")
    head = oh.build_head(int(g["seed"]))
    maps, proj, wh = oh.head_inputs(int(g["bs"]))
    return g, head, maps, proj, wh


def _compare(got, ref, what, atol):
    got, ref = got.detach().cpu().double(), torch.as_tensor(ref).double()
    err = (got - ref).abs().max().item()
    p = pcc(got, ref)
    print(f"{what}: max abs err {err:.2e}, pcc {p:.7f}")
    assert err <= atol and p >= 0.99999, what


def test_head_fp32_matches_reference_twin(cuda_device, twin):
    """fp32 maps and fp32 linears: every decoder's predictions, and the first and last
    decoders' classifications and qualities, against the reference twin's outputs."""
    g, head, maps, proj, wh = twin
    d = torch.device("cuda:0")
    gh = Sparse4DHead(d, preprocess_head_parameters(head), {"FEATURE_DTYPE": torch.float32})
    out = gh.forward([m.to(d) for m in maps], proj.to(d), wh.to(d), SHAPES, int(g["bs"]))
    torch.cuda.synchronize()
    assert len(out["prediction"]) == 6
    for i, pr in enumerate(out["prediction"]):
        _compare(pr, g[f"prediction{i}"], f"prediction[{i}]", 2e-3)
    for i, c in enumerate(out["classification"]):
        assert (c is None) == (f"classification{i}" not in g)
        if c is not None:
            _compare(c, g[f"classification{i}"], f"cls[{i}]", 2e-3)
            _compare(out["quality"][i], g[f"quality{i}"], f"quality[{i}]", 2e-3)


def _ring_case(bs=2, seed=9):
    cfg = syn.DFAConfig(bs=bs)
    ins = syn.make_inputs(cfg, seed, feature_dtype=torch.bfloat16)
    return cfg, ins


@pytest.mark.parametrize("attention", [torch.float32, torch.bfloat16])
def test_head_graph_replay_equals_eager_and_oracle(cuda_device, twin, attention):
    """The benchmark configuration (bf16 maps, TF32 linears; attention in fp32 or bf16) on the
    synthetic camera ring with anchors spread over the scene: one CUDA-graph replay of the whole
    decoder equals the eager pass bit for bit, and both follow the fp32 oracle head within the
    bf16/TF32 tolerance."""
    _, head, _, _, _ = twin
    d = torch.device("cuda:0")
    cfg, ins = _ring_case()
    anchor = ins.anchor
    gh = Sparse4DHead(d, preprocess_head_parameters(head), {"FEATURE_DTYPE": torch.bfloat16,
                                                             "MATMUL_PRECISION": "tf32",
                                                             "ATTENTION_DTYPE": attention})
    from sparse4d_tt_b200 import ops

    packed = ops.pack_feature_maps([m.to(d) for m in ins.feature_maps], dtype=torch.bfloat16)
    eager = gh.forward(packed, ins.projection_mat.to(d), ins.image_wh.to(d), cfg.spatial_shapes, cfg.bs,
                       anchor=anchor.to(d))
    eager_pred = [p.clone() for p in eager["prediction"]]
    graph = HeadGraph(gh, cfg.bs, cfg.spatial_shapes)
    out = graph.run(packed[0], ins.projection_mat.to(d), ins.image_wh.to(d), anchor.to(d))
    torch.cuda.synchronize()
    for a, b in zip(out["prediction"], eager_pred):
        assert torch.equal(a, b)
    ref = head(ins.feature_maps, ins.projection_mat, ins.image_wh, bs=cfg.bs, anchor=anchor)
    prev_g, prev_r = anchor, anchor
    for i, (a, r) in enumerate(zip(eager_pred, ref["prediction"])):
        a = a.cpu()
        p = pcc(a - prev_g, r - prev_r)  # this decoder's refinement step
        print(f"decoder {i} refinement vs fp32 oracle: pcc {p:.7f}")
        assert p >= 0.999
        prev_g, prev_r = a, r
