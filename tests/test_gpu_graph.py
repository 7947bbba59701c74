"""CUDA-graph execution (graph.py): a captured stack of DFA layers replays the eager chain bit
for bit, picks up new inputs written into its static buffers, and recomputes the per-frame
camera terms on every replay."""
import pytest
import torch

from oracle import dfa_torch as oto
from helpers import max_rel_err, pcc
from sparse4d_tt_b200 import DFAStack, DeformableFeatureAggregation, chained_camera_terms, ops
from sparse4d_tt_b200 import synthetic as syn

pytestmark = pytest.mark.gpu

CONFIG = {"FEATURE_DTYPE": torch.bfloat16, "MATMUL_PRECISION": "tf32"}


def _layers(cfg, n, seed=300):
    return [DeformableFeatureAggregation("cuda:0", syn.make_params(cfg, torch.Generator().manual_seed(seed + i)),
                                         CONFIG) for i in range(n)]


def _inputs(cfg, n, seed):
    ins = syn.make_inputs(cfg, seed, feature_dtype=torch.bfloat16)
    gen = torch.Generator().manual_seed(seed + 1)
    anchors, a = [], ins.anchor
    for _ in range(n):
        anchors.append(a)
        a = syn.refine_anchors(a, gen)
    embeds = [syn.normal(tuple(ins.anchor_embed.shape), gen) for _ in range(n)]
    return ins, anchors, embeds


def _eager(layers, cfg, ins, anchors, embeds, packed):
    d = torch.device("cuda:0")
    inst, out = ins.instance_feature.to(d), None
    for i, mod in enumerate(layers):
        mod.reset_frame_cache()
        out = mod.run(inst, anchors[i].to(d), embeds[i].to(d), packed, ins.projection_mat.to(d), ins.image_wh.to(d),
                      cfg.spatial_shapes, cfg.bs, cfg.num_anchor)
        inst = out[..., :256]
    return out


@pytest.mark.parametrize("bs,n_layers", [(1, 1), (2, 3)])
def test_stack_replay_equals_eager(cuda_device, bs, n_layers):
    cfg = syn.DFAConfig(bs=bs, num_anchor=900)
    layers = _layers(cfg, n_layers)
    stack = DFAStack(layers, bs, cfg.num_anchor, cfg.spatial_shapes)
    d = torch.device("cuda:0")
    for seed in (5, 6):  # two different batches through the same graph
        ins, anchors, embeds = _inputs(cfg, n_layers, seed)
        packed = ops.pack_feature_maps([m.to(d) for m in ins.feature_maps], dtype=torch.bfloat16)
        out = stack.run(ins.instance_feature, anchors, embeds, packed[0], ins.projection_mat, ins.image_wh).clone()
        torch.cuda.synchronize()
        ref = _eager(layers, cfg, ins, anchors, embeds, packed)
        torch.cuda.synchronize()
        assert torch.equal(out, ref), (seed, (out - ref).abs().max().item())


def test_chained_camera_terms_eager_equal_unchained(cuda_device):
    """With the layers chained, each layer starts the next layer's camera terms on that layer's
    side stream before its own gather (10 frames: 9,000 rows, where eager calls use the side
    stream); the outputs are bitwise those of the unchained layers, and the links are gone
    after the block."""
    cfg = syn.DFAConfig(bs=10, num_anchor=900)
    n = 3
    layers = _layers(cfg, n)
    d = torch.device("cuda:0")
    ins, anchors, embeds = _inputs(cfg, n, 11)
    packed = ops.pack_feature_maps([m.to(d) for m in ins.feature_maps], dtype=torch.bfloat16)
    proj, wh = ins.projection_mat.to(d), ins.image_wh.to(d)
    anchors, embeds = [a.to(d) for a in anchors], [e.to(d) for e in embeds]

    def run(chain):
        for mod in layers:
            mod.reset_frame_cache()
        inst, out = ins.instance_feature.to(d), None
        with chained_camera_terms(layers if chain else []):
            for i, mod in enumerate(layers):
                out = mod.run(inst, anchors[i], embeds[i], packed, proj, wh, cfg.spatial_shapes, cfg.bs, cfg.num_anchor)
                if chain and i + 1 < n:
                    assert layers[i + 1]._cached_camera_logits is not None  # started by layer i
                inst = out[..., :256]
        return out.clone()

    ref = run(False)
    got = run(True)
    torch.cuda.synchronize()
    assert torch.equal(got, ref), (got - ref).abs().max().item()
    assert all(m.next_layer is None for m in layers)


def test_stack_single_layer_against_oracle(cuda_device):
    cfg = syn.DFAConfig(bs=1, num_anchor=900)
    layers = _layers(cfg, 1, seed=77)
    stack = DFAStack(layers, 1, 900, cfg.spatial_shapes)
    ins, anchors, embeds = _inputs(cfg, 1, 9)
    packed = ops.pack_feature_maps([m.to("cuda:0") for m in ins.feature_maps], dtype=torch.bfloat16)
    out = stack.run(ins.instance_feature, anchors, embeds, packed[0], ins.projection_mat, ins.image_wh).cpu()
    params = syn.make_params(cfg, torch.Generator().manual_seed(77))
    ref = oto.dfa_layer(params, ins.instance_feature, anchors[0], embeds[0], ins.feature_maps, ins.projection_mat,
                        ins.image_wh)
    assert pcc(out, ref) >= 0.9999 and max_rel_err(out, ref) <= 1e-2


def test_stack_recomputes_camera_terms(cuda_device):
    """A new projection written into the static buffer changes the result (the camera encoder
    is part of the graph, not a cached value)."""
    cfg = syn.DFAConfig(bs=1, num_anchor=128)
    layers = _layers(cfg, 1, seed=91)
    stack = DFAStack(layers, 1, 128, cfg.spatial_shapes)
    ins, anchors, embeds = _inputs(cfg, 1, 12)
    packed = ops.pack_feature_maps([m.to("cuda:0") for m in ins.feature_maps], dtype=torch.bfloat16)
    a = stack.run(ins.instance_feature, anchors, embeds, packed[0], ins.projection_mat, ins.image_wh).clone()
    proj2 = ins.projection_mat.clone()
    proj2[:, :, :3, :3] *= 1.02
    b = stack.run(projection_mat=proj2).clone()
    c = stack.run(projection_mat=ins.projection_mat).clone()
    torch.cuda.synchronize()
    assert not torch.equal(a, b) and torch.equal(a, c)


def test_stack_timed_replays(cuda_device):
    """time_gathers: each layer's gather launch is bracketed by event-record nodes of the graph,
    which hold the device times of the latest replay; timing changes nothing in the output."""
    cfg = syn.DFAConfig(bs=2, num_anchor=900)
    layers = _layers(cfg, 2, seed=41)
    plain = DFAStack(layers, 2, 900, cfg.spatial_shapes)
    timed = DFAStack(layers, 2, 900, cfg.spatial_shapes, time_gathers=True)
    ins, anchors, embeds = _inputs(cfg, 2, 13)
    packed = ops.pack_feature_maps([m.to("cuda:0") for m in ins.feature_maps], dtype=torch.bfloat16)
    a = plain.run(ins.instance_feature, anchors, embeds, packed[0], ins.projection_mat, ins.image_wh).clone()
    for _ in range(3):
        b = timed.run(ins.instance_feature, anchors, embeds, packed[0], ins.projection_mat, ins.image_wh)
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    t = timed.gather_times_ms()
    assert len(t) == 2 and all(0.0 < x < 50.0 for x in t), t
    assert all(m.event_log is None for m in layers)
    with pytest.raises(RuntimeError):
        plain.gather_times_ms()


def test_pipelined_stack_matches_stack(cuda_device):
    """PipelinedDFAStack: four batches streamed from pinned host memory through the two graphs
    (uploads overlapping replays) give exactly what one DFAStack gives on each batch."""
    from sparse4d_tt_b200 import PipelinedDFAStack

    cfg = syn.DFAConfig(bs=2, num_anchor=900)
    layers = _layers(cfg, 2, seed=320)
    pipe = PipelinedDFAStack(layers, cfg.bs, cfg.num_anchor, cfg.spatial_shapes)
    ref_stack = DFAStack(layers, cfg.bs, cfg.num_anchor, cfg.spatial_shapes)
    batches, outs = [], []
    for seed in (11, 12, 13, 14):
        ins, anchors, embeds = _inputs(cfg, 2, seed)
        packed = ops.pack_feature_maps([m.to("cuda:0") for m in ins.feature_maps], dtype=torch.bfloat16)
        host = dict(instance_feature=ins.instance_feature.pin_memory(), anchors=[a.pin_memory() for a in anchors],
                    anchor_embeds=[e.pin_memory() for e in embeds], mc_ms_feat=packed[0].cpu().pin_memory(),
                    projection_mat=ins.projection_mat.pin_memory(), image_wh=ins.image_wh.pin_memory())
        batches.append(host)
        outs.append(torch.empty(cfg.bs, cfg.num_anchor, 512, pin_memory=True))
    for host, out in zip(batches, outs):
        pipe.submit(out=out, **host)
    pipe.synchronize()
    for host, out in zip(batches, outs):
        ref = ref_stack.run(host["instance_feature"], host["anchors"], host["anchor_embeds"], host["mc_ms_feat"],
                            host["projection_mat"], host["image_wh"]).cpu()
        assert torch.equal(out, ref)
