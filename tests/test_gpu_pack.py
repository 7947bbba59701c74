"""Packing of per-level maps into the gather's channels-last layout (s4d_pack_feature_maps)
against a torch restatement of the layout: bit-exact, casts included (both round to nearest
even)."""
import numpy as np
import pytest
import torch

from oracle import dfa_numpy as onp
from sparse4d_tt_b200 import ops

pytestmark = pytest.mark.gpu

SHAPES = [(64, 176), (32, 88), (16, 44), (8, 22)]


def _reference(maps_nchw, dtype):
    bs, nc = maps_nchw[0].shape[:2]
    cols = [f.flatten(3).transpose(2, 3) for f in maps_nchw]  # [bs, Ncam, HW, C]
    return torch.cat(cols, dim=2).reshape(bs, -1, maps_nchw[0].shape[2]).to(dtype)


@pytest.mark.parametrize("src,dst", [(torch.float32, torch.bfloat16), (torch.float32, torch.float32),
                                     (torch.bfloat16, torch.bfloat16), (torch.bfloat16, torch.float32)])
@pytest.mark.parametrize("channels_last", [False, True])
def test_pack_matches_torch_layout(cuda_device, src, dst, channels_last):
    dev = torch.device("cuda:0")
    g = torch.Generator(device=dev).manual_seed(3)
    shapes = SHAPES + [(5, 7)]  # a level that fills no whole 64-pixel tile
    maps = [torch.randn(2, 6, 256, h, w, generator=g, device=dev).to(src) for h, w in shapes]
    ref = _reference(maps, dst)
    src_maps = [m.permute(0, 1, 3, 4, 2).contiguous() for m in maps] if channels_last else maps
    packed, shape, start = ops.pack_feature_maps(src_maps, dtype=dst, channels_last=channels_last)
    torch.cuda.synchronize()
    assert packed.dtype == dst and torch.equal(packed, ref)
    assert shape.tolist() == [[list(s) for s in shapes]] * 6
    per_cam = sum(h * w for h, w in shapes)
    assert start[1, 0].item() == per_cam and start[0, 1].item() == 64 * 176


def test_pack_into_preallocated_buffer(cuda_device):
    dev = torch.device("cuda:0")
    maps = [torch.randn(1, 3, 128, h, w, device=dev) for h, w in SHAPES]
    out = torch.full((1, 3 * sum(h * w for h, w in SHAPES), 128), -1.0, dtype=torch.bfloat16, device=dev)
    packed, _, _ = ops.pack_feature_maps(maps, dtype=torch.bfloat16, out=out)
    torch.cuda.synchronize()
    assert packed.data_ptr() == out.data_ptr() and torch.equal(out, _reference(maps, torch.bfloat16))


@pytest.mark.parametrize("channels_last", [False, True])
def test_pack_matches_numpy_oracle(cuda_device, channels_last):
    rng = np.random.default_rng(1)
    maps = [rng.standard_normal((2, 3, 256, h, w)).astype(np.float32) for h, w in ((4, 6), (2, 3))]
    feat_np, shape_np, start_np = onp.pack_feature_maps(maps)
    tm = [torch.from_numpy(m).cuda() for m in maps]
    if channels_last:
        tm = [m.permute(0, 1, 3, 4, 2).contiguous() for m in tm]
    feat, shape, start = ops.pack_feature_maps(tm, channels_last=channels_last)
    assert np.array_equal(feat.cpu().numpy(), feat_np)
    assert np.array_equal(shape.cpu().numpy(), shape_np) and np.array_equal(start.cpu().numpy(), start_np)
