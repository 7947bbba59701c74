"""The bench's deterministic counts (CPU): in-bounds samples and unique tap pixels, checked
against grid_sample itself (zeros padding, align_corners=False) on seeded locations."""
import os
import sys

import torch
import torch.nn.functional as F

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import bench  # noqa: E402

SHAPES = [(16, 44), (8, 22), (4, 11), (2, 6)]


def _locations(seed, bs=2, A=50, nc=3, P=5):
    g = torch.Generator().manual_seed(seed)
    return torch.rand(bs, A, nc, P, 2, generator=g, dtype=torch.float32) * 1.6 - 0.3


def test_inbounds_samples_match_grid_sample_of_ones():
    """A sample has an in-bounds tap exactly when grid_sample of an all-ones map is positive there
    (every in-bounds tap of such a sample has a positive bilinear weight)."""
    loc = _locations(3)
    bs, A, nc, P, _ = loc.shape
    want = 0
    for h, w in SHAPES:
        ones = torch.ones(bs * nc, 1, h, w)
        grid = (loc.permute(0, 2, 1, 3, 4).reshape(bs * nc, A, P, 2) * 2 - 1)
        v = F.grid_sample(ones, grid, mode="bilinear", padding_mode="zeros", align_corners=False)
        want += int((v > 0).sum())
    assert bench.inbounds_samples(loc, SHAPES) == want


def test_unique_tap_pixels_match_direct_enumeration():
    """The unique rows the taps touch, against a plain enumeration of every sample's in-bounds
    taps (grid_sample's unnormalisation ((g + 1) * W - 1) / 2 with g = 2u - 1, in fp32)."""
    loc = _locations(5, bs=1, A=20, nc=2, P=3)
    bs, A, nc, P, _ = loc.shape
    hw = [h * w for h, w in SHAPES]
    start = torch.tensor([[c * sum(hw) + sum(hw[:l]) for l in range(len(SHAPES))] for c in range(nc)],
                         dtype=torch.int32)
    num_feat = nc * sum(hw)
    want = set()
    for c in range(nc):
        for l, (h, w) in enumerate(SHAPES):
            ix = ((loc[0, :, c, :, 0] * 2 - 1 + 1) * w - 1) * 0.5
            iy = ((loc[0, :, c, :, 1] * 2 - 1 + 1) * h - 1) * 0.5
            x0s, y0s = ix.floor().long().tolist(), iy.floor().long().tolist()
            for a in range(A):
                for p in range(P):
                    for dx in (0, 1):
                        for dy in (0, 1):
                            x, y = x0s[a][p] + dx, y0s[a][p] + dy
                            if 0 <= x < w and 0 <= y < h:
                                want.add(int(start[c, l]) + y * w + x)
    assert bench.unique_tap_pixels(loc, SHAPES, start, num_feat) == len(want)
