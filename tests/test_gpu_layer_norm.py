"""s4d_layer_norm (the decoder's LayerNorms) against float64 nn.LayerNorm: every width it
implements, row counts from 1 to the 32-frame decoder's 28,800, with and without the affine
part, and inputs with a large common offset (where a one-pass variance would cancel)."""
import pytest
import torch
import torch.nn.functional as F

from sparse4d_tt_b200 import ops

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("width", [32, 64, 128, 256, 512])
@pytest.mark.parametrize("rows", [1, 7, 1000, 28800])
def test_layer_norm_matches_float64(cuda_device, width, rows):
    gen = torch.Generator().manual_seed(width * 7 + rows)
    x = (torch.randn(rows, width, generator=gen) * 3 + 50).cuda()
    w = torch.randn(width, generator=gen).cuda()
    b = torch.randn(width, generator=gen).cuda()
    got = ops.layer_norm(x, w, b)
    ref = F.layer_norm(x.double(), (width,), w.double(), b.double(), 1e-5)
    torch.cuda.synchronize()
    err = (got.double() - ref).abs().max().item()
    assert err <= 2e-5 * (1 + w.abs().max().item()), err
    plain = ops.layer_norm(x, None, None)
    ref0 = F.layer_norm(x.double(), (width,), None, None, 1e-5)
    assert (plain.double() - ref0).abs().max().item() <= 2e-5


def test_layer_norm_batched_shape_and_head_path(cuda_device):
    """[bs, A, C] inputs keep their shape; the head's helper routes the contiguous fp32 rows to
    the kernel and anything else to torch."""
    from sparse4d_tt_b200.head import _layer_norm

    x = torch.randn(2, 900, 256, device="cuda")
    w, b = torch.randn(256, device="cuda"), torch.randn(256, device="cuda")
    y = _layer_norm(x, w, b)
    assert y.shape == x.shape
    assert torch.allclose(y, F.layer_norm(x, (256,), w, b, 1e-5), atol=1e-5)
    odd = torch.randn(5, 48, device="cuda")
    assert torch.allclose(_layer_norm(odd, torch.ones(48, device="cuda"), torch.zeros(48, device="cuda")),
                          F.layer_norm(odd, (48,)), atol=1e-6)
