"""The InstanceBank oracle against the reference's own projection (golden vectors made by
tests/golden/make_golden.py from model/instance_bank.py:322-369) and top-k semantics."""
import numpy as np
import torch

import fixtures as fx
from oracle import instance_bank_torch as oib


def test_projection_matches_reference_golden():
    g = fx.load("instance_bank_projection")
    out = oib.anchor_projection(torch.from_numpy(g["anchor"]), torch.from_numpy(g["T"]),
                                torch.from_numpy(g["time_interval"]))
    np.testing.assert_allclose(out.numpy(), g["out"], rtol=1e-6, atol=1e-6)


def test_projection_keeps_reference_yaw_slot_order():
    """Identity transform, no motion: the [cos, sin] pair is written to the (sin, cos) slots."""
    a = torch.zeros(1, 1, 11)
    a[0, 0, 6], a[0, 0, 7] = 0.6, 0.8  # sin, cos
    out = oib.anchor_projection(a, torch.eye(4)[None], None)
    assert out[0, 0, 6].item() == 0.800000011920929 and abs(out[0, 0, 7].item() - 0.6) < 1e-7


def test_topk_stable_matches_torch_without_ties_and_orders_ties_by_index():
    g = torch.Generator().manual_seed(0)
    s = torch.rand(3, 900, generator=g)
    v, i = oib.topk_stable(s, 300)
    tv, ti = torch.topk(s, 300, dim=-1)
    assert torch.equal(v, tv) and torch.equal(i, ti)
    s = torch.zeros(1, 10)
    s[0, 7] = 1.0
    _, i = oib.topk_stable(s, 4)
    assert i.tolist() == [[7, 0, 1, 2]]


def test_oracle_sequence_keeps_600_cached_plus_300_new():
    g = torch.Generator().manual_seed(1)
    bank = oib.InstanceBankOracle(torch.rand(900, 11, generator=g), torch.rand(900, 256, generator=g))
    metas = {"timestamp": torch.tensor([0.0, 0.0], dtype=torch.float64),
             "img_metas": [{"T_global": np.eye(4), "T_global_inv": np.eye(4)}] * 2}
    inst, anc, cf, ca, ti = bank.get(2, metas)
    assert cf is None and ti.tolist() == [0.5, 0.5]
    conf = torch.rand(2, 900, 10, generator=g)
    bank.cache(inst, anc, conf, metas)
    assert bank.cached_feature.shape == (2, 600, 256) and bank.confidence.shape == (2, 600)
    metas2 = {"timestamp": torch.tensor([0.5, 3.0], dtype=torch.float64), "img_metas": metas["img_metas"]}
    inst, anc, cf, ca, ti = bank.get(2, metas2)
    assert bank.mask.tolist() == [True, False] and ti.tolist() == [0.5, 0.5]
    f2, a2 = bank.update(inst, anc, conf)
    assert torch.equal(f2[0, :600], cf[0]) and torch.equal(f2[1], inst[1])
