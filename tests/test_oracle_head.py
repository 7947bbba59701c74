"""The head oracle (oracle/head_torch.py, a restatement of the reference's single-frame decoder
head twin) against the fixture written by running the reference twin itself
(tests/golden/make_golden.py head_twin_s42): the same parameters bit for bit under seed 42, the
same inputs, and the same predictions, classifications and qualities."""
import numpy as np
import pytest
import torch

import fixtures as fx
from oracle import head_torch as oh


@pytest.fixture(scope="module")
def case():
    g = fx.load("head_twin_s42")
    head = oh.build_head(int(g["seed"]))
    maps, proj, wh = oh.head_inputs(int(g["bs"]))
    return g, head, maps, proj, wh


def test_head_parameters_and_inputs_match_the_reference(case):
    g, head, maps, proj, wh = case
    sd = head.state_dict()
    assert list(sd.keys()) == [str(k) for k in g["param_names"]]
    for (k, v), ck in zip(sd.items(), g["param_ck"]):
        assert np.allclose(fx.checksum(v), ck, rtol=1e-12, atol=0), k
    for i, m in enumerate(maps):
        assert np.allclose(fx.checksum(m), g[f"ck_map{i}"], rtol=1e-12, atol=0)
    assert np.allclose(fx.checksum(proj), g["ck_projection_mat"], rtol=1e-12, atol=0)
    assert list(head.operation_order) == [str(o) for o in g["operation_order"]]


def test_head_outputs_match_the_reference(case):
    g, head, maps, proj, wh = case
    out = head(maps, proj, wh, bs=int(g["bs"]))
    for i, pr in enumerate(out["prediction"]):
        np.testing.assert_allclose(pr.numpy(), g[f"prediction{i}"], rtol=1e-4, atol=1e-4)
    for i, c in enumerate(out["classification"]):
        assert (c is None) == (f"classification{i}" not in g)
        if c is not None:
            np.testing.assert_allclose(c.numpy(), g[f"classification{i}"], rtol=1e-4, atol=1e-4)
            np.testing.assert_allclose(out["quality"][i].numpy(), g[f"quality{i}"], rtol=1e-4, atol=1e-4)
