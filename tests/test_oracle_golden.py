"""The CPU oracle is pinned against golden vectors made by the reference's own
oracles (tests/golden/make_golden.py). No GPU needed."""
import os

import numpy as np
import pytest
import torch

import cases
from oracle import dflash as odf
from oracle import dpace as odp

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _load(name):
    return np.load(os.path.join(GOLDEN, name))


@pytest.fixture(scope="module")
def gd():
    return _load("dpace_golden.npz")


@pytest.fixture(scope="module")
def gf():
    return _load("dflash_golden.npz")


def _grad_check(g, key, case, grad, atol):
    if f"{key}/grad" in g.files:
        np.testing.assert_allclose(grad, g[f"{key}/grad"], rtol=0, atol=atol)
    else:
        idx = g[f"{key}/probe_idx"]
        np.testing.assert_allclose(grad.reshape(-1)[idx], g[f"{key}/probe_val"], rtol=0, atol=atol)
    assert abs(np.abs(grad.astype(np.float64)).sum() - float(g[f"{key}/grad_abs_sum"])) <= \
        1e-5 * float(g[f"{key}/grad_abs_sum"]) + 1e-9


@pytest.mark.parametrize("case", cases.DPACE_CASES, ids=lambda c: c["name"])
def test_dpace_oracle_matches_reference(gd, case):
    x, t, m = cases.dpace_inputs(case)
    key = case["name"]
    assert cases.digest(x, t, m) == str(gd[f"{key}/sha256"]), "input generator drifted"
    ref = float(gd[f"{key}/loss"])
    assert ref == pytest.approx(float(gd[f"{key}/loss_spec"]), rel=1e-6, abs=1e-9)
    # torch restatement: same float32 ops as the reference -> identical numbers
    loss, grad = odp.dpace_fwd_bwd_torch(torch.from_numpy(x), torch.from_numpy(t), case["alpha"],
                                         None if m is None else torch.from_numpy(m),
                                         case["loss_type"])
    assert float(loss) == ref
    _grad_check(gd, key, case, grad.numpy(), atol=0.0)
    # float64 restatement bounds the float32 rounding of the reference
    l64, g64, _, _ = odp.dpace_f64(x, t, case["alpha"], m, case["loss_type"])
    assert l64 == pytest.approx(ref, rel=2e-6, abs=1e-9)
    _grad_check(gd, key, case, g64, atol=1e-7)


@pytest.mark.parametrize("case", cases.DFLASH_CASES, ids=lambda c: c["name"])
def test_dflash_oracle_matches_reference(gf, case):
    x, y, m = cases.dflash_inputs(case)
    key = case["name"]
    assert cases.digest(x, y, m) == str(gf[f"{key}/sha256"]), "input generator drifted"
    ref = float(gf[f"{key}/loss"])
    mt = None if m is None else torch.from_numpy(m)
    loss, grad = odf.dflash_fwd_bwd_torch(torch.from_numpy(x), torch.from_numpy(y), mt,
                                          case["gamma"], case["sfa"], case["kind"],
                                          case["block_size"])
    assert float(loss) == ref
    _grad_check(gf, key, case, grad.numpy(), atol=0.0)
    l64, g64, _ = odf.dflash_f64(x, y, m, case["gamma"], case["sfa"], case["kind"],
                                 case["block_size"])
    assert l64 == pytest.approx(ref, rel=2e-5, abs=1e-8)
    _grad_check(gf, key, case, g64, atol=1e-7)


def test_oracle_value_errors():
    x = torch.zeros(1, 2, 4)
    t = torch.zeros(1, 2, dtype=torch.int64)
    with pytest.raises(ValueError):
        odp.dpace_loss_torch(x, t, 1.5)
    with pytest.raises(ValueError):
        odp.dpace_loss_torch(x, t, 0.5, None, "topk_mask")


def test_golden_edge_values(gd, gf):
    assert float(gd["allmasked_N4_B8_V512/loss"]) == 0.0
    assert float(gf["kl_allmasked_N4_B8_V512/loss"]) == 0.0
    # B=1 without sample_from_anchor: the only slot is the anchor, weight 0
    assert float(gf["kl_B1_N8_V1024/loss"]) == 0.0
