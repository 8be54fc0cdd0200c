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


def test_flat_gradient_bound_is_below_fp32_resolution_for_the_oracle():
    """Draw 0 of the D-PACE random sweep (tests/test_random_gpu.py, seed 1000:
    sigma 5, lse ~ 20): the reference's fp32 oracle itself is more than 1e-6
    from the float64 gradient, and within 1e-6 + ulp_fp32(lse_row) * |g| -- the
    bound the sweep applies to the kernel."""
    rng = np.random.default_rng(1000)
    V = int(np.exp(rng.uniform(0, np.log(70000))))
    B = int(rng.integers(1, 33))
    N = int(rng.integers(1, 7))
    while N * B * V > 2_000_000 and N > 1:
        N -= 1
    sigma = float(rng.choice([0.5, 2.0, 5.0]))
    x = torch.from_numpy(rng.normal(0, sigma, (N, B, V)).astype(np.float32))
    t = torch.from_numpy(rng.integers(0, V, (N, B)))
    mode = int(rng.integers(0, 3))
    m = None if mode == 0 else torch.from_numpy((rng.random((N, B)) < rng.uniform(0.3, 1.0)).astype(np.float32))
    alpha = float(rng.uniform(0, 1))
    lt = odp.LOSS_TYPES[int(rng.integers(0, 3))]
    assert sigma == 5.0
    _, g_ref = odp.dpace_fwd_bwd_torch(x, t, alpha, m, lt)
    _, g64, lse64, _ = odp.dpace_f64(x.numpy(), t.numpy(), alpha, None if m is None else m.numpy(), lt)
    err = np.abs(g_ref.numpy().astype(np.float64) - g64)
    tol = 1e-6 + np.spacing(np.abs(lse64).astype(np.float32)).astype(np.float64)[..., None] * np.abs(g64)
    assert float(err.max()) > 1e-6
    assert bool((err <= tol).all())
