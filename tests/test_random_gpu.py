"""Randomized parity sweep (fixed seeds, reproducible): shapes, masks, loss
types and knobs drawn at random for both losses and both logit dtypes,
every result checked against the oracle -- loss 1e-5 relative; gradient,
elementwise, 1e-6 absolute plus 4e-6 relative. The relative part is fp32's
resolution of the log-sum-exp: logits drawn with sigma 5 give lse ~ 20,
whose float ulp is ~2e-6, and p = e^(x - lse) inherits that relative error
in any fp32 implementation (the oracle's as much as the kernel's); these
draws also reach |dL/dx| ~ 5 through D-PACE continuation-value weights S/P.
(The fixed-shape parity tests keep the plain 1e-6 absolute bound.) For bf16
the oracle runs on the widened logits and the bf16 gradient may also differ
by half a bf16 ulp."""
import numpy as np
import pytest
import torch

from oracle import dflash as odf
from oracle import dpace as odp

pytestmark = pytest.mark.gpu

LOSS_TYPES = ["dpace", "dpace-cumulative-confidence-only", "dpace-continuation-value-only"]


def _shape(rng, bmax):
    V = int(np.exp(rng.uniform(0, np.log(70000))))
    B = int(rng.integers(1, bmax + 1))
    N = int(rng.integers(1, 7))
    while N * B * V > 2_000_000 and N > 1:
        N -= 1
    return N, B, max(V, 1)


def _check(loss, grad, want, g_ref, dtype):
    assert abs(loss - float(want)) <= 1e-5 * abs(float(want)) + 1e-10, (loss, float(want))
    g = grad.float().cpu()
    tol = 1e-6 + 4e-6 * g_ref.abs()
    if dtype == torch.bfloat16:
        tol = tol + 2.0 ** -8 * g_ref.abs()
    assert bool(((g - g_ref).abs() <= tol).all()), float(((g - g_ref).abs() - tol).max())


@pytest.mark.parametrize("seed", range(24))
def test_random_dpace(cuda, seed):
    from losses import dpace_loss

    rng = np.random.default_rng(1000 + seed)
    N, B, V = _shape(rng, 32)
    dtype = torch.bfloat16 if seed % 3 == 2 else torch.float32
    sigma = float(rng.choice([0.5, 2.0, 5.0]))
    x = torch.from_numpy(rng.normal(0, sigma, (N, B, V)).astype(np.float32)).cuda().to(dtype)
    t = torch.from_numpy(rng.integers(0, V, (N, B))).cuda()
    mode = int(rng.integers(0, 3))
    m = None if mode == 0 else torch.from_numpy((rng.random((N, B)) < rng.uniform(0.3, 1.0)).astype(np.float32)).cuda()
    if mode == 2:
        m = m.bool()
    alpha = float(rng.uniform(0, 1))
    lt = LOSS_TYPES[int(rng.integers(0, 3))]
    xg = x.clone().requires_grad_(True)
    loss = dpace_loss(xg, t, alpha, m, lt)
    loss.backward()
    want, g_ref = odp.dpace_fwd_bwd_torch(x.float().cpu(), t.cpu(), alpha, None if m is None else m.cpu(), lt)
    _check(float(loss.detach()), xg.grad, want, g_ref, dtype)


@pytest.mark.parametrize("seed", range(24))
def test_random_dflash(cuda, seed):
    from models.dflash import dflash_loss

    rng = np.random.default_rng(2000 + seed)
    N, B, V = _shape(rng, 48)
    dtype = torch.bfloat16 if seed % 3 == 2 else torch.float32
    sigma = float(rng.choice([0.5, 2.0, 5.0]))
    x = torch.from_numpy(rng.normal(0, sigma, (N, B, V)).astype(np.float32)).cuda()
    y = (x + torch.randn_like(x) * float(rng.uniform(0.5, 2.0))).to(dtype)
    x = x.to(dtype)
    mask = None if rng.random() < 0.4 else torch.from_numpy(rng.uniform(0, 1, (N, B)).astype(np.float32)).cuda()
    kind = "kl" if rng.random() < 0.6 else "ce"
    block_size = None if rng.random() < 0.5 else int(rng.integers(1, B + 1))
    gamma = float(rng.choice([0.5, 4.0, 30.0]))
    sfa = bool(rng.random() < 0.3)
    xg = x.clone().requires_grad_(True)
    loss = dflash_loss(xg, y, mask, gamma, sfa, kind, block_size)
    loss.backward()
    want, g_ref = odf.dflash_fwd_bwd_torch(x.float().cpu(), y.float().cpu(), None if mask is None else mask.cpu(),
                                           gamma, sfa, kind, block_size)
    _check(float(loss.detach()), xg.grad, want, g_ref, dtype)
