"""DFlash objective on the GPU through the reference-facing API
(models.dflash.loss -> C ABI -> sm_100a kernels), checked against golden
vectors of the reference's embedded speculators oracle and the CPU oracle.

Tolerances: loss 1e-5 relative, gradient 1e-6 absolute."""
import os

import numpy as np
import pytest
import torch

import cases
from oracle import dflash as odf

pytestmark = pytest.mark.gpu

LOSS_RTOL = 1e-5
GRAD_ATOL = 1e-6
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.fixture(scope="module")
def gf():
    return np.load(os.path.join(GOLDEN, "dflash_golden.npz"))


def _close_loss(got, want):
    assert abs(got - want) <= LOSS_RTOL * abs(want) + 1e-12, (got, want)


def _run(x, y, m, gamma=4.0, sfa=False, kind="kl", block_size=None):
    from models.dflash import dflash_loss

    xt = torch.from_numpy(x).cuda().requires_grad_(True)
    yt = torch.from_numpy(y).cuda()
    mt = None if m is None else torch.from_numpy(m).cuda()
    loss = dflash_loss(xt, yt, mt, gamma, sfa, kind, block_size)
    loss.backward()
    return float(loss.detach()), xt.grad.cpu().numpy()


@pytest.mark.parametrize("case", cases.DFLASH_CASES, ids=lambda c: c["name"])
def test_dflash_matches_reference_golden(cuda, gf, case):
    x, y, m = cases.dflash_inputs(case)
    key = case["name"]
    assert cases.digest(x, y, m) == str(gf[f"{key}/sha256"])
    loss, grad = _run(x, y, m, case["gamma"], case["sfa"], case["kind"], case["block_size"])
    _close_loss(loss, float(gf[f"{key}/loss"]))
    if f"{key}/grad" in gf.files:
        np.testing.assert_allclose(grad, gf[f"{key}/grad"], rtol=0, atol=GRAD_ATOL)
    else:
        idx = gf[f"{key}/probe_idx"]
        np.testing.assert_allclose(grad.reshape(-1)[idx], gf[f"{key}/probe_val"], rtol=0,
                                   atol=GRAD_ATOL)
    _, g_or = odf.dflash_fwd_bwd_torch(torch.from_numpy(x), torch.from_numpy(y),
                                       None if m is None else torch.from_numpy(m), case["gamma"],
                                       case["sfa"], case["kind"], case["block_size"])
    np.testing.assert_allclose(grad, g_or.numpy(), rtol=0, atol=GRAD_ATOL)


def _pair(N, B, V, seed):
    rng = np.random.default_rng(seed)
    return (rng.normal(size=(N, B, V)).astype(np.float32), rng.normal(size=(N, B, V)).astype(np.float32))


def test_all_masked_is_zero(cuda):
    from models.dflash import fused_dflash_loss

    x, y = _pair(4, 8, 512, 0)
    z = torch.zeros(4, 8, device="cuda")
    assert float(fused_dflash_loss(torch.from_numpy(x).cuda(), torch.from_numpy(y).cuda(), z)) == 0.0


def test_slot_zero_decay(cuda):
    from models.dflash.loss import _forward

    x, y = _pair(4, 8, 512, 1)
    xt, yt = torch.from_numpy(x).cuda(), torch.from_numpy(y).cuda()
    _, rows, _, _ = _forward(xt, yt, None, 4.0, False, "kl", None)
    _, rows_s, _, _ = _forward(xt, yt, None, 4.0, True, "kl", None)
    assert float(rows[:, 0].abs().max()) == 0.0
    assert float(rows_s[:, 0].abs().max()) > 0.0
    assert float(rows[:, 1:].abs().min()) > 0.0


def test_masked_and_anchor_rows_zero_grad(cuda):
    from models.dflash import dflash_loss

    x, y = _pair(2, 8, 256, 2)
    m = torch.ones(2, 8, device="cuda")
    m[:, 3] = 0.0
    m[:, 0] = 0.0
    xt = torch.from_numpy(x).cuda().requires_grad_(True)
    yt = torch.from_numpy(y).cuda().requires_grad_(True)
    dflash_loss(xt, yt, m).backward()
    assert float(xt.grad[:, 3].abs().max()) == 0.0
    assert float(xt.grad[:, 0].abs().max()) == 0.0
    assert float(xt.grad[:, 2].abs().max()) > 0.0
    assert yt.grad is None  # verifier logits get no gradient


@pytest.mark.parametrize("kind", ["kl", "ce"])
def test_finite_difference(cuda, kind):
    from models.dflash import dflash_loss

    rng = np.random.default_rng(3)
    N, B, V = 2, 4, 64
    lo = rng.normal(size=(N, B, V)).astype(np.float32)
    yt = torch.from_numpy(rng.normal(size=(N, B, V)).astype(np.float32)).cuda()
    m = torch.from_numpy((rng.random((N, B)) < 0.8).astype(np.float32)).cuda()
    x = torch.from_numpy(lo).cuda().requires_grad_(True)
    dflash_loss(x, yt, m, 4.0, False, kind).backward()
    eps, worst = 1e-3, 0.0
    for _ in range(10):
        n, b, v = rng.integers(0, N), rng.integers(0, B), rng.integers(0, V)
        lp = torch.from_numpy(lo.copy()).cuda()
        lp[n, b, v] += eps
        lm = torch.from_numpy(lo.copy()).cuda()
        lm[n, b, v] -= eps
        fd = (float(dflash_loss(lp, yt, m, 4.0, False, kind)) -
              float(dflash_loss(lm, yt, m, 4.0, False, kind))) / (2 * eps)
        worst = max(worst, abs(fd - float(x.grad[n, b, v])))
    assert worst < 3e-3


def test_bitwise_repeatable_and_errors(cuda):
    from models.dflash import dflash_loss, fused_dflash_loss

    x, y = _pair(16, 8, 8192, 4)
    xt, yt = torch.from_numpy(x).cuda(), torch.from_numpy(y).cuda()
    a = fused_dflash_loss(xt, yt)
    for _ in range(10):
        assert torch.equal(fused_dflash_loss(xt, yt), a)
    with pytest.raises(ValueError):
        fused_dflash_loss(xt, yt, gamma=0.0)
    with pytest.raises(ValueError):
        fused_dflash_loss(xt, yt, kind="tv")
    with pytest.raises(AssertionError):
        fused_dflash_loss(xt, yt, block_size=9)
    with pytest.raises(AssertionError):
        fused_dflash_loss(xt, torch.zeros(16, 8, 4, device="cuda"))
    with torch.no_grad():
        assert bool(torch.isfinite(dflash_loss(xt[:2], yt[:2])))


def test_batch_independence(cuda):
    from models.dflash import fused_dflash_loss
    from models.dflash.loss import _forward

    x, y = _pair(16, 8, 8192, 5)
    xt, yt = torch.from_numpy(x).cuda(), torch.from_numpy(y).cuda()
    one = float(fused_dflash_loss(xt[:1], yt[:1]))
    _, rows, _, _ = _forward(xt, yt, None, 4.0, False, "kl", None)
    assert abs(float(rows[0].sum()) - one) <= 1e-6 * max(1.0, abs(one))


@pytest.mark.parametrize("V", [5, 1001, 4099])
def test_ragged_and_misaligned(cuda, V):
    """Draft and verifier rows with different 16-byte phase (scalar path), and
    rows not on 16-byte boundaries."""
    from models.dflash import dflash_loss

    rng = np.random.default_rng(V)
    N, B = 3, 8
    bx = torch.from_numpy(rng.normal(size=N * B * V + 1).astype(np.float32)).cuda()
    y = torch.from_numpy(rng.normal(size=(N, B, V)).astype(np.float32)).cuda()
    for kind in ("kl", "ce"):
        leaf = bx.detach().clone().requires_grad_(True)
        loss = dflash_loss(leaf[1:].view(N, B, V), y, None, 4.0, False, kind, 3)
        loss.backward()
        want, g = odf.dflash_fwd_bwd_torch(bx[1:].view(N, B, V).cpu(), y.cpu(), None, 4.0, False,
                                           kind, 3)
        _close_loss(float(loss.detach()), float(want))
        np.testing.assert_allclose(leaf.grad[1:].view(N, B, V).cpu().numpy(), g.numpy(), rtol=0,
                                   atol=GRAD_ATOL)


@pytest.mark.parametrize("kind", ["kl", "ce"])
def test_full_size_correlated_verifier(cuda, kind):
    """[64, 16, 128256]: draft ~ N(0, 2^2), verifier = draft + N(0, 1), gamma 4,
    anchor slot unscored, all slots masked in: whole loss and gradient against
    the CPU oracle."""
    from models.dflash import dflash_loss

    g = torch.Generator(device="cuda").manual_seed(7)
    x = torch.randn(64, 16, 128256, device="cuda", generator=g) * 2.0
    y = x + torch.randn(64, 16, 128256, device="cuda", generator=g)
    xg = x.clone().requires_grad_(True)
    loss = dflash_loss(xg, y, None, 4.0, False, kind)
    loss.backward()
    want, gr = odf.dflash_fwd_bwd_torch(x.cpu(), y.cpu(), None, 4.0, False, kind)
    _close_loss(float(loss.detach()), float(want))
    diff = (xg.grad.cpu() - gr).abs().max().item()
    assert diff <= GRAD_ATOL, diff


SHAPE_CASES = [c for c in cases.DFLASH_CASES if c["name"] in (
    "kl_bern.5_N8_B8_V1024", "ce_bern.5_N8_B8_V1024", "kl_V7_N6_B8", "kl_V1000_N6_B8",
    "kl_sfa_N4_B8_V1024", "ce_bs4_N4_B16_V1024", "kl_bs3_N3_B8_V256_ragged", "ce_ties_N4_B8_V64",
    "ws3_kl_N4_B16_V128256_sd2_corr", "ws3_ce_N2_B16_V128256_sd2_corr")]


@pytest.mark.parametrize("shape", [0, 1, 2, 3, 4, 5, 6, 10, 11, 12, 13, 14])
def test_every_launch_shape_matches_golden(cuda, gf, shape):
    """Shapes 0-6: warp-specialized bulk-copy ring variants; 10-14: 128-bit-load kernels."""
    from specdec import _lib

    try:
        _lib.set_launch_shape(_lib.KERNEL_DFLASH_FWD, shape)
        _lib.set_launch_shape(_lib.KERNEL_DFLASH_BWD, shape)
        for case in SHAPE_CASES:
            x, y, m = cases.dflash_inputs(case)
            key = case["name"]
            loss, grad = _run(x, y, m, case["gamma"], case["sfa"], case["kind"], case["block_size"])
            _close_loss(loss, float(gf[f"{key}/loss"]))
            if f"{key}/grad" in gf.files:
                np.testing.assert_allclose(grad, gf[f"{key}/grad"], rtol=0, atol=GRAD_ATOL)
            else:
                idx = gf[f"{key}/probe_idx"]
                np.testing.assert_allclose(grad.reshape(-1)[idx], gf[f"{key}/probe_val"], rtol=0,
                                           atol=GRAD_ATOL)
    finally:
        _lib.set_launch_shape(_lib.KERNEL_DFLASH_FWD, _lib.SHAPE_DEFAULT)
        _lib.set_launch_shape(_lib.KERNEL_DFLASH_BWD, _lib.SHAPE_DEFAULT)


def test_static_interleave_and_schedule_independence(cuda):
    """Ring kernels with the static block interleave give the same bits as the
    dynamic queue (partials are slotted by block index)."""
    from specdec import _lib, ops

    g = torch.Generator(device="cuda").manual_seed(9)
    x = torch.randn(16, 16, 128256, device="cuda", generator=g) * 2.0
    y = x + torch.randn(16, 16, 128256, device="cuda", generator=g)
    for kind in (0, 1):
        ref = None
        for dynamic in (True, False, True):
            _lib.set_block_queue(dynamic)
            loss, rows, scale, lzq, lzp, tgt = ops.dflash_forward(x, y, None, 4.0, False, kind, 16)
            gr = ops.dflash_backward(x, y if kind == 0 else None, scale, lzq, lzp, tgt, None, kind)
            if ref is None:
                ref = (loss.clone(), rows.clone(), gr.clone())
            else:
                assert torch.equal(loss, ref[0]) and torch.equal(rows, ref[1]) and torch.equal(gr, ref[2])
    _lib.set_block_queue(True)


def test_more_than_32_positions(cuda):
    """B > 32 positions per sequence (allowed by the reference): the ring
    finalize loops over rows; results match the oracle."""
    from models.dflash import dflash_loss

    rng = np.random.default_rng(40)
    N, B, V = 2, 40, 3000
    x = rng.normal(size=(N, B, V)).astype(np.float32)
    y = rng.normal(size=(N, B, V)).astype(np.float32)
    xt = torch.from_numpy(x).cuda().requires_grad_(True)
    loss = dflash_loss(xt, torch.from_numpy(y).cuda(), None, 4.0, False, "kl", 8)
    loss.backward()
    want, g = odf.dflash_fwd_bwd_torch(torch.from_numpy(x), torch.from_numpy(y), None, 4.0, False, "kl", 8)
    _close_loss(float(loss.detach()), float(want))
    np.testing.assert_allclose(xt.grad.cpu().numpy(), g.numpy(), rtol=0, atol=GRAD_ATOL)
