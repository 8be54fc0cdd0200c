"""bfloat16 logits through the reference-facing API (losses.dpace, models.dflash
-> *_bf16 C entry points -> bf16 ring kernels).

The reference takes fp32 only, so the oracle for a bf16 input is the
reference's fp32 oracle applied to the exactly widened values. The kernels
compute in fp32 from those same values, so:
  - loss: within 1e-5 relative of the oracle (as for fp32 inputs);
  - gradient (bf16, rounded to nearest even from fp32): within half a bf16
    ulp of the oracle's fp32 gradient plus the fp32 tolerance,
        |g - g_ref| <= 2^-8 |g_ref| + 2e-6,
    and equal to bf16(g_ref) for all but a handful of elements (those whose
    fp32 value sits within the fp32 error of a rounding boundary).
"""
import numpy as np
import pytest
import torch

import cases
from oracle import dflash as odf
from oracle import dpace as odp

pytestmark = pytest.mark.gpu

LOSS_RTOL = 1e-5
BF16_RTOL = 2.0 ** -8
GRAD_ATOL = 2e-6
MIN_EXACT = 0.995  # fraction of gradient elements equal to bf16(oracle)


def _bf16(a: np.ndarray, dev="cuda") -> torch.Tensor:
    return torch.from_numpy(a).to(dev).to(torch.bfloat16)


def _close_loss(got, want):
    assert abs(got - want) <= LOSS_RTOL * abs(want) + 1e-12, (got, want)


def _check_grad(g: torch.Tensor, g_ref: torch.Tensor):
    assert g.dtype == torch.bfloat16
    gf = g.float().cpu()
    g_ref = g_ref.float().cpu()
    err = (gf - g_ref).abs()
    bound = BF16_RTOL * g_ref.abs() + GRAD_ATOL
    assert bool((err <= bound).all()), float((err - bound).max())
    if g_ref.numel():
        exact = float((g.cpu() == g_ref.to(torch.bfloat16)).float().mean())
        assert exact >= MIN_EXACT, exact


def _dpace(x16, t, m, alpha=0.5, loss_type="dpace"):
    from losses import dpace_loss

    xg = x16.clone().requires_grad_(True)
    loss = dpace_loss(xg, t, alpha, m, loss_type)
    loss.backward()
    return float(loss.detach()), xg.grad


@pytest.mark.parametrize("case", cases.DPACE_CASES, ids=lambda c: c["name"])
def test_dpace_bf16_matches_oracle_on_widened_logits(cuda, case):
    x, t, m = cases.dpace_inputs(case)
    x16 = _bf16(x)
    tt = torch.from_numpy(t).cuda()
    mt = None if m is None else torch.from_numpy(m).cuda()
    loss, g = _dpace(x16, tt, mt, case["alpha"], case["loss_type"])
    want, g_ref = odp.dpace_fwd_bwd_torch(x16.float().cpu(), tt.cpu(), case["alpha"],
                                          None if mt is None else mt.cpu(), case["loss_type"])
    _close_loss(loss, float(want))
    _check_grad(g, g_ref)


def _dflash(x16, y16, m, gamma=4.0, sfa=False, kind="kl", block_size=None):
    from models.dflash import dflash_loss

    xg = x16.clone().requires_grad_(True)
    loss = dflash_loss(xg, y16, m, gamma, sfa, kind, block_size)
    loss.backward()
    return float(loss.detach()), xg.grad


@pytest.mark.parametrize("case", cases.DFLASH_CASES, ids=lambda c: c["name"])
def test_dflash_bf16_matches_oracle_on_widened_logits(cuda, case):
    x, y, m = cases.dflash_inputs(case)
    x16, y16 = _bf16(x), _bf16(y)
    mt = None if m is None else torch.from_numpy(m).cuda()
    loss, g = _dflash(x16, y16, mt, case["gamma"], case["sfa"], case["kind"], case["block_size"])
    want, g_ref = odf.dflash_fwd_bwd_torch(x16.float().cpu(), y16.float().cpu(),
                                           None if mt is None else mt.cpu(), case["gamma"],
                                           case["sfa"], case["kind"], case["block_size"])
    _close_loss(loss, float(want))
    _check_grad(g, g_ref)


def test_dpace_bf16_full_size_llama3_vocab(cuda):
    """[64, 16, 128256] bf16, logits ~ N(0, 2^2), prefix mask k ~ U{0..4}."""
    g = torch.Generator(device="cuda").manual_seed(7)
    N, B, V = 64, 16, 128256
    x16 = (torch.randn(N, B, V, device="cuda", generator=g) * 2.0).to(torch.bfloat16)
    t = torch.randint(0, V, (N, B), device="cuda", generator=g)
    k = torch.randint(0, 5, (N, 1), device="cuda", generator=g)
    m = (torch.arange(B, device="cuda").view(1, B) >= k).float()
    loss, grad = _dpace(x16, t, m)
    want, g_ref = odp.dpace_fwd_bwd_torch(x16.float().cpu(), t.cpu(), 0.5, m.cpu(), "dpace")
    _close_loss(loss, float(want))
    _check_grad(grad, g_ref)


@pytest.mark.parametrize("kind", ["kl", "ce"])
def test_dflash_bf16_full_size_llama3_vocab(cuda, kind):
    """[32, 16, 128256] bf16, draft ~ N(0, 2^2), verifier = draft + N(0, 1)."""
    g = torch.Generator(device="cuda").manual_seed(11)
    N, B, V = 32, 16, 128256
    x = torch.randn(N, B, V, device="cuda", generator=g) * 2.0
    y = x + torch.randn(N, B, V, device="cuda", generator=g)
    x16, y16 = x.to(torch.bfloat16), y.to(torch.bfloat16)
    del x, y
    loss, grad = _dflash(x16, y16, None, kind=kind)
    want, g_ref = odf.dflash_fwd_bwd_torch(x16.float().cpu(), y16.float().cpu(), None, 4.0, False, kind)
    _close_loss(loss, float(want))
    _check_grad(grad, g_ref)


def test_bf16_misaligned_view_is_copied_and_correct(cuda):
    from losses import fused_dpace_loss

    rng = np.random.default_rng(3)
    N, B, V = 3, 4, 1001
    base = _bf16(rng.normal(size=(N * B * V + 3,)).astype(np.float32))
    x16 = base[3:].view(N, B, V)  # 6 bytes past a 16-byte boundary
    assert x16.data_ptr() % 16 != 0 and x16.is_contiguous()
    t = torch.from_numpy(rng.integers(0, V, (N, B))).cuda()
    loss = float(fused_dpace_loss(x16, t))
    want, _ = odp.dpace_fwd_bwd_torch(x16.float().cpu(), t.cpu())
    _close_loss(loss, float(want))
    loss2, g = _dpace(x16, t, None)
    _close_loss(loss2, float(want))
    _, g_ref = odp.dpace_fwd_bwd_torch(x16.float().cpu(), t.cpu())
    _check_grad(g, g_ref)


def test_bf16_abi_rejects_misaligned_pointers(cuda):
    from specdec import _lib

    lib = _lib.load()
    N, B, V = 1, 2, 64
    x = torch.zeros(N * B * V + 8, dtype=torch.bfloat16, device="cuda")
    t = torch.zeros(N, B, dtype=torch.int64, device="cuda")
    out = [torch.empty(N, B, device="cuda") for _ in range(2)]
    loss = torch.empty((), device="cuda")
    scratch = torch.empty(1 << 16, dtype=torch.uint8, device="cuda")
    counters = torch.zeros(1 << 12, dtype=torch.uint8, device="cuda")
    code = lib.specdec_dpace_forward_bf16(
        x.data_ptr() + 8, t.data_ptr(), None, N, B, V, 0.5, 0, N, loss.data_ptr(), None,
        out[0].data_ptr(), out[1].data_ptr(), None, scratch.data_ptr(), scratch.numel(),
        counters.data_ptr(), counters.numel(), None)
    assert code == _lib.ERR_ARGUMENT
    assert b"16-byte" in lib.specdec_last_error()
    g = torch.empty_like(x)
    code = lib.specdec_dpace_backward_bf16(
        x.data_ptr(), t.data_ptr(), out[0].data_ptr(), out[1].data_ptr(), None, g.data_ptr() + 8,
        N, B, V, None, None, 0, None)
    assert code == _lib.ERR_ARGUMENT


def test_dflash_mixed_dtypes_widen_the_bf16_side(cuda):
    from models.dflash import dflash_loss

    rng = np.random.default_rng(5)
    x = torch.from_numpy(rng.normal(size=(4, 8, 3000)).astype(np.float32)).cuda()
    y16 = _bf16(rng.normal(size=(4, 8, 3000)).astype(np.float32))
    xg = x.clone().requires_grad_(True)
    loss = dflash_loss(xg, y16)
    loss.backward()
    want, g_ref = odf.dflash_fwd_bwd_torch(x.cpu(), y16.float().cpu())
    _close_loss(float(loss.detach()), float(want))
    assert xg.grad.dtype == torch.float32
    assert float((xg.grad.cpu() - g_ref).abs().max()) <= 1e-6


@pytest.mark.parametrize("shape", [0, 1, 2, 3, 4, 5, 6, 7, 8, 10])
def test_bf16_every_launch_shape(cuda, shape):
    """Every bf16 ring shape (10 selects the fp32 128-bit-load kernels, for
    which bf16 uses ring shape 0; 7 and 8 exist for the D-PACE kernels only,
    the DFlash ones keep their default) gives the oracle's results."""
    from specdec import _lib

    kernels = (0, 1) if shape in (7, 8) else range(4)

    rng = np.random.default_rng(9)
    N, B, V = 6, 8, 20011
    x16 = _bf16(rng.normal(scale=2.0, size=(N, B, V)).astype(np.float32))
    y16 = _bf16(rng.normal(scale=2.0, size=(N, B, V)).astype(np.float32))
    t = torch.from_numpy(rng.integers(0, V, (N, B))).cuda()
    m = torch.from_numpy((rng.random((N, B)) < 0.8).astype(np.float32)).cuda()
    try:
        for k in kernels:
            _lib.set_launch_shape(k, shape, 0)
        loss, g = _dpace(x16, t, m)
        want, g_ref = odp.dpace_fwd_bwd_torch(x16.float().cpu(), t.cpu(), 0.5, m.cpu())
        _close_loss(loss, float(want))
        _check_grad(g, g_ref)
        for kind in ("kl", "ce"):
            loss, g = _dflash(x16, y16, m, kind=kind)
            want, g_ref = odf.dflash_fwd_bwd_torch(x16.float().cpu(), y16.float().cpu(), m.cpu(), kind=kind)
            _close_loss(loss, float(want))
            _check_grad(g, g_ref)
    finally:
        for k in range(4):
            _lib.set_launch_shape(k, _lib.SHAPE_DEFAULT, 0)


def test_bf16_ring_results_are_schedule_independent(cuda):
    """Dynamic block queue and static interleave give bitwise equal results."""
    from specdec import _lib

    rng = np.random.default_rng(12)
    N, B, V = 16, 16, 50000
    x16 = _bf16(rng.normal(scale=2.0, size=(N, B, V)).astype(np.float32))
    y16 = _bf16(rng.normal(scale=2.0, size=(N, B, V)).astype(np.float32))
    t = torch.from_numpy(rng.integers(0, V, (N, B))).cuda()
    res = []
    try:
        for dynamic in (1, 0):
            _lib.set_block_queue(dynamic)
            a = _dpace(x16, t, None)
            b = _dflash(x16, y16, None)
            res.append((a, b))
    finally:
        _lib.set_block_queue(1)
    (a1, b1), (a2, b2) = res
    assert a1[0] == a2[0] and torch.equal(a1[1], a2[1])
    assert b1[0] == b2[0] and torch.equal(b1[1], b2[1])


def test_bf16_masked_rows_exact_zero_and_all_masked(cuda):
    from losses import dpace_loss
    from models.dflash import dflash_loss

    rng = np.random.default_rng(13)
    x16 = _bf16(rng.normal(size=(3, 8, 777)).astype(np.float32))
    t = torch.from_numpy(rng.integers(0, 777, (3, 8))).cuda()
    m = torch.ones(3, 8, device="cuda")
    m[:, :3] = 0
    xg = x16.clone().requires_grad_(True)
    dpace_loss(xg, t, 0.5, m).backward()
    assert float(xg.grad[:, :3].float().abs().max()) == 0.0
    assert float(xg.grad[:, 3:].float().abs().max()) > 0.0
    z = torch.zeros(3, 8, device="cuda")
    xg = x16.clone().requires_grad_(True)
    loss = dflash_loss(xg, x16, z)
    loss.backward()
    assert float(loss) == 0.0 and float(xg.grad.float().abs().max()) == 0.0


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("B,block_size", [(40, 16), (64, 16), (48, 5)])
def test_dflash_more_than_32_positions(cuda, dtype, B, block_size):
    """B > 32 positions per sequence (anchors x block): the ring finalize
    loops over rows; results as the oracle's."""
    rng = np.random.default_rng(B)
    N, V = 3, 5000
    x = torch.from_numpy(rng.normal(scale=2.0, size=(N, B, V)).astype(np.float32)).cuda().to(dtype)
    y = torch.from_numpy(rng.normal(scale=2.0, size=(N, B, V)).astype(np.float32)).cuda().to(dtype)
    m = torch.from_numpy((rng.random((N, B)) < 0.7).astype(np.float32)).cuda()
    for kind in ("kl", "ce"):
        loss, g = _dflash(x, y, m, kind=kind, block_size=block_size)
        want, g_ref = odf.dflash_fwd_bwd_torch(x.float().cpu(), y.float().cpu(), m.cpu(), 4.0, False, kind,
                                               block_size)
        _close_loss(loss, float(want))
        if dtype == torch.bfloat16:
            _check_grad(g, g_ref)
        else:
            assert float((g.cpu() - g_ref).abs().max()) <= 1e-6
