"""D-PACE on the GPU through the reference-facing API (losses.dpace -> C ABI ->
sm_100a kernels), checked against the golden vectors of the reference's own
oracle and against the CPU oracle.

Tolerances: loss 1e-5 relative, gradient 1e-6 absolute."""
import os

import numpy as np
import pytest
import torch

import cases
from oracle import dpace as odp

pytestmark = pytest.mark.gpu

LOSS_RTOL = 1e-5
GRAD_ATOL = 1e-6
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.fixture(scope="module")
def gd():
    return np.load(os.path.join(GOLDEN, "dpace_golden.npz"))


def _run(x, t, m, alpha=0.5, loss_type="dpace", dev="cuda"):
    from losses import dpace_loss

    xt = torch.from_numpy(x).to(dev).requires_grad_(True)
    tt = torch.from_numpy(t).to(dev)
    mt = None if m is None else torch.from_numpy(m).to(dev)
    loss = dpace_loss(xt, tt, alpha, mt, loss_type)
    loss.backward()
    return float(loss.detach()), xt.grad.cpu().numpy()


def _close_loss(got, want):
    assert abs(got - want) <= LOSS_RTOL * abs(want) + 1e-12, (got, want)


@pytest.mark.parametrize("case", cases.DPACE_CASES, ids=lambda c: c["name"])
def test_dpace_matches_reference_golden(cuda, gd, case):
    x, t, m = cases.dpace_inputs(case)
    key = case["name"]
    assert cases.digest(x, t, m) == str(gd[f"{key}/sha256"])
    loss, grad = _run(x, t, m, case["alpha"], case["loss_type"])
    _close_loss(loss, float(gd[f"{key}/loss"]))
    if f"{key}/grad" in gd.files:
        np.testing.assert_allclose(grad, gd[f"{key}/grad"], rtol=0, atol=GRAD_ATOL)
    else:
        idx = gd[f"{key}/probe_idx"]
        np.testing.assert_allclose(grad.reshape(-1)[idx], gd[f"{key}/probe_val"], rtol=0,
                                   atol=GRAD_ATOL)
    # whole gradient against the CPU oracle (torch float32, same ops as the reference)
    _, g_or = odp.dpace_fwd_bwd_torch(torch.from_numpy(x), torch.from_numpy(t), case["alpha"],
                                      None if m is None else torch.from_numpy(m), case["loss_type"])
    np.testing.assert_allclose(grad, g_or.numpy(), rtol=0, atol=GRAD_ATOL)


def test_all_masked_is_exactly_zero(cuda):
    from losses import dpace_loss, fused_dpace_loss

    rng = np.random.default_rng(0)
    x = torch.from_numpy(rng.normal(size=(4, 8, 512)).astype(np.float32)).cuda()
    t = torch.from_numpy(rng.integers(0, 512, (4, 8))).cuda()
    z = torch.zeros(4, 8, device="cuda")
    assert float(fused_dpace_loss(x, t, 0.5, z)) == 0.0
    xg = x.clone().requires_grad_(True)
    dpace_loss(xg, t, 0.5, z).backward()
    assert float(xg.grad.abs().max()) == 0.0


def test_masked_rows_get_exactly_zero_grad(cuda):
    from losses import dpace_loss

    rng = np.random.default_rng(1)
    x = torch.from_numpy(rng.normal(size=(2, 8, 256)).astype(np.float32)).cuda().requires_grad_(True)
    t = torch.from_numpy(rng.integers(0, 256, (2, 8))).cuda()
    m = torch.ones(2, 8, device="cuda")
    m[:, 3] = 0.0
    dpace_loss(x, t, 0.5, m).backward()
    assert float(x.grad[:, 3].abs().max()) == 0.0
    assert float(x.grad[:, 2].abs().max()) > 0.0


def test_bool_mask_and_none_mask(cuda):
    from losses import dpace_loss, fused_dpace_loss

    rng = np.random.default_rng(2)
    x = torch.from_numpy(rng.normal(size=(4, 8, 512)).astype(np.float32)).cuda()
    t = torch.from_numpy(rng.integers(0, 512, (4, 8))).cuda()
    mk = torch.ones(4, 8, device="cuda")
    mk[0] = 0.0
    a = float(dpace_loss(x, t, 0.5, mk.bool()))
    b = float(fused_dpace_loss(x, t, 0.5, mk))
    assert a == b
    assert float(fused_dpace_loss(x, t)) == float(fused_dpace_loss(x, t, 0.5, torch.ones(4, 8, device="cuda")))


def test_forward_is_bitwise_repeatable(cuda):
    from losses import fused_dpace_loss

    rng = np.random.default_rng(3)
    x = torch.from_numpy(rng.normal(size=(16, 8, 8192)).astype(np.float32)).cuda()
    t = torch.from_numpy(rng.integers(0, 8192, (16, 8))).cuda()
    a = fused_dpace_loss(x, t)
    for _ in range(10):
        assert torch.equal(fused_dpace_loss(x, t), a)


def test_out_of_range_target_raises(cuda):
    from losses import dpace_loss, fused_dpace_loss

    x = torch.randn(2, 8, 100, device="cuda")
    t = torch.randint(0, 100, (2, 8), device="cuda")
    bad = t.clone()
    bad[0, 0] = 999999
    with pytest.raises(ValueError):
        fused_dpace_loss(x, bad)
    bad[0, 0] = -1
    with pytest.raises(ValueError):
        dpace_loss(x, bad)
    # the error state does not leak into the next call
    assert torch.isfinite(fused_dpace_loss(x, t))


def test_value_errors(cuda):
    from losses import fused_dpace_loss

    x = torch.randn(1, 8, 64, device="cuda")
    t = torch.randint(0, 64, (1, 8), device="cuda")
    with pytest.raises(ValueError):
        fused_dpace_loss(x, t, 1.5)
    with pytest.raises(ValueError):
        fused_dpace_loss(x, t, 0.5, None, "topk_mask")
    with pytest.raises(AssertionError):
        fused_dpace_loss(torch.randn(1, 33, 64, device="cuda"), torch.zeros(1, 33, dtype=torch.int64, device="cuda"))


def test_works_under_no_grad(cuda):
    from losses import dpace_loss

    with torch.no_grad():
        loss = dpace_loss(torch.randn(2, 8, 300, device="cuda"), torch.randint(0, 300, (2, 8), device="cuda"))
    assert bool(torch.isfinite(loss))


def test_finite_difference(cuda):
    from losses import dpace_loss

    rng = np.random.default_rng(4)
    N, B, V = 2, 4, 64
    lo = rng.normal(size=(N, B, V)).astype(np.float32)
    t = torch.from_numpy(rng.integers(0, V, (N, B))).cuda()
    m = torch.from_numpy((rng.random((N, B)) < 0.6).astype(np.float32)).cuda()
    x = torch.from_numpy(lo).cuda().requires_grad_(True)
    dpace_loss(x, t, 0.5, m).backward()
    eps, worst = 1e-3, 0.0
    for _ in range(12):
        n, b, v = rng.integers(0, N), rng.integers(0, B), rng.integers(0, V)
        lp = torch.from_numpy(lo.copy()).cuda()
        lp[n, b, v] += eps
        lm = torch.from_numpy(lo.copy()).cuda()
        lm[n, b, v] -= eps
        fd = (float(dpace_loss(lp, t, 0.5, m)) - float(dpace_loss(lm, t, 0.5, m))) / (2 * eps)
        worst = max(worst, abs(fd - float(x.grad[n, b, v])))
    assert worst < 3e-3


@pytest.mark.parametrize("V", [1, 3, 5, 1001, 4099, 32001])
def test_ragged_and_misaligned_rows(cuda, V):
    """Rows that do not start on a 16-byte boundary (V % 4 != 0), and a base
    pointer offset by one float: head/tail handling and the scalar store path."""
    from losses import dpace_loss

    rng = np.random.default_rng(V)
    N, B = 3, 8
    buf = torch.from_numpy(rng.normal(size=N * B * V + 1).astype(np.float32)).cuda()
    x = buf[1:].view(N, B, V)
    assert x.data_ptr() % 16 != 0
    t = torch.from_numpy(rng.integers(0, V, (N, B))).cuda()
    m = torch.from_numpy((rng.random((N, B)) < 0.7).astype(np.float32)).cuda()
    leaf = buf.detach().clone().requires_grad_(True)
    loss = dpace_loss(leaf[1:].view(N, B, V), t, 0.5, m)
    loss.backward()
    want, g = odp.dpace_fwd_bwd_torch(x.cpu(), t.cpu(), 0.5, m.cpu())
    _close_loss(float(loss.detach()), float(want))
    np.testing.assert_allclose(leaf.grad[1:].view(N, B, V).cpu().numpy(), g.numpy(), rtol=0, atol=GRAD_ATOL)


def test_custom_stream(cuda):
    """Launches go to torch's current stream (the reference assumed the default one)."""
    from losses import dpace_loss

    rng = np.random.default_rng(5)
    lo = rng.normal(0, 2, size=(8, 16, 32000)).astype(np.float32)
    tg = rng.integers(0, 32000, (8, 16))
    want, g = odp.dpace_fwd_bwd_torch(torch.from_numpy(lo), torch.from_numpy(tg))
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        x = torch.from_numpy(lo).cuda().requires_grad_(True)
        t = torch.from_numpy(tg).cuda()
        loss = dpace_loss(x, t)
        loss.backward()
        got = loss.detach().clone()
        grad = x.grad.clone()
    s.synchronize()
    _close_loss(float(got), float(want))
    np.testing.assert_allclose(grad.cpu().numpy(), g.numpy(), rtol=0, atol=GRAD_ATOL)


def test_empty_batch(cuda):
    from losses import dpace_loss

    x = torch.zeros(0, 8, 16, device="cuda", requires_grad=True)
    t = torch.zeros(0, 8, dtype=torch.int64, device="cuda")
    loss = dpace_loss(x, t)
    assert torch.isnan(loss)
    loss.backward()
    assert x.grad.shape == x.shape


def _workload(N, B, V, sigma, kmax, seed, dev="cuda"):
    g = torch.Generator(device=dev).manual_seed(seed)
    x = torch.randn(N, B, V, device=dev, generator=g) * sigma
    t = torch.randint(0, V, (N, B), device=dev, generator=g)
    k = torch.randint(0, kmax + 1, (N, 1), device=dev, generator=g)
    m = (torch.arange(B, device=dev).view(1, B) >= k).float()
    return x, t, m


@pytest.mark.parametrize("loss_type", ["dpace", "dpace-cumulative-confidence-only",
                                       "dpace-continuation-value-only"])
def test_full_size_llama3_vocab(cuda, loss_type):
    """[64, 16, 128256], logits ~ N(0, 2^2), per-sequence prefix mask k ~ U{0..4},
    alpha 0.5: the whole loss and gradient against the CPU oracle."""
    from losses import dpace_loss

    x, t, m = _workload(64, 16, 128256, 2.0, 4, 0)
    xg = x.clone().requires_grad_(True)
    loss = dpace_loss(xg, t, 0.5, m, loss_type)
    loss.backward()
    want, g = odp.dpace_fwd_bwd_torch(x.cpu(), t.cpu(), 0.5, m.cpu(), loss_type)
    _close_loss(float(loss.detach()), float(want))
    diff = (xg.grad.cpu() - g).abs().max().item()
    assert diff <= GRAD_ATOL, diff


def test_large_batch_shard_every_sequence_against_the_oracle(cuda):
    """[64, 32, 151936] (one of eight shards of the 512-sequence workload),
    logits ~ N(0, 3^2), prefix mask k ~ U{0..8}, alpha 0.5: the shard's loss
    (divisor 64) and its WHOLE gradient against the CPU oracle, which runs on
    8 sequences at a time (its loss and gradient for a chunk, scaled by
    8/64 -- a power of two, so the scaling is exact). Loss 1e-5 relative,
    every gradient element 1e-6 absolute. Also: the one-call forward+backward
    (backward chained to the finalize) equals the separate calls bit for bit,
    sharding linearity, and exact zeros on the masked prefix rows."""
    from specdec import ops

    N, B, V, C = 64, 32, 151936, 8
    x, t, m = _workload(N, B, V, 3.0, 8, 1)
    loss, lse, scale, loss_n = ops.dpace_forward(x, t, m, 0.5, 0, want_loss_n=True)
    g = ops.dpace_backward(x, t, lse, scale, None)
    loss_f, g_f, lse_f, scale_f, _ = ops.dpace_forward_backward(x, t, m, 0.5, 0)
    torch.cuda.synchronize()
    assert float(loss_f) == float(loss)
    assert torch.equal(lse_f, lse) and torch.equal(scale_f, scale)
    assert torch.equal(g_f, g)
    del g_f
    want_total = 0.0
    worst = 0.0
    for lo in range(0, N, C):
        sl = slice(lo, lo + C)
        want_c, g_c = odp.dpace_fwd_bwd_torch(x[sl].cpu(), t[sl].cpu(), 0.5, m[sl].cpu())
        want_total += float(want_c) * C / N
        worst = max(worst, float((g[sl].cpu() - g_c * (C / N)).abs().max()))
        # per-sequence losses of the chunk
        for n in range(lo, lo + C):
            wn = float(odp.dpace_loss_torch(x[n:n + 1].cpu(), t[n:n + 1].cpu(), 0.5, m[n:n + 1].cpu()))
            assert abs(float(loss_n[n]) - wn) <= LOSS_RTOL * abs(wn) + 1e-12, n
    _close_loss(float(loss), want_total)
    assert worst <= GRAD_ATOL, worst
    parts = []
    for lo in range(0, N, 16):
        p, _, _, _ = ops.dpace_forward(x[lo:lo + 16], t[lo:lo + 16], m[lo:lo + 16], 0.5, 0, n_global=N)
        parts.append(float(p))
    assert abs(sum(parts) - float(loss)) <= 1e-5 * abs(float(loss))
    dead = (m == 0)
    assert bool(dead.any())
    assert float(g[dead].abs().max()) == 0.0


SHAPE_CASES = [c for c in cases.DPACE_CASES if c["name"] in (
    "bern.5_N8_B8_V1024", "B32_N8_V1024", "V7_N6_B8", "V1000_N6_B8", "shift-20_N8_B4_V1024",
    "type_SP_N4_B8_V1024", "seq0masked_N4_B8_V512", "ws2_N4_B16_V128256_sd2_prefix4")]


@pytest.mark.parametrize("shape", [0, 1, 2, 3, 4, 5, 6, 7, 8, 10, 11, 12, 13, 14])
def test_every_launch_shape_matches_golden(cuda, gd, shape):
    """Shapes 0-8: warp-specialized bulk-copy ring variants; 10-14: 128-bit-load kernels."""
    from specdec import _lib

    try:
        _lib.set_launch_shape(_lib.KERNEL_DPACE_FWD, shape)
        _lib.set_launch_shape(_lib.KERNEL_DPACE_BWD, shape)
        for case in SHAPE_CASES:
            x, t, m = cases.dpace_inputs(case)
            key = case["name"]
            loss, grad = _run(x, t, m, case["alpha"], case["loss_type"])
            _close_loss(loss, float(gd[f"{key}/loss"]))
            if f"{key}/grad" in gd.files:
                np.testing.assert_allclose(grad, gd[f"{key}/grad"], rtol=0, atol=GRAD_ATOL)
            else:
                idx = gd[f"{key}/probe_idx"]
                np.testing.assert_allclose(grad.reshape(-1)[idx], gd[f"{key}/probe_val"], rtol=0,
                                           atol=GRAD_ATOL)
    finally:
        _lib.set_launch_shape(_lib.KERNEL_DPACE_FWD, _lib.SHAPE_DEFAULT)
        _lib.set_launch_shape(_lib.KERNEL_DPACE_BWD, _lib.SHAPE_DEFAULT)


def test_static_block_interleave_matches_golden(cuda, gd):
    """The ring kernels with the atomic block queue off (static interleave)."""
    from specdec import _lib

    try:
        _lib.set_block_queue(False)
        for case in SHAPE_CASES:
            x, t, m = cases.dpace_inputs(case)
            loss, grad = _run(x, t, m, case["alpha"], case["loss_type"])
            _close_loss(loss, float(gd[f"{case['name']}/loss"]))
            _, g_or = odp.dpace_fwd_bwd_torch(torch.from_numpy(x), torch.from_numpy(t), case["alpha"],
                                              None if m is None else torch.from_numpy(m),
                                              case["loss_type"])
            np.testing.assert_allclose(grad, g_or.numpy(), rtol=0, atol=GRAD_ATOL)
    finally:
        _lib.set_block_queue(True)


def test_ring_results_are_schedule_independent(cuda):
    """Partials are slotted by block index, so the dynamic queue's schedule does
    not change a single bit of the loss or the gradient."""
    from specdec import _lib, ops

    x, t, m = _workload(16, 16, 128256, 2.0, 4, 3)
    ref = None
    for dynamic in (True, False, True):
        _lib.set_block_queue(dynamic)
        loss, lse, scale, _ = ops.dpace_forward(x, t, m, 0.5, 0)
        g = ops.dpace_backward(x, t, lse, scale, None)
        if ref is None:
            ref = (loss.clone(), lse.clone(), g.clone())
        else:
            assert torch.equal(loss, ref[0]) and torch.equal(lse, ref[1]) and torch.equal(g, ref[2])
    _lib.set_block_queue(True)
