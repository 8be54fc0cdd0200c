"""D-PACE forward + backward in one launch (specdec_dpace_forward_backward):
the shared-memory pipeline runs for the reference shapes; it agrees with the
separate forward and backward kernels to float rounding (its partial sums
merge in another order) and with the oracle to the parity tolerance; it is
deterministic and independent of the number of slots; masked rows get exact
zeros; dloss is applied by the autograd backward; expired waits are reported;
CUDA graph capture replays it."""
import pytest
import torch

from oracle import dpace as odp

pytestmark = pytest.mark.gpu


def _inputs(N, B, V, seed, dtype=torch.float32, mask_p=0.8, sigma=2.0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = (torch.randn(N, B, V, device="cuda", generator=g) * sigma).to(dtype)
    t = torch.randint(0, V, (N, B), device="cuda", generator=g)
    m = (torch.rand(N, B, device="cuda", generator=g) < mask_p).float()
    return x, t, m


def _separate(x, t, m, alpha, lt):
    from specdec import ops

    loss, lse, scale, _ = ops.dpace_forward(x, t, m, alpha, lt)
    return loss, ops.dpace_backward(x, t, lse, scale, None), lse, scale


def _slots(B, V, dtype):
    from specdec import _lib

    return _lib.load().specdec_dpace_pipeline_slots(B, V, int(dtype == torch.bfloat16), torch.cuda.current_device())


def _close(a, b, rtol, atol):
    a, b = a.float(), b.float()
    return bool(((a - b).abs() <= atol + rtol * b.abs()).all())


def test_pipeline_taken_for_reference_shapes(cuda):
    # [*, 16, 128256] and [*, 16, 32000]: fp32 and bf16 run the pipeline
    assert _slots(16, 128256, torch.float32) >= 3
    assert _slots(16, 128256, torch.bfloat16) >= _slots(16, 128256, torch.float32)
    assert _slots(16, 32000, torch.float32) >= 3
    # V * 4 bytes not a multiple of 16, or tiny rows: the separate kernels
    assert _slots(16, 50257, torch.float32) == 0
    assert _slots(4, 37, torch.float32) == 0


SHAPES = [(64, 16, 128256, 0), (8, 32, 50304, 2), (16, 16, 16384, 2), (5, 3, 4096, 0), (2, 32, 1024, 1),
          (40, 7, 3001, 1), (3, 1, 1, 0), (8, 32, 50257, 2)]


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("N,B,V,lt", SHAPES)
def test_fused_matches_separate_kernels(cuda, dtype, N, B, V, lt):
    from specdec import ops

    x, t, m = _inputs(N, B, V, N * 7 + V, dtype)
    loss_s, grad_s, lse_s, scale_s = _separate(x, t, m, 0.5, lt)
    loss_f, grad_f, lse_f, scale_f, _ = ops.dpace_forward_backward(x, t, m, 0.5, lt)
    torch.cuda.synchronize()
    assert abs(float(loss_f) - float(loss_s)) <= 2e-6 * abs(float(loss_s)) + 1e-12
    assert _close(lse_f, lse_s, 1e-6, 1e-6)
    assert _close(scale_f, scale_s, 1e-5, 1e-12)
    # p = e^(x - lse) inherits lse's relative rounding; a bf16 gradient may
    # also round to the neighbouring bf16 value (one ulp: up to 2^-7 relative)
    rtol = 2.0 ** -7 if dtype == torch.bfloat16 else 2e-5
    assert _close(grad_f, grad_s, rtol, 1e-9)


@pytest.mark.parametrize("N,B,V,lt", [(6, 16, 20000, 0), (4, 32, 8192, 1), (9, 5, 12288, 2)])
def test_fused_matches_oracle(cuda, N, B, V, lt):
    from specdec import ops

    x, t, m = _inputs(N, B, V, 3 + V, mask_p=0.7)
    assert _slots(B, V, torch.float32) >= 3
    name = ["dpace", "dpace-cumulative-confidence-only", "dpace-continuation-value-only"][lt]
    want, g_ref = odp.dpace_fwd_bwd_torch(x.cpu(), t.cpu(), 0.5, m.cpu(), name)
    loss, grad, _, _, _ = ops.dpace_forward_backward(x, t, m, 0.5, lt)
    assert abs(float(loss) - float(want)) <= 1e-5 * abs(float(want))
    assert float((grad.cpu() - g_ref).abs().max()) <= 1e-6


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_slots_do_not_change_results(cuda, dtype):
    from specdec import _lib, ops

    x, t, m = _inputs(24, 16, 128256, 5, dtype)
    lib = _lib.load()
    kmax = _slots(16, 128256, dtype)
    assert kmax >= 3
    outs = []
    try:
        for k in range(3, kmax + 1):
            _lib.check(lib.specdec_set_pipe_slots(k), "specdec_set_pipe_slots")
            assert _slots(16, 128256, dtype) == k
            loss, grad, lse, scale, _ = ops.dpace_forward_backward(x, t, m, 0.5, 0)
            outs.append((float(loss), grad.clone(), lse.clone(), scale.clone()))
    finally:
        lib.specdec_set_pipe_slots(0)
    for o in outs[1:]:
        assert o[0] == outs[0][0]
        assert torch.equal(o[1], outs[0][1]) and torch.equal(o[2], outs[0][2]) and torch.equal(o[3], outs[0][3])


def test_slot_cap_rejects_out_of_range(cuda):
    from specdec import _lib

    lib = _lib.load()
    assert lib.specdec_set_pipe_slots(2) != 0
    assert lib.specdec_set_pipe_slots(9) != 0
    assert lib.specdec_set_pipe_slots(0) == 0


def test_deterministic_and_loss_n(cuda):
    from specdec import ops

    x, t, m = _inputs(32, 16, 128256, 21)
    a = ops.dpace_forward_backward(x, t, m, 0.3, 2, want_loss_n=True)
    b = ops.dpace_forward_backward(x, t, m, 0.3, 2, want_loss_n=True)
    assert float(a[0]) == float(b[0])
    assert all(torch.equal(u, v) for u, v in zip(a[1:], b[1:]))
    _, _, _, loss_n_s = ops.dpace_forward(x, t, m, 0.3, 2, want_loss_n=True)
    assert _close(a[4], loss_n_s, 2e-6, 1e-9)
    assert abs(float(a[0]) - float(a[4].sum() / 32)) <= 1e-5 * abs(float(a[0]))


def test_masked_rows_exact_zero_and_all_masked(cuda):
    from specdec import ops

    x, t, _ = _inputs(12, 16, 32000, 8)
    m = torch.ones(12, 16, device="cuda")
    m[:, :3] = 0
    m[5] = 0
    _, grad, lse, scale, _ = ops.dpace_forward_backward(x, t, m, 0.5, 0)
    dead = m == 0
    assert float(grad[dead].abs().max()) == 0.0
    assert float(lse[dead].abs().max()) == 0.0 and float(scale[dead].abs().max()) == 0.0
    loss, grad, _, _, _ = ops.dpace_forward_backward(x, t, torch.zeros_like(m), 0.5, 0)
    assert float(loss) == 0.0 and float(grad.abs().max()) == 0.0


def test_out_of_range_target_raises(cuda):
    from specdec import ops

    x, t, m = _inputs(4, 16, 32000, 9)
    t[2, 5] = 32000
    with pytest.raises(ValueError):
        ops.dpace_forward_backward(x, t, m, 0.5, 0)
    t[2, 5] = 7
    ops.dpace_forward_backward(x, t, m, 0.5, 0)


@pytest.fixture
def fused_autograd():
    from specdec import ops

    saved = ops.FUSED_BACKWARD
    ops.set_fused_backward(True)
    yield
    ops.set_fused_backward(saved)


def test_autograd_uses_dloss_and_matches_oracle(cuda, fused_autograd):
    from losses import dpace_loss

    x, t, m = _inputs(6, 16, 20000, 11)
    want, g_ref = odp.dpace_fwd_bwd_torch(x.cpu(), t.cpu(), 0.5, m.cpu())
    for factor in (1.0, 3.0, -0.25):
        xg = x.clone().requires_grad_(True)
        loss = dpace_loss(xg, t, 0.5, m)
        (loss * factor).backward()
        assert abs(float(loss.detach()) - float(want)) <= 1e-5 * abs(float(want))
        assert float((xg.grad.cpu() - factor * g_ref).abs().max()) <= 1e-6 * max(1.0, abs(factor))


def test_retained_graph_second_backward(cuda, fused_autograd):
    from losses import dpace_loss

    x, t, m = _inputs(4, 16, 9000, 12)
    xg = x.clone().requires_grad_(True)
    loss = dpace_loss(xg, t, 0.5, m)
    loss.backward(retain_graph=True)
    g1 = xg.grad.clone()
    loss.backward()
    assert float((xg.grad - 2 * g1).abs().max()) <= 1e-6


def test_autograd_fused_matches_separate(cuda):
    from losses import dpace_loss
    from specdec import ops

    x, t, m = _inputs(8, 16, 30000, 15)
    grads, losses = [], []
    saved = ops.FUSED_BACKWARD
    try:
        for fused in (False, True):
            ops.set_fused_backward(fused)
            xg = x.clone().requires_grad_(True)
            loss = dpace_loss(xg, t, 0.5, m)
            (loss * 2.0).backward()
            grads.append(xg.grad)
            losses.append(float(loss.detach()))
    finally:
        ops.set_fused_backward(saved)
    assert abs(losses[0] - losses[1]) <= 2e-6 * abs(losses[0])
    assert _close(grads[1], grads[0], 2e-5, 1e-9)


def test_fused_expired_wait_reported_then_normal(cuda):
    from specdec import _lib, ops

    x, t, m = _inputs(64, 16, 40000, 13)
    assert _slots(16, 40000, torch.float32) >= 3
    before = ops.dpace_forward_backward(x, t, m, 0.5, 0)
    lib = _lib.load()
    try:
        _lib.check(lib.specdec_test_withhold_stage(1), "specdec_test_withhold_stage")
        with pytest.raises(RuntimeError, match="timed out"):
            ops.dpace_forward_backward(x, t, m, 0.5, 0)
    finally:
        lib.specdec_test_withhold_stage(0)
    torch.cuda.synchronize()
    after = ops.dpace_forward_backward(x, t, m, 0.5, 0)
    torch.cuda.synchronize()
    assert float(after[0]) == float(before[0]) and torch.equal(after[1], before[1])


def test_fused_graph_capture(cuda):
    from specdec import ops

    x, t, m = _inputs(8, 16, 50000, 14)
    side = torch.cuda.Stream()
    for _ in range(2):
        with torch.cuda.stream(side):
            ops.dpace_forward_backward(x, t, m, 0.5, 0, validate=False)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side):
        loss_g, grad_g, _, _, _ = ops.dpace_forward_backward(x, t, m, 0.5, 0, validate=False)
    g = torch.Generator(device="cuda").manual_seed(99)
    x.copy_(torch.randn(x.shape, device="cuda", generator=g) * 2)
    graph.replay()
    torch.cuda.synchronize()
    loss_d, grad_d, _, _, _ = ops.dpace_forward_backward(x, t, m, 0.5, 0, validate=False)
    torch.cuda.synchronize()
    assert float(loss_g) == float(loss_d) and torch.equal(grad_g, grad_d)
