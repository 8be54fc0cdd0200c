"""D-PACE forward + backward in one call (specdec_dpace_forward_backward):
bit-for-bit the separate forward and backward calls, for both logit types;
the autograd mode that computes the gradient in the forward applies dloss in
the backward and survives a retained graph; expired waits are reported; CUDA
graph capture replays it."""
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


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("N,B,V,lt", [(64, 16, 128256, 0), (8, 32, 50257, 2), (40, 7, 3001, 1),
                                      (200, 4, 37, 0), (3, 1, 1, 0), (16, 16, 16384, 2)])
def test_forward_backward_equals_separate_calls(cuda, dtype, N, B, V, lt):
    from specdec import ops

    x, t, m = _inputs(N, B, V, N * 7 + V, dtype)
    loss_s, grad_s, lse_s, scale_s = _separate(x, t, m, 0.5, lt)
    loss_f, grad_f, lse_f, scale_f, _ = ops.dpace_forward_backward(x, t, m, 0.5, lt)
    torch.cuda.synchronize()
    assert float(loss_f) == float(loss_s)
    assert torch.equal(lse_f, lse_s) and torch.equal(scale_f, scale_s)
    assert torch.equal(grad_f, grad_s)


def test_forward_backward_matches_oracle_and_loss_n(cuda):
    from specdec import ops

    x, t, m = _inputs(6, 16, 20000, 3, mask_p=0.7)
    want, g_ref = odp.dpace_fwd_bwd_torch(x.cpu(), t.cpu(), 0.5, m.cpu(), "dpace-continuation-value-only")
    loss, grad, _, _, loss_n = ops.dpace_forward_backward(x, t, m, 0.5, 2, want_loss_n=True)
    assert abs(float(loss) - float(want)) <= 1e-5 * abs(float(want))
    assert float((grad.cpu() - g_ref).abs().max()) <= 1e-6
    assert abs(float(loss) - float(loss_n.sum() / 6)) <= 1e-5 * abs(float(loss))


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


def test_autograd_modes_agree(cuda):
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
    # dloss = 2 scales exactly in both orders
    assert losses[0] == losses[1] and torch.equal(grads[0], grads[1])


def test_expired_wait_reported_then_normal(cuda):
    from specdec import _lib, ops

    x, t, m = _inputs(64, 16, 40000, 13)
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


def test_graph_capture(cuda):
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
    loss_s, grad_s, _, _ = _separate(x, t, m, 0.5, 0)
    assert float(loss_g) == float(loss_s) and torch.equal(grad_g, grad_s)
