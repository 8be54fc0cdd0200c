"""Failure detection on the GPU without a fault: a bounded wait that runs out.

specdec_test_withhold_stage(1) makes CTA 0 of the next D-PACE or DFlash
forward never post its first stage. Its consumer warps wait on that stage's mbarrier, give up
after the 1 s limit, record the timeout in the status word, wait (bounded) for
the copies they may still have in flight and return; the launch completes.
The host must see the error (D-PACE: RuntimeError through the drop-in API,
status 5 and a NaN loss through the C ABI; DFlash: a NaN loss) and the next
call must be normal: context usable, counters zero, results equal to the
oracle's."""
import pytest
import torch

from oracle import dpace as odp

pytestmark = pytest.mark.gpu


def _inputs():
    # 41 M elements: ~2500 ring blocks, several per CTA, so CTA 0 is busy
    g = torch.Generator(device="cuda").manual_seed(21)
    x = torch.randn(64, 16, 40000, device="cuda", generator=g) * 2.0
    t = torch.randint(0, 40000, (64, 16), device="cuda", generator=g)
    return x, t


def test_expired_wait_is_reported_and_the_next_call_is_normal(cuda):
    from losses import dpace_loss, fused_dpace_loss
    from specdec import _lib

    x, t = _inputs()
    want, g_ref = odp.dpace_fwd_bwd_torch(x.cpu(), t.cpu())
    lib = _lib.load()
    try:
        _lib.check(lib.specdec_test_withhold_stage(1), "specdec_test_withhold_stage")
        with pytest.raises(RuntimeError, match="timed out"):
            fused_dpace_loss(x, t)
    finally:
        lib.specdec_test_withhold_stage(0)
    torch.cuda.synchronize()
    # the context and the workspace are usable again
    loss = float(fused_dpace_loss(x, t))
    assert abs(loss - float(want)) <= 1e-5 * abs(float(want))
    xg = x.clone().requires_grad_(True)
    dpace_loss(xg, t).backward()
    assert float((xg.grad.cpu() - g_ref).abs().max()) <= 1e-6


def test_expired_wait_status_through_the_c_abi(cuda):
    from specdec import _lib

    lib = _lib.load()
    x, t = _inputs()
    N, B, V = x.shape
    loss = torch.empty((), device="cuda")
    lse = torch.empty(N, B, device="cuda")
    scale = torch.empty(N, B, device="cuda")
    status = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    sb = lib.specdec_dpace_scratch_bytes(N, B, V, 0)
    cb = lib.specdec_dpace_counter_bytes(N, B)
    scratch = torch.empty(sb, dtype=torch.uint8, device="cuda")
    counters = torch.zeros(cb, dtype=torch.uint8, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream

    def call():
        return lib.specdec_dpace_forward(x.data_ptr(), t.data_ptr(), None, N, B, V, 0.5, 0, N, loss.data_ptr(),
                                         None, lse.data_ptr(), scale.data_ptr(), status.data_ptr(),
                                         scratch.data_ptr(), sb, counters.data_ptr(), cb, stream)

    try:
        lib.specdec_test_withhold_stage(1)
        assert call() == _lib.OK  # the launch itself succeeds
        torch.cuda.synchronize()
        assert int(status.item()) == _lib.ERR_CUDA
        assert bool(torch.isnan(loss))  # never a plausible wrong number
    finally:
        lib.specdec_test_withhold_stage(0)
    counters.zero_()  # after a timeout the caller clears its counters
    assert call() == _lib.OK
    torch.cuda.synchronize()
    assert int(status.item()) == _lib.OK
    want, _ = odp.dpace_fwd_bwd_torch(x.cpu(), t.cpu())
    assert abs(float(loss) - float(want)) <= 1e-5 * abs(float(want))


def test_dflash_expired_wait_gives_nan_loss_and_the_next_call_is_normal(cuda):
    """The DFlash forward has no status word (its reference interface has no
    device-side check): an expired wait shows as a NaN loss."""
    from models.dflash import fused_dflash_loss
    from oracle import dflash as odf
    from specdec import _lib

    x, _ = _inputs()
    y = 0.5 * x  # a different distribution: KL well away from 0
    lib = _lib.load()
    try:
        _lib.check(lib.specdec_test_withhold_stage(1), "specdec_test_withhold_stage")
        loss = fused_dflash_loss(x, y)
        torch.cuda.synchronize()
        assert bool(torch.isnan(loss))
    finally:
        lib.specdec_test_withhold_stage(0)
    want, _ = odf.dflash_fwd_bwd_torch(x.cpu(), y.cpu())
    loss = float(fused_dflash_loss(x, y))
    assert abs(loss - float(want)) <= 1e-5 * abs(float(want))
