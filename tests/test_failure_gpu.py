"""Failure detection on the GPU without a fault: a bounded wait that runs out.

specdec_test_withhold_stage(1) makes CTA 0 of the next D-PACE or DFlash
launch on the ring path (forward or backward) never post its first stage. Its
consumer warps wait on that stage's mbarrier, give up after the 1 s limit,
record the timeout, wait (bounded) for the copies they may still have in
flight and return; the launch completes. The host must see the error --
forward: a NaN loss and NaN per-row outputs (so a backward from them is NaN
throughout), status 5 for D-PACE, RuntimeError through the drop-in API;
backward: status 5 and NaN over every block the failed CTA may have left
unfinished, never a partly stale gradient -- and the next call must be
normal: context usable, counters zero, results equal to the oracle's."""
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


def _dpace_state(x, t):
    from specdec import ops

    loss, lse, scale, _ = ops.dpace_forward(x, t, None, 0.5, 0)
    return lse, scale


def _nan_blocks_else_exact(g, g_ref):
    """Every element is NaN or within 1e-6 of the oracle; returns the NaN count."""
    nan = torch.isnan(g)
    ok = (g - g_ref).abs() <= 1e-6
    assert bool((nan | ok).all())
    return int(nan.sum())


def test_backward_expired_wait_gives_status_and_nan_blocks(cuda):
    from specdec import _lib, ops

    x, t = _inputs()
    _, g_ref = odp.dpace_fwd_bwd_torch(x.cpu(), t.cpu())
    lse, scale = _dpace_state(x, t)
    lib = _lib.load()
    try:
        _lib.check(lib.specdec_test_withhold_stage(1), "specdec_test_withhold_stage")
        g = ops.dpace_backward(x, t, lse, scale, None)  # asynchronous: no error yet
        torch.cuda.synchronize()
    finally:
        lib.specdec_test_withhold_stage(0)
    assert int(_lib.status_words(x.device)[_lib.STATUS_DPACE_BWD]) == _lib.ERR_CUDA
    n = _nan_blocks_else_exact(g.cpu(), g_ref)
    assert 0 < n <= 2 * 16384  # the (at most two) blocks CTA 0 held
    with pytest.raises(RuntimeError, match="earlier backward"):
        ops.check_backward(x.device)
    ops.check_backward(x.device)  # reported once
    g = ops.dpace_backward(x, t, lse, scale, None)
    assert float((g.cpu() - g_ref).abs().max()) <= 1e-6
    ops.check_backward(x.device)


def test_backward_expired_wait_is_raised_by_the_next_forward(cuda):
    from losses import fused_dpace_loss
    from specdec import _lib, ops

    x, t = _inputs()
    lse, scale = _dpace_state(x, t)
    lib = _lib.load()
    try:
        lib.specdec_test_withhold_stage(1)
        ops.dpace_backward(x, t, lse, scale, None)
    finally:
        lib.specdec_test_withhold_stage(0)
    with pytest.raises(RuntimeError, match="earlier backward"):
        fused_dpace_loss(x, t)
    want, _ = odp.dpace_fwd_bwd_torch(x.cpu(), t.cpu())
    assert abs(float(fused_dpace_loss(x, t)) - float(want)) <= 1e-5 * abs(float(want))


def test_backward_expired_wait_status_without_counters(cuda):
    """Static block interleave (no counter block): the entry point clears the
    status word on the stream and the failed CTA raises it; that CTA owns
    every grid-th block, and all of its blocks not finished are NaN."""
    import math

    from specdec import _lib

    lib = _lib.load()
    x, t = _inputs()
    N, B, V = x.shape
    _, g_ref = odp.dpace_fwd_bwd_torch(x.cpu(), t.cpu())
    lse, scale = _dpace_state(x, t)
    g = torch.empty_like(x)
    status = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream

    def call():
        return lib.specdec_dpace_backward(x.data_ptr(), t.data_ptr(), lse.data_ptr(), scale.data_ptr(), None,
                                          g.data_ptr(), N, B, V, status.data_ptr(), None, 0, stream)

    try:
        lib.specdec_test_withhold_stage(1)
        assert call() == _lib.OK
        torch.cuda.synchronize()
    finally:
        lib.specdec_test_withhold_stage(0)
    assert int(status.item()) == _lib.ERR_CUDA
    ctas = lib.specdec_launch_ctas(_lib.KERNEL_DPACE_BWD, N * B, V, 0)
    per_cta = math.ceil(math.ceil(N * B * V / 16384) / ctas)
    assert 0 < _nan_blocks_else_exact(g.cpu(), g_ref) <= per_cta * 16384
    assert call() == _lib.OK
    torch.cuda.synchronize()
    assert int(status.item()) == _lib.OK
    assert float((g.cpu() - g_ref).abs().max()) <= 1e-6


def test_dflash_backward_expired_wait_gives_status_and_nan_blocks(cuda):
    from oracle import dflash as odf
    from specdec import _lib, ops

    x, _ = _inputs()
    y = 0.5 * x
    _, g_ref = odf.dflash_fwd_bwd_torch(x.cpu(), y.cpu())
    B = x.shape[1]
    _, _, scale, lzq, lzp, _ = ops.dflash_forward(x, y, None, 4.0, False, 0, B)
    lib = _lib.load()
    try:
        lib.specdec_test_withhold_stage(1)
        g = ops.dflash_backward(x, y, scale, lzq, lzp, None, None, 0)
        torch.cuda.synchronize()
    finally:
        lib.specdec_test_withhold_stage(0)
    assert int(_lib.status_words(x.device)[_lib.STATUS_DFLASH_BWD]) == _lib.ERR_CUDA
    assert 0 < _nan_blocks_else_exact(g.cpu(), g_ref) <= 2 * 16384
    with pytest.raises(RuntimeError, match="earlier backward"):
        ops.check_backward(x.device)
    g = ops.dflash_backward(x, y, scale, lzq, lzp, None, None, 0)
    assert float((g.cpu() - g_ref).abs().max()) <= 1e-6


def test_dflash_forward_expired_wait_makes_the_whole_gradient_nan(cuda):
    """A failed forward writes NaN scale / log-normalisers, so autograd's
    backward from it cannot return a plausible gradient."""
    from models.dflash import dflash_loss
    from specdec import _lib

    x, _ = _inputs()
    y = 0.5 * x
    xg = x.clone().requires_grad_(True)
    lib = _lib.load()
    try:
        lib.specdec_test_withhold_stage(1)
        loss = dflash_loss(xg, y)
    finally:
        lib.specdec_test_withhold_stage(0)
    loss.backward()
    torch.cuda.synchronize()
    assert bool(torch.isnan(loss.detach()))
    assert bool(torch.isnan(xg.grad).all())


def _attn_inputs(seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    B, T, H = 2, 528, 2
    return [torch.randn(B, T, H, 64, device="cuda", generator=g).to(torch.bfloat16) for _ in range(4)]


def test_attention_expired_wait_gives_status_and_nan_rows(cuda):
    """The drafter's attention: with a stage withheld the grid's first CTA
    (batch 0, head 0, the last query tile -- the block slots, rows 512..527)
    gives up after its bounded wait; *status is 5 and exactly its rows of o
    and lse are NaN; every other row equals a normal call's. The backward the
    same: status 5, the failed CTAs' rows of dq (query rows 512..527) and of
    dk / dv (keys 0..127) NaN, the rest normal."""
    from specdec import _lib

    lib = _lib.load()
    q, k, v, do = _attn_inputs(5)
    B, T, H, _ = q.shape
    s = torch.cuda.current_stream().cuda_stream

    def fwd(status):
        o = torch.empty_like(q)
        lse = torch.empty(B, H, T, device="cuda")
        rc = lib.specdec_dflash_attention_forward(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(),
                                                  lse.data_ptr(), B, T, H, 64, 512, 0.125, status.data_ptr(), s)
        assert rc == _lib.OK, _lib.last_error()
        return o, lse

    def bwd(o, lse, status):
        dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
        wsb = lib.specdec_dflash_attention_workspace_bytes(B, T, H)
        ws = torch.empty(wsb, dtype=torch.uint8, device="cuda")
        rc = lib.specdec_dflash_attention_backward(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(),
                                                   lse.data_ptr(), do.data_ptr(), dq.data_ptr(), dk.data_ptr(),
                                                   dv.data_ptr(), B, T, H, 64, 512, 0.125, status.data_ptr(),
                                                   ws.data_ptr(), wsb, s)
        assert rc == _lib.OK, _lib.last_error()
        return dq, dk, dv

    good = torch.zeros(1, dtype=torch.int32, device="cuda")
    o_ref, lse_ref = fwd(good)
    dq_ref, dk_ref, dv_ref = bwd(o_ref, lse_ref, good)
    torch.cuda.synchronize()
    assert int(good.item()) == 0
    bad = torch.zeros(1, dtype=torch.int32, device="cuda")
    try:
        _lib.check(lib.specdec_test_withhold_stage(1), "specdec_test_withhold_stage")
        o, lse = fwd(bad)
    finally:
        lib.specdec_test_withhold_stage(0)
    torch.cuda.synchronize()
    assert int(bad.item()) == 5
    failed = torch.zeros(B, T, H, dtype=torch.bool, device="cuda")
    failed[0, 512:, 0] = True
    assert bool(torch.isnan(o.float())[failed].all()) and bool(torch.isnan(lse[0, 0, 512:]).all())
    assert torch.equal(o[~failed], o_ref[~failed])
    keep = torch.ones(B, H, T, dtype=torch.bool, device="cuda")
    keep[0, 0, 512:] = False
    assert torch.equal(lse[keep], lse_ref[keep])
    # the backward, from the good forward's outputs
    bad.zero_()
    try:
        _lib.check(lib.specdec_test_withhold_stage(1), "specdec_test_withhold_stage")
        dq, dk, dv = bwd(o_ref, lse_ref, bad)
    finally:
        lib.specdec_test_withhold_stage(0)
    torch.cuda.synchronize()
    assert int(bad.item()) == 5
    fq = torch.zeros(B, T, H, dtype=torch.bool, device="cuda")
    fq[0, 512:, 0] = True
    fk = torch.zeros(B, T, H, dtype=torch.bool, device="cuda")
    fk[0, :128, 0] = True
    assert bool(torch.isnan(dq.float())[fq].all()) and torch.equal(dq[~fq], dq_ref[~fq])
    assert bool(torch.isnan(dk.float())[fk].all()) and torch.equal(dk[~fk], dk_ref[~fk])
    assert bool(torch.isnan(dv.float())[fk].all()) and torch.equal(dv[~fk], dv_ref[~fk])
    # the next calls are normal
    again = torch.zeros(1, dtype=torch.int32, device="cuda")
    o2, lse2 = fwd(again)
    dq2, dk2, dv2 = bwd(o2, lse2, again)
    torch.cuda.synchronize()
    assert int(again.item()) == 0 and torch.equal(o2, o_ref) and torch.equal(dq2, dq_ref)


def test_attention_expired_wait_is_raised_by_the_next_check(cuda):
    """Through the drafter module: the sticky stream status word carries an
    attention timeout to the next synchronising check (RuntimeError), which
    clears it."""
    from specdec import _lib, drafter, ops

    lib = _lib.load()
    q, k, v, _ = _attn_inputs(6)
    ops.check_backward()  # clean start
    try:
        _lib.check(lib.specdec_test_withhold_stage(1), "specdec_test_withhold_stage")
        with torch.no_grad():
            o = drafter.dflash_attention(q, k, v, 512)
    finally:
        lib.specdec_test_withhold_stage(0)
    with pytest.raises(RuntimeError, match="attention"):
        ops.check_backward()
    assert bool(torch.isnan(o[0, 512:, 0].float()).all())
    ops.check_backward()  # cleared
    with torch.no_grad():
        o2 = drafter.dflash_attention(q, k, v, 512)
    ops.check_backward()
    assert not bool(torch.isnan(o2.float()).any())
