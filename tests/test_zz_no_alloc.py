"""The no-allocation D-PACE forward (specdec_dpace_forward_noalloc).

That entry point exists for callers that cannot allocate device memory (a
plugin host that passes only input and output buffers, or a process whose
device memory is all held by its own pool): it keeps its scratch in a fixed
array inside libspecdec.so instead of asking for a workspace. This test calls
it through the C ABI twice in a row, on two different batches, and checks each
result against the allocating entry point, specdec_dpace_forward, on the same
inputs: loss within 1e-5 relative, per-row lse and scale within 1e-6
absolute. It also checks that the size limit is exactly the documented one
(the workspace queries against the array's two regions: a problem just inside
runs and matches, one just outside is refused up front), that argument errors
are reported before the size check, and that a call whose bounded wait ran out
(the failure-detection hook) reports it and leaves the shared array usable for
the next call without any clearing by the caller. The file is named to be
collected last.
"""
import ctypes

import pytest
import torch

from specdec import _lib, ops

pytestmark = pytest.mark.gpu

LOSS_RTOL = 1e-5
ROW_ATOL = 1e-6
# the built-in array: 4 MiB, the first 64 KiB for counters, the rest scratch
ARRAY_BYTES = 4 << 20
COUNTER_REGION = 64 << 10


def _batch(N, B, V, seed, dev):
    g = torch.Generator(device=dev).manual_seed(seed)
    x = torch.randn(N, B, V, device=dev, generator=g) * 2.0
    t = torch.randint(0, V, (N, B), device=dev, generator=g)
    k = torch.randint(0, 5, (N, 1), device=dev, generator=g)
    m = (torch.arange(B, device=dev).view(1, B) >= k).float()
    return x, t, m


def _noalloc(lib, x, t, m, alpha=0.5, loss_type=0, expect_status=_lib.OK):
    N, B, V = x.shape
    dev = x.device
    loss = torch.empty((), device=dev)
    loss_n = torch.empty(N, device=dev)
    lse = torch.empty(N, B, device=dev)
    scale = torch.empty(N, B, device=dev)
    status = torch.full((1,), -1, dtype=torch.int32, device=dev)
    rc = lib.specdec_dpace_forward_noalloc(
        x.data_ptr(), t.data_ptr(), m.data_ptr(), N, B, V, alpha, loss_type, N, loss.data_ptr(),
        loss_n.data_ptr(), lse.data_ptr(), scale.data_ptr(), status.data_ptr(),
        torch.cuda.current_stream(dev).cuda_stream)
    assert rc == _lib.OK, _lib.last_error()
    torch.cuda.synchronize(dev)
    assert int(status.item()) == expect_status
    return loss, loss_n, lse, scale


def _check_against_allocating(lib, x, t, m, tag):
    want_loss, want_lse, want_scale, want_loss_n = ops.dpace_forward(x, t, m, 0.5, 0, want_loss_n=True)
    loss, loss_n, lse, scale = _noalloc(lib, x, t, m)
    w = float(want_loss)
    assert abs(float(loss) - w) <= LOSS_RTOL * abs(w), (tag, float(loss), w)
    assert (lse - want_lse).abs().max().item() <= ROW_ATOL, tag
    assert (scale - want_scale).abs().max().item() <= ROW_ATOL, tag
    assert (loss_n - want_loss_n).abs().max().item() <= LOSS_RTOL * want_loss_n.abs().max().item(), tag


def _fits(lib, N, B, V, dev):
    return (lib.specdec_dpace_counter_bytes(N, B) <= COUNTER_REGION
            and lib.specdec_dpace_scratch_bytes(N, B, V, dev) <= ARRAY_BYTES - COUNTER_REGION)


def test_noalloc_matches_allocating_forward(cuda):
    lib = _lib.load()
    for call, (N, B, V, seed) in enumerate([(16, 16, 128256, 11), (8, 32, 151936, 12)]):
        x, t, m = _batch(N, B, V, seed, cuda)
        _check_against_allocating(lib, x, t, m, call)


def test_noalloc_limit_is_the_documented_query(cuda):
    """The largest N that the workspace queries say fits runs and matches;
    one more sequence is refused with SPECDEC_ERR_WORKSPACE, nothing launched."""
    lib = _lib.load()
    B, V = 32, 1024
    lo, hi = 1, 1 << 15  # lo fits, hi does not
    assert _fits(lib, lo, B, V, cuda.index) and not _fits(lib, hi, B, V, cuda.index)
    while hi - lo > 1:
        mid = (lo + hi) // 2
        lo, hi = (mid, hi) if _fits(lib, mid, B, V, cuda.index) else (lo, mid)
    x, t, m = _batch(lo, B, V, 13, cuda)
    _check_against_allocating(lib, x, t, m, f"N={lo}")
    fake = ctypes.c_void_p(256)  # never touched: refused before any launch
    rc = lib.specdec_dpace_forward_noalloc(fake, fake, None, hi, B, V, 0.5, 0, hi, fake, None, fake,
                                           fake, None, None)
    assert rc == _lib.ERR_WORKSPACE, _lib.last_error()


def test_noalloc_argument_errors_come_before_the_size_check(cuda):
    lib = _lib.load()
    N, B, V = 1024, 32, 151936  # far too large for the array
    fake = ctypes.c_void_p(256)
    rc = lib.specdec_dpace_forward_noalloc(fake, fake, None, N, B, V, 1.5, 0, N, fake, None, fake, fake,
                                           None, None)
    assert rc == _lib.ERR_VALUE  # alpha outside [0, 1], as specdec_dpace_forward reports it
    rc = lib.specdec_dpace_forward_noalloc(fake, fake, None, N, B, V, 0.5, 7, N, fake, None, fake, fake,
                                           None, None)
    assert rc == _lib.ERR_VALUE  # unknown loss_type
    rc = lib.specdec_dpace_forward_noalloc(fake, fake, None, N, B, V, 0.5, 0, N, None, None, fake, fake,
                                           None, None)
    assert rc == _lib.ERR_ARGUMENT  # null loss output
    rc = lib.specdec_dpace_forward_noalloc(fake, fake, None, N, B, V, 0.5, 0, N - 1, fake, None, fake, fake,
                                           None, None)
    assert rc == _lib.ERR_ARGUMENT  # n_global < N


def test_noalloc_recovers_after_an_expired_wait(cuda):
    """A call whose bounded wait ran out reports it (status 5, NaN loss); the
    next calls on the shared array are exact again with no clearing by the
    caller (each call clears the array's counter region on its stream)."""
    lib = _lib.load()
    x, t, m = _batch(64, 16, 40000, 14, cuda)
    try:
        _lib.check(lib.specdec_test_withhold_stage(1), "specdec_test_withhold_stage")
        loss, _, _, _ = _noalloc(lib, x, t, m, expect_status=_lib.ERR_CUDA)
    finally:
        lib.specdec_test_withhold_stage(0)
    assert bool(torch.isnan(loss))
    for call in range(2):
        _check_against_allocating(lib, x, t, m, f"after timeout, call {call}")


def test_noalloc_refuses_oversized_problem(cuda):
    lib = _lib.load()
    N, B, V = 1024, 32, 151936  # scratch far above the built-in 4 MiB
    fake = ctypes.c_void_p(256)  # never touched: the size check comes first
    rc = lib.specdec_dpace_forward_noalloc(fake, fake, None, N, B, V, 0.5, 0, N, fake, None, fake,
                                           fake, None, None)
    assert rc == _lib.ERR_WORKSPACE
    assert "no-allocation entry point holds" in _lib.last_error()
