"""The no-allocation D-PACE forward (specdec_dpace_forward_noalloc).

That entry point exists for callers that cannot allocate device memory (a
plugin host that passes only input and output buffers, or a process whose
device memory is all held by its own pool): it keeps its scratch in a fixed
array inside libspecdec.so instead of asking for a workspace. This test calls
it through the C ABI twice in a row, on two different batches, and checks each
result against the allocating entry point, specdec_dpace_forward, on the same
inputs: loss within 1e-5 relative, per-row lse and scale within 1e-6
absolute. It also checks that a problem too large for the built-in array is
refused up front. The file is named to be collected last.
"""
import ctypes

import pytest
import torch

from specdec import _lib, ops

pytestmark = pytest.mark.gpu

LOSS_RTOL = 1e-5
ROW_ATOL = 1e-6


def _batch(N, B, V, seed, dev):
    g = torch.Generator(device=dev).manual_seed(seed)
    x = torch.randn(N, B, V, device=dev, generator=g) * 2.0
    t = torch.randint(0, V, (N, B), device=dev, generator=g)
    k = torch.randint(0, 5, (N, 1), device=dev, generator=g)
    m = (torch.arange(B, device=dev).view(1, B) >= k).float()
    return x, t, m


def _noalloc(lib, x, t, m, alpha=0.5, loss_type=0):
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
    assert int(status.item()) == _lib.OK
    return loss, loss_n, lse, scale


def test_noalloc_matches_allocating_forward(cuda):
    lib = _lib.load()
    for call, (N, B, V, seed) in enumerate([(16, 16, 128256, 11), (8, 32, 151936, 12)]):
        x, t, m = _batch(N, B, V, seed, cuda)
        want_loss, want_lse, want_scale, want_loss_n = ops.dpace_forward(x, t, m, 0.5, 0,
                                                                         want_loss_n=True)
        loss, loss_n, lse, scale = _noalloc(lib, x, t, m)
        w = float(want_loss)
        assert abs(float(loss) - w) <= LOSS_RTOL * abs(w), (call, float(loss), w)
        assert (lse - want_lse).abs().max().item() <= ROW_ATOL, call
        assert (scale - want_scale).abs().max().item() <= ROW_ATOL, call
        assert (loss_n - want_loss_n).abs().max().item() <= LOSS_RTOL * want_loss_n.abs().max().item()


def test_noalloc_refuses_oversized_problem(cuda):
    lib = _lib.load()
    N, B, V = 1024, 32, 151936  # scratch far above the built-in 4 MiB
    fake = ctypes.c_void_p(256)  # never touched: the size check comes first
    rc = lib.specdec_dpace_forward_noalloc(fake, fake, None, N, B, V, 0.5, 0, N, fake, None, fake,
                                           fake, None, None)
    assert rc == _lib.ERR_WORKSPACE
    assert "no-allocation entry point holds" in _lib.last_error()
