"""specdec.dist on one GPU with a single-rank NCCL group: the sharded losses
equal the unsharded ones, and LossReducer (loss all_reduce on a side stream,
overlapping the backward) delivers the global loss after wait()."""
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def nccl_group(cuda):
    import torch.distributed as dist

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    store = dist.TCPStore("127.0.0.1", port, 1, True)
    dist.init_process_group("nccl", store=store, rank=0, world_size=1, device_id=cuda)
    yield
    torch.cuda.synchronize()
    dist.destroy_process_group()


def _inputs(seed, N=4, B=8, V=3001):
    rng = np.random.default_rng(seed)
    x = torch.from_numpy(rng.normal(scale=2.0, size=(N, B, V)).astype(np.float32)).cuda()
    t = torch.from_numpy(rng.integers(0, V, (N, B))).cuda()
    return x, t


def test_sharded_losses_match_unsharded(nccl_group):
    from losses import dpace_loss
    from models.dflash import dflash_loss
    from specdec.dist import sharded_dflash_loss, sharded_dpace_loss

    x, t = _inputs(0)
    a = x.clone().requires_grad_(True)
    b = x.clone().requires_grad_(True)
    la = dpace_loss(a, t)
    lb = sharded_dpace_loss(b, t)
    la.backward()
    lb.backward()
    assert float(la) == float(lb)
    assert torch.equal(a.grad, b.grad)
    y = x + 1.0
    a = x.clone().requires_grad_(True)
    b = x.clone().requires_grad_(True)
    la = dflash_loss(a, y)
    lb = sharded_dflash_loss(b, y)
    la.backward()
    lb.backward()
    assert float(la) == float(lb)
    assert torch.equal(a.grad, b.grad)


def test_loss_reducer_overlaps_backward_and_delivers_the_sum(nccl_group):
    from specdec import ops
    from specdec.dist import LossReducer

    x, t = _inputs(1)
    red = LossReducer(x.device)
    totals = []
    for _ in range(3):
        loss, lse, scale, _ = ops.dpace_forward(x, t, None, 0.5, 0)
        total = red.start(loss)
        g = ops.dpace_backward(x, t, lse, scale, None)
        red.wait()
        totals.append(float(total))
        assert float(total) == float(loss)  # one rank: the sum is the partial
        assert bool(torch.isfinite(g).all())
    assert totals[0] == totals[1] == totals[2]
