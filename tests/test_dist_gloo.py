"""Sequence sharding across ranks on CPU with the gloo backend (world size 2).

Checks the host logic of specdec.dist without a GPU: balanced contiguous
shards, the global loss equal on every rank and equal to the whole-batch
loss, local gradients equal to the whole-batch gradient's slice, and a rank
that fails before the loss reduction surfacing as an error on its peer (no
hang). The per-shard loss is the CPU oracle with the global divisor, the role
the CUDA kernels play on GPUs."""
import multiprocessing as mp
import os
import socket
import sys
import traceback
from datetime import timedelta

import numpy as np
import pytest
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _setup_paths():
    for p in (os.path.join(REPO, "cuda-spec-decode_b200"), REPO):
        if p not in sys.path:
            sys.path.insert(0, p)


def _worker(rank, world, port, mode, q):
    _setup_paths()
    import torch.distributed as dist

    from oracle import dpace as odp
    from specdec import dist as sd

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
        rng = np.random.default_rng(0)
        N, B, V = 7, 8, 64
        x = torch.from_numpy(rng.normal(0, 2, (N, B, V)).astype(np.float32))
        t = torch.from_numpy(rng.integers(0, V, (N, B)))
        m = torch.ones(N, B)
        m[:, :2] = 0.0
        lo, hi = sd.shard_range(N, rank, world)
        if mode == "fail" and rank == 1:
            raise RuntimeError("injected failure before the loss reduction")
        xs = x[lo:hi].clone().requires_grad_(True)
        partial = odp.dpace_loss_torch(xs, t[lo:hi], 0.5, m[lo:hi]) * ((hi - lo) / N)
        loss = sd.allreduce_loss(partial)
        loss.backward()
        xf = x.clone().requires_grad_(True)
        full = odp.dpace_loss_torch(xf, t, 0.5, m)
        full.backward()
        q.put((rank, "ok", float(loss.detach()), float(full.detach()),
               float((xs.grad - xf.grad[lo:hi]).abs().max()), (lo, hi)))
        dist.destroy_process_group()
    except Exception as e:  # reported to the parent, which decides pass/fail
        q.put((rank, "error", type(e).__name__, str(e)[:200], traceback.format_exc()[-400:], None))


def _run(mode, world=2, timeout=60):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    for _ in range(world):
        r = q.get(timeout=timeout)
        out[r[0]] = r
    for p in procs:
        p.join(timeout=timeout)
        if p.is_alive():
            p.kill()
    return out


def test_shard_range_is_balanced_and_covering():
    sys.path.insert(0, os.path.join(REPO, "cuda-spec-decode_b200"))
    from specdec.dist import shard_range

    for n in (0, 1, 7, 64, 512):
        for world in (1, 2, 3, 4, 8):
            spans = [shard_range(n, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            for (a, b), (c, d) in zip(spans, spans[1:]):
                assert b == c
            sizes = [b - a for a, b in spans]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_range(4, 2, 2)


def test_two_rank_loss_and_gradients():
    out = _run("ok")
    assert set(out) == {0, 1}
    for r in (0, 1):
        rank, status, loss, full, gdiff, span = out[r]
        assert status == "ok", out[r]
        assert abs(loss - full) <= 1e-6 * abs(full)
        assert gdiff <= 1e-7
    assert out[0][2] == out[1][2]  # identical global loss on every rank


def test_failed_rank_surfaces_as_error_on_peer():
    out = _run("fail")
    assert out[1][1] == "error" and "injected" in out[1][3]
    assert out[0][1] == "error", out[0]  # the peer's reduction errors out instead of hanging


def _grad_worker(rank, world, port, q):
    _setup_paths()
    import torch.distributed as dist

    from specdec.graphs import allreduce_grads

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
        torch.manual_seed(0)
        params = [torch.nn.Parameter(torch.randn(3, 5)), torch.nn.Parameter(torch.randn(7)),
                  torch.nn.Parameter(torch.randn(2, 2, 2))]
        g = torch.Generator().manual_seed(100 + rank)
        for p in params:
            p.grad = torch.randn(p.shape, generator=g)
        local = [p.grad.clone() for p in params]
        allreduce_grads(params)
        q.put((rank, [l.numpy() for l in local], [p.grad.numpy() for p in params]))
        dist.destroy_process_group()
    except Exception:
        q.put((rank, "error", traceback.format_exc()))


def test_allreduce_grads_averages_over_ranks():
    """specdec.graphs.allreduce_grads: every rank ends with the mean of the
    ranks' gradients, tensor by tensor, in the original shapes."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_grad_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict()
    for _ in range(2):
        r, a, b = q.get(timeout=60)
        assert a != "error", b
        res[r] = (a, b)
    for p in procs:
        p.join(timeout=30)
    mean = [(x + y) / 2 for x, y in zip(res[0][0], res[1][0])]
    for r in range(2):
        for m_, got in zip(mean, res[r][1]):
            assert got.shape == m_.shape
            np.testing.assert_allclose(got, m_, rtol=1e-6, atol=1e-7)
