"""A whole training step -- forward, objective, backward, gradient clipping and
the optimizer update -- captured once as a CUDA graph and replayed.

The drafter's step (models/dflash/model.py:152-170 through the reference
pipeline's loop, pipeline.py:85-117) is a few hundred small launches; run
eagerly from Python, the GPU waits on the host between many of them. Replayed
as one graph the launches go out back to back.

    step = GraphedStep(fn, feats, tokens)     # fn(feats, tokens) -> loss
    loss = step()                             # replay on the resident inputs
    loss = step(new_feats, new_tokens)        # copy new inputs in, then replay

Requirements on ``fn``, as for any CUDA-graph capture:
- no host synchronisation (the library's D-PACE target-range read-back is
  skipped while a stream is capturing; ``check()`` reads the captured
  forward's status word after a replay instead);
- optimizers built with ``capturable=True`` (for AdamW also ``fused=True``:
  the capturable foreach form is dozens of elementwise launches per step);
  autocast with ``cache_enabled=False``;
- gradients are set to None before capture (done here), so the captured
  backward writes them fresh on every replay.
Warm-up calls and the capture run on one side stream, so the library's
per-stream workspace and status words exist before capture starts. Replays of
one GraphedStep must not overlap (they share that workspace).

Data parallel over N GPUs: call ``allreduce_grads(params)`` after
``loss.backward()`` inside ``fn`` (one NCCL all-reduce of the flat gradient,
captured with the step) on a model that is not wrapped in DDP; every rank
builds, warms up, captures and replays the same step. Release the
GraphedStep before ``destroy_process_group``.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from . import _lib


def allreduce_grads(params, group=None) -> None:
    """Averages the parameters' gradients over the ranks of `group` with one
    all-reduce of a flat buffer (one NCCL call instead of one per tensor).
    Nothing in it synchronises with the host, so it captures inside a CUDA
    graph with the rest of the step: every rank replays the same collective.
    Every rank must pass the same parameters, with gradients."""
    grads = [p.grad for p in params if p.grad is not None]
    if not grads:
        return
    flat = torch.cat([g.reshape(-1) for g in grads])
    dist.all_reduce(flat, group=group)
    flat.div_(dist.get_world_size(group))
    for g, v in zip(grads, torch._utils._unflatten_dense_tensors(flat, grads)):
        g.copy_(v)


class GraphedStep:
    def __init__(self, fn, *example_inputs: torch.Tensor, warmup: int = 3, optimizers=()):
        self.fn = fn
        self.static = [t.detach().clone() for t in example_inputs]
        dev = self.static[0].device if self.static else torch.device("cuda", torch.cuda.current_device())
        self.device = dev
        self.stream = torch.cuda.Stream(dev)
        self.stream.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(self.stream):
            for _ in range(warmup):
                fn(*self.static)
        torch.cuda.current_stream(dev).wait_stream(self.stream)
        torch.cuda.synchronize(dev)
        for opt in optimizers:
            opt.zero_grad(set_to_none=True)
        with torch.cuda.stream(self.stream):
            self.status = _lib.status_words(dev)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=self.stream):
            self.out = fn(*self.static)
        torch.cuda.synchronize(dev)

    def __call__(self, *inputs: torch.Tensor):
        if inputs:
            if len(inputs) != len(self.static):
                raise ValueError(f"expected {len(self.static)} inputs, got {len(inputs)}")
            for st, x in zip(self.static, inputs):
                st.copy_(x, non_blocking=True)
        self.graph.replay()
        return self.out

    def check(self) -> None:
        """Synchronises and raises as the eager calls would have: ValueError
        for a D-PACE target outside [0, V) in the last replay, RuntimeError
        for an expired bounded wait in any captured kernel."""
        st = self.status[:4].tolist()
        if st[_lib.STATUS_DPACE_BWD] or st[_lib.STATUS_DFLASH_BWD]:
            self.status[1:3].zero_()
            raise RuntimeError("a backward kernel of the captured step had a bounded wait expire")
        if st[_lib.STATUS_DRAFTER]:
            self.status[3:4].zero_()
            raise RuntimeError("an attention kernel of the captured step had a bounded wait expire")
        if st[_lib.STATUS_DPACE_FWD] == _lib.ERR_TARGET_RANGE:
            raise ValueError("targets out of range")
        if st[_lib.STATUS_DPACE_FWD] == _lib.ERR_CUDA:
            raise RuntimeError("a forward kernel of the captured step had a bounded wait expire")
