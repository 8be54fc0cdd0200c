"""N-sharded losses over torch.distributed.

Every D-PACE sequence and every DFlash row is independent of the other
sequences, so a batch of N_global sequences splits into contiguous shards of
whole sequences, one per rank, with no exchange of logits or gradients. Each
rank computes its partial loss with the global divisor,
    partial_r = sum_{n in shard r} loss_n / N_global,
and one 4-byte all_reduce(SUM) gives every rank the global loss. The gradient
of the global loss with respect to a rank's own logits is exactly the
gradient of its partial (the other ranks' terms do not depend on them), so the
backward runs locally with dloss = 1 and no collective.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def shard_range(n_total: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous, balanced [start, stop) of n_total items for `rank`; the first
    n_total % world ranks take one extra item."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank/world {rank}/{world}")
    base, extra = divmod(int(n_total), world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def allreduce_loss(partial: torch.Tensor, group=None) -> torch.Tensor:
    """Global sum of per-rank partial losses, identical on every rank; the
    gradient flows only into this rank's `partial`, with weight 1."""
    total = partial.detach().clone()
    dist.all_reduce(total, op=dist.ReduceOp.SUM, group=group)
    return partial + (total - partial.detach())


class LossReducer:
    """The 4-byte loss all_reduce on a side stream, off the compute stream's
    critical path.

    The backward needs only this rank's scale (dloss = 1 for the partial), never
    the global loss, so the collective can run while the backward kernel
    streams. start(partial) after the forward returns the tensor that will hold
    the global loss; wait() makes the current stream wait for it (call it
    before anything reads that tensor, e.g. at the end of the step). Every
    rank must call start/wait in the same order, like any collective.
    """

    def __init__(self, device, group=None):
        self.device = torch.device(device)
        self.stream = torch.cuda.Stream(device=self.device)
        self.group = group

    def start(self, partial: torch.Tensor) -> torch.Tensor:
        total = partial.detach().clone()
        self.stream.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(self.stream):
            dist.all_reduce(total, op=dist.ReduceOp.SUM, group=self.group)
        total.record_stream(self.stream)
        return total

    def wait(self) -> None:
        torch.cuda.current_stream(self.device).wait_stream(self.stream)


def sharded_dpace_loss(logits, targets, alpha: float = 0.5, position_mask=None,
                       loss_type: str = "dpace", n_global: int | None = None, group=None):
    """dpace_loss over a batch split by sequence across ranks. `logits` etc. are
    this rank's shard; n_global is the total number of sequences (summed over
    ranks with one extra all_reduce when None)."""
    from losses.dpace import DPACELoss

    if n_global is None:
        n = torch.tensor([logits.shape[0]], dtype=torch.int64, device=logits.device)
        dist.all_reduce(n, group=group)
        n_global = int(n.item())
    partial = DPACELoss.apply(logits, targets, alpha, position_mask, loss_type, n_global)
    return allreduce_loss(partial, group)


def sharded_dflash_loss(logits, target_logits, loss_mask=None, gamma: float = 4.0,
                        sample_from_anchor: bool = False, kind: str = "kl",
                        block_size: int | None = None, n_global: int | None = None, group=None):
    """dflash_loss over a batch split by sequence across ranks (see sharded_dpace_loss)."""
    from models.dflash.loss import DFlashLoss

    if n_global is None:
        n = torch.tensor([logits.shape[0]], dtype=torch.int64, device=logits.device)
        dist.all_reduce(n, group=group)
        n_global = int(n.item())
    partial = DFlashLoss.apply(logits, target_logits, loss_mask, gamma, sample_from_anchor, kind,
                               block_size, n_global)
    return allreduce_loss(partial, group)
