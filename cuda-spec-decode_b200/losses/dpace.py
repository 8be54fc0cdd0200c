"""D-PACE loss on B200: drop-in for the reference's ``losses.dpace``.

Same entry points, argument names, defaults and exception types as
harvestingmoon/cuda-spec-decode losses/dpace.py:
  - dpace_loss        (dpace.py:234-243)  autograd-aware, returns a 0-d tensor
  - fused_dpace_loss  (dpace.py:190-195)  forward only; takes torch CUDA
                                          tensors (the reference took cupy)
  - _check            (dpace.py:157-173)  host-side validation
The math follows the torch oracle losses/dpace_ref.py:8-51:
    ce_j   = logsumexp(x_j) - x_j[target_j]
    q_j    = exp(-ce_j)
    sm_j   = (1 - alpha) q_j + alpha   if mask_j > 0 else 1
    P_j    = prod_{i<=j} sm_i;  S_j = sum_{k>=j} P_k [mask_k > 0]
    w_j    = {S_j, P_j, S_j / max(P_j, tiny)}[loss_type] * [mask_j > 0]
    loss   = sum_{n,j} w_j ce_j / N
    dL/dx  = (w_j / N) * (softmax(x_j) - onehot(target_j))     (w detached)
computed by the sm_100a kernels in libspecdec.so; there is no other path.

Beyond the reference (whose kernels take fp32 only, README.md:263): logits may
also be bfloat16. The kernels widen every element exactly and compute in
fp32, so the loss is the fp32 loss of the widened logits; the gradient is
returned in bfloat16 (rounded to nearest even), like the logits.
"""
from __future__ import annotations

import torch

from specdec import ops

_LOSS_TYPES = ops.DPACE_LOSS_TYPES


def _check(logits: torch.Tensor, targets: torch.Tensor, mask: torch.Tensor | None, alpha: float,
           loss_type: str) -> None:
    """Host checks in the reference's order (losses/dpace.py:157-170).

    The target range check (dpace.py:171-173) runs inside the forward kernel
    and is raised after it as ValueError.
    """
    assert logits.ndim == 3 and logits.dtype in ops.LOGIT_DTYPES, "logits must be float32 (or bfloat16) [N, B, V]"
    assert targets.shape == logits.shape[:2] and targets.dtype == torch.int64, \
        "targets must be int64 [N, B]"
    assert mask is None or (mask.shape == logits.shape[:2] and mask.dtype == torch.float32), \
        "position mask must be float32 [N, B]"
    N, B, V = logits.shape
    assert 1 <= B <= 32, "kernel configured for block_size <= 32"
    assert logits.is_contiguous() and targets.is_contiguous() \
        and (mask is None or mask.is_contiguous()), "inputs must be contiguous"
    if not 0.0 <= alpha <= 1.0:
        raise ValueError(f"dpace_alpha must be in [0, 1], got {alpha}")
    if loss_type not in _LOSS_TYPES:
        raise ValueError(f"unknown loss_type {loss_type!r}")
    if V == 0 and N * B > 0:
        raise ValueError(f"targets out of range [0, {V})")


def _prepare(logits, targets, position_mask):
    assert logits.is_cuda and logits.dtype in ops.LOGIT_DTYPES, "logits must be float32 (or bfloat16) cuda"
    assert targets.dtype == torch.int64, "targets must be int64"
    logits = logits.detach().contiguous()
    targets = targets.detach().contiguous()
    mask = None
    if position_mask is not None:
        mask = position_mask.detach().to(device=logits.device, dtype=torch.float32).contiguous()
    return logits, targets, mask


def _forward(logits, targets, mask, alpha, loss_type, n_global=None):
    """Returns (loss 0-d, lse [N,B], scale [N,B]); inputs already prepared."""
    _check(logits, targets, mask, alpha, loss_type)
    if logits.shape[0] == 0:
        nan = torch.full((), float("nan"), dtype=torch.float32, device=logits.device)
        empty = torch.zeros(logits.shape[:2], dtype=torch.float32, device=logits.device)
        return nan, empty, empty
    loss, lse, scale, _ = ops.dpace_forward(logits, targets, mask, alpha, _LOSS_TYPES[loss_type],
                                            n_global=n_global)
    return loss, lse, scale


def fused_dpace_loss(logits: torch.Tensor, targets: torch.Tensor, alpha: float = 0.5,
                     position_mask=None, loss_type: str = "dpace") -> torch.Tensor:
    """Forward-only D-PACE loss (eval). logits [N,B,V] float32 (or bfloat16) CUDA, targets [N,B] int64."""
    logits, targets, mask = _prepare(logits, targets, position_mask)
    return _forward(logits, targets, mask, alpha, loss_type)[0]


class DPACELoss(torch.autograd.Function):
    """Autograd glue (reference: losses/dpace.py:201-226). The weights are
    detached, so the gradient is one fused expression: (w_j/N)(softmax - onehot).

    Default (as the reference): the backward kernel runs in the autograd
    backward with the real dloss. With specdec.ops.set_fused_backward(True)
    the forward computes the gradient for dloss = 1 in the same call
    (specdec_dpace_forward_backward) and keeps it; the backward then only
    multiplies by dloss on the device, which is no pass at all when dloss is 1
    (loss.backward()). A second backward through the same graph
    (retain_graph) recomputes the gradient with the backward kernel."""

    @staticmethod
    def forward(ctx, logits, targets, alpha, position_mask, loss_type, n_global=None):
        x, t, mask = _prepare(logits, targets, position_mask)
        ctx.grad = None
        if ops.FUSED_BACKWARD and ctx.needs_input_grad[0] and x.numel():
            _check(x, t, mask, alpha, loss_type)
            loss, ctx.grad, lse, scale, _ = ops.dpace_forward_backward(
                x, t, mask, alpha, _LOSS_TYPES[loss_type], n_global=n_global)
        else:
            loss, lse, scale = _forward(x, t, mask, alpha, loss_type, n_global)
        ctx.save_for_backward(x, t, lse, scale)
        return loss

    @staticmethod
    def backward(ctx, dloss):
        x, t, lse, scale = ctx.saved_tensors
        grad = None
        if ctx.needs_input_grad[0]:
            if ctx.grad is not None:
                grad, ctx.grad = ctx.grad, None
                if dloss is not None:
                    ops.scale_inplace(grad, dloss)
            else:
                grad = ops.dpace_backward(x, t, lse, scale, dloss) if x.numel() else torch.zeros_like(x)
        return grad, None, None, None, None, None


def dpace_loss(logits, targets, alpha: float = 0.5, position_mask=None, loss_type: str = "dpace"):
    """D-PACE loss for torch tensors, with autograd.

    logits [N,B,V] float32 (or bfloat16) cuda, targets [N,B] int64, position_mask [N,B] bool/float or None.
    Returns sum(w*ce)/N as a 0-d float32 tensor.
    """
    return DPACELoss.apply(logits, targets, alpha, position_mask, loss_type)
