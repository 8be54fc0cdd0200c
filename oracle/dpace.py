"""D-PACE oracle (CPU). Test infrastructure only -- see oracle/__init__.py.

Restates harvestingmoon/cuda-spec-decode:
  losses/dpace_ref.py:8-51          d_pace_loss (torch): CE via F.cross_entropy,
                                    detached weights via cumprod and a reversed
                                    cumsum, loss = sum(ce * w) / N
  losses/tests/test_dpace.py:21-45  _naive_dpace_weight / oracle_loss (the
                                    specforge statement of the same weights)
The torch form reproduces the reference's float32 arithmetic op for op (torch
CPU cumprod/cumsum accumulate in double); the numpy form is an independent
float64 statement with the closed-form gradient, used to bound the error of
both.
"""
from __future__ import annotations

import numpy as np
import torch
import torch.nn.functional as F

LOSS_TYPES = ("dpace", "dpace-cumulative-confidence-only", "dpace-continuation-value-only")


def _validate(alpha: float, loss_type: str) -> None:
    # losses/dpace_ref.py:22-25
    if not 0.0 <= alpha <= 1.0:
        raise ValueError(f"dpace_alpha must be in [0, 1], got {alpha}")
    if loss_type not in LOSS_TYPES:
        raise ValueError(f"unknown loss_type {loss_type!r}")


def dpace_weights_torch(q: torch.Tensor, keep: torch.Tensor, alpha: float,
                        loss_type: str) -> torch.Tensor:
    """Detached D-PACE weights from q = exp(-ce) and a 0/1 keep mask.

    losses/dpace_ref.py:35-49: smooth = (1-a) q + a on kept slots, 1 elsewhere;
    P = cumprod(smooth); S = reversed cumsum of P * keep; w = S | P | S / P,
    times keep.
    """
    smooth = (1.0 - alpha) * q + alpha
    smooth = torch.where(keep > 0, smooth, torch.ones_like(smooth))
    prefix = torch.cumprod(smooth, dim=-1)
    if loss_type == "dpace-cumulative-confidence-only":
        w = prefix
    else:
        suffix = torch.flip(torch.cumsum(torch.flip(prefix * keep, dims=[-1]), dim=-1), dims=[-1])
        w = suffix if loss_type == "dpace" else suffix / prefix.clamp_min(torch.finfo(prefix.dtype).tiny)
    return w * keep


def dpace_loss_torch(logits: torch.Tensor, targets: torch.Tensor, alpha: float = 0.5,
                     position_mask: torch.Tensor | None = None,
                     loss_type: str = "dpace") -> torch.Tensor:
    """losses/dpace_ref.py:8-51 on any device; differentiable in logits."""
    _validate(alpha, loss_type)
    n, b, v = logits.shape
    keep = (torch.ones_like(targets, dtype=logits.dtype) if position_mask is None
            else (position_mask > 0).to(logits.dtype))
    ce = F.cross_entropy(logits.reshape(-1, v), targets.reshape(-1), reduction="none").view_as(targets)
    with torch.no_grad():
        w = dpace_weights_torch(torch.exp(-ce), keep, alpha, loss_type)
    return (ce * w).sum() / float(n)


def dpace_fwd_bwd_torch(logits: torch.Tensor, targets: torch.Tensor, alpha: float = 0.5,
                        position_mask: torch.Tensor | None = None,
                        loss_type: str = "dpace"):
    """(loss, dloss/dlogits) through torch autograd on the CPU, float32."""
    x = logits.detach().cpu().float().clone().requires_grad_(True)
    m = None if position_mask is None else position_mask.detach().cpu()
    loss = dpace_loss_torch(x, targets.detach().cpu(), alpha, m, loss_type)
    loss.backward()
    return loss.detach(), x.grad


def dpace_f64(logits: np.ndarray, targets: np.ndarray, alpha: float = 0.5,
              position_mask: np.ndarray | None = None, loss_type: str = "dpace"):
    """Float64 statement: returns (loss, grad, lse, weights)."""
    _validate(alpha, loss_type)
    x = np.asarray(logits, dtype=np.float64)
    n, b, v = x.shape
    t = np.asarray(targets, dtype=np.int64)
    keep = np.ones((n, b)) if position_mask is None else (np.asarray(position_mask) > 0).astype(np.float64)
    mx = x.max(axis=-1, keepdims=True)
    ex = np.exp(x - mx)
    z = ex.sum(axis=-1, keepdims=True)
    lse = (mx + np.log(z))[..., 0]
    xt = np.take_along_axis(x, t[..., None], axis=-1)[..., 0]
    ce = lse - xt
    smooth = np.where(keep > 0, (1.0 - alpha) * np.exp(-ce) + alpha, 1.0)
    P = np.cumprod(smooth, axis=-1)
    S = np.cumsum((P * keep)[:, ::-1], axis=-1)[:, ::-1]
    if loss_type == "dpace":
        w = S
    elif loss_type == "dpace-cumulative-confidence-only":
        w = P
    else:
        w = S / np.maximum(P, np.finfo(np.float32).tiny)
    w = w * keep
    loss = float((ce * w).sum() / n)
    g = ex / z
    np.put_along_axis(g, t[..., None], np.take_along_axis(g, t[..., None], axis=-1) - 1.0, axis=-1)
    g *= (w / n)[..., None]
    return loss, g, lse, w
