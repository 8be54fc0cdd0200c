"""DFlash objective oracle (CPU). Test infrastructure only -- see oracle/__init__.py.

Restates the speculators objective that harvestingmoon/cuda-spec-decode
embeds as its oracle in models/dflash/tests/test_loss.py:21-49
(dflash_loss_decay, kl_div_loss, ce_loss, loss_function, EPS = 1e-5), with the
decay position j % block_size of test_loss.py:62. The torch form reproduces
the oracle's float32 arithmetic op for op; the numpy form is an independent
float64 statement with the closed-form gradient.
"""
from __future__ import annotations

import numpy as np
import torch
import torch.nn.functional as F

EPS = 1e-5
KINDS = ("kl", "ce")


def slot_decay(pos: torch.Tensor, gamma: float, sample_from_anchor: bool) -> torch.Tensor:
    """test_loss.py:23-27: exp(-pos/g) with the anchor scored, else
    exp(-max(pos-1, 0)/g) with slot 0 weighted 0."""
    if sample_from_anchor:
        return torch.exp(-pos / gamma)
    d = torch.exp(-((pos - 1).clamp(min=0)) / gamma)
    return d * (pos != 0).to(d.dtype)


def kl_rows(logits: torch.Tensor, target_logits: torch.Tensor) -> torch.Tensor:
    """test_loss.py:30-33: KL(softmax(target) || softmax(logits)) per row."""
    log_q = F.log_softmax(logits, dim=-1, dtype=torch.float32)
    p = F.softmax(target_logits, dim=-1, dtype=torch.float32)
    return F.kl_div(log_q, p, reduction="none", log_target=False).sum(dim=-1)


def ce_rows(logits: torch.Tensor, target_logits: torch.Tensor) -> torch.Tensor:
    """test_loss.py:36-40: CE of logits against argmax(target_logits) per row."""
    v = logits.shape[-1]
    ids = torch.argmax(target_logits, dim=-1)
    return F.cross_entropy(logits.reshape(-1, v), ids.reshape(-1), reduction="none",
                           ignore_index=-100).reshape(ids.shape)


def dflash_loss_torch(logits: torch.Tensor, target_logits: torch.Tensor,
                      loss_mask: torch.Tensor | None = None, gamma: float = 4.0,
                      sample_from_anchor: bool = False, kind: str = "kl",
                      block_size: int | None = None) -> torch.Tensor:
    """test_loss.py:43-49 with pos = arange(B) % block_size; differentiable in logits."""
    n, b, v = logits.shape
    bs = b if block_size is None else block_size
    el = (kl_rows if kind == "kl" else ce_rows)(logits, target_logits)
    m = (torch.ones((n, b), dtype=el.dtype, device=el.device) if loss_mask is None
         else loss_mask.to(el.dtype))
    pos = (torch.arange(b, device=el.device).view(1, -1) % bs).to(el.dtype)
    el = el * m
    el = el * slot_decay(pos, gamma, sample_from_anchor)
    return (el.sum(dim=1) / (m.sum(dim=1) + EPS)).mean()


def dflash_fwd_bwd_torch(logits, target_logits, loss_mask=None, gamma=4.0,
                         sample_from_anchor=False, kind="kl", block_size=None):
    """(loss, dloss/dlogits) through torch autograd on the CPU, float32."""
    x = logits.detach().cpu().float().clone().requires_grad_(True)
    xt = target_logits.detach().cpu().float()
    m = None if loss_mask is None else loss_mask.detach().cpu()
    loss = dflash_loss_torch(x, xt, m, gamma, sample_from_anchor, kind, block_size)
    loss.backward()
    return loss.detach(), x.grad


def dflash_f64(logits: np.ndarray, target_logits: np.ndarray, loss_mask=None, gamma=4.0,
               sample_from_anchor=False, kind="kl", block_size=None):
    """Float64 statement: returns (loss, grad, per-row weight)."""
    x = np.asarray(logits, dtype=np.float64)
    y = np.asarray(target_logits, dtype=np.float64)
    n, b, v = x.shape
    bs = b if block_size is None else block_size
    m = np.ones((n, b)) if loss_mask is None else np.asarray(loss_mask, dtype=np.float64)
    pos = (np.arange(b) % bs).astype(np.float64)
    if sample_from_anchor:
        d = np.exp(-pos / gamma)
    else:
        d = np.exp(-np.maximum(pos - 1, 0) / gamma) * (pos != 0)
    lq = x - x.max(-1, keepdims=True)
    lq = lq - np.log(np.exp(lq).sum(-1, keepdims=True))
    q = np.exp(lq)
    if kind == "kl":
        lp = y - y.max(-1, keepdims=True)
        lp = lp - np.log(np.exp(lp).sum(-1, keepdims=True))
        p = np.exp(lp)
        el = (p * (lp - lq)).sum(-1)
        target_dist = p
    else:
        ids = np.argmax(y, axis=-1)
        el = -np.take_along_axis(lq, ids[..., None], axis=-1)[..., 0]
        target_dist = np.zeros_like(q)
        np.put_along_axis(target_dist, ids[..., None], 1.0, axis=-1)
    w = m * d[None, :] / (m.sum(1, keepdims=True) + EPS)
    loss = float((w * el).sum() / n)
    g = (w / n)[..., None] * (q - target_dist)
    return loss, g, w
