"""DFlash objective on B200: drop-in for the reference's ``models.dflash.loss``.

Same entry points, argument names, defaults and exception types as
harvestingmoon/cuda-spec-decode models/dflash/loss.py:
  - dflash_loss        (loss.py:277-289)  autograd-aware, returns a 0-d tensor
  - fused_dflash_loss  (loss.py:215-224)  forward only (torch CUDA tensors)
  - dflash_objective   (loss.py:227-233)  binds verifier logits for the
                                          compute_loss(loss_fn=...) hook
  - _check             (loss.py:178-191)  host-side validation
The math follows the speculators oracle embedded in
models/dflash/tests/test_loss.py:21-49:
    el_j  = KL(softmax(target_j) || softmax(logits_j))   or   CE(logits_j, argmax target_j)
    pos_j = j % block_size
    d_j   = exp(-pos_j/gamma)                       if sample_from_anchor
          = exp(-(pos_j-1)/gamma) * [pos_j != 0]    otherwise
    loss  = mean_n( sum_j mask_j d_j el_j / (sum_j mask_j + 1e-5) )
    dL/dlogits = (mask_j d_j / denom_n / N) * (softmax(logits_j) - softmax(target_j) | onehot)
The decay index is j % block_size as in the oracle (test_loss.py:62); the
reference kernel indexes (n*B + j) % block_size (loss.py:115-116), which
differs only when B is not a multiple of block_size.

Beyond the reference (fp32 only, README.md:263): logits and target_logits may
also be bfloat16. The kernels widen every element exactly and compute in fp32;
the gradient comes back in the logits' dtype (bf16 rounded to nearest even).
When the two dtypes differ, the bf16 one is widened to fp32 first (exact).
"""
from __future__ import annotations

import torch

from specdec import ops

_KINDS = ops.DFLASH_KINDS


def _check(logits, target_logits, mask, gamma, kind, block_size) -> None:
    """Host checks in the reference's order (models/dflash/loss.py:178-191)."""
    assert logits.ndim == 3 and logits.dtype in ops.LOGIT_DTYPES, "logits must be float32 (or bfloat16) [N, B, V]"
    assert target_logits.shape == logits.shape and target_logits.dtype == logits.dtype, \
        "target_logits must be [N, B, V] of the logits' dtype"
    assert mask is None or (mask.shape == logits.shape[:2] and mask.dtype == torch.float32), \
        "loss_mask must be float32 [N, B]"
    N, B, V = logits.shape
    assert block_size is None or 1 <= block_size <= B, "block_size must be in [1, B]"
    assert logits.is_contiguous() and target_logits.is_contiguous() \
        and (mask is None or mask.is_contiguous()), "inputs must be contiguous"
    if not gamma > 0:
        raise ValueError(f"gamma must be > 0, got {gamma}")
    if kind not in _KINDS:
        raise ValueError(f"unknown loss kind {kind!r}, expected one of {sorted(_KINDS)}")


def _prepare(logits, target_logits, loss_mask):
    assert logits.is_cuda and logits.dtype in ops.LOGIT_DTYPES, "logits must be float32 (or bfloat16) cuda"
    assert target_logits.shape == logits.shape, "target_logits must match logits' shape"
    assert target_logits.dtype in ops.LOGIT_DTYPES, "target_logits must be float32 (or bfloat16)"
    logits = logits.detach()
    target_logits = target_logits.detach().to(logits.device)
    if target_logits.dtype != logits.dtype:  # mixed: widen the bf16 one (exact)
        logits, target_logits = logits.float(), target_logits.float()
    logits = logits.contiguous()
    target_logits = target_logits.contiguous()
    mask = None
    if loss_mask is not None:
        mask = loss_mask.detach().to(device=logits.device, dtype=torch.float32).contiguous()
    return logits, target_logits, mask


def _forward(logits, target_logits, mask, gamma, sample_from_anchor, kind, block_size,
             n_global=None):
    """Returns (loss 0-d, loss_rows [N,B], scale [N,B], (logzq, logzp, target_id))."""
    _check(logits, target_logits, mask, gamma, kind, block_size)
    N, B, V = logits.shape
    bs = B if block_size is None else int(block_size)
    loss, rows, scale, lzq, lzp, tgt = ops.dflash_forward(
        logits, target_logits, mask, gamma, sample_from_anchor, _KINDS[kind], bs, n_global)
    return loss, rows, scale, (lzq, lzp, tgt)


def fused_dflash_loss(logits, target_logits, loss_mask=None, gamma: float = 4.0,
                      sample_from_anchor: bool = False, kind: str = "kl",
                      block_size: int | None = None) -> torch.Tensor:
    """Forward-only DFlash loss (eval). logits/target_logits [N,B,V] float32 (or bfloat16) CUDA."""
    x, xt, mask = _prepare(logits, target_logits, loss_mask)
    return _forward(x, xt, mask, gamma, sample_from_anchor, kind, block_size)[0]


def dflash_objective(target_logits, **kwargs):
    """Bind the verifier logits so the objective fits the (logits, targets) hook.

    ``DFlashSpeculator.compute_loss(..., loss_fn=...)`` calls
    ``loss_fn(logits, targets)``; this objective needs the verifier's logits
    rather than token ids (reference: models/dflash/loss.py:227-233).
    """
    return lambda logits, _targets: dflash_loss(logits, target_logits, **kwargs)


class DFlashLoss(torch.autograd.Function):
    """Autograd glue (reference: models/dflash/loss.py:239-269). The verifier
    logits get no gradient."""

    @staticmethod
    def forward(ctx, logits, target_logits, loss_mask, gamma, sample_from_anchor, kind,
                block_size, n_global=None):
        x, xt, mask = _prepare(logits, target_logits, loss_mask)
        loss, _, scale, (lzq, lzp, tgt) = _forward(x, xt, mask, gamma, sample_from_anchor, kind,
                                                   block_size, n_global)
        ctx.kind = _KINDS[kind]
        ctx.save_for_backward(x, xt if ctx.kind == 0 else None, scale, lzq, lzp, tgt)
        return loss

    @staticmethod
    def backward(ctx, dloss):
        x, xt, scale, lzq, lzp, tgt = ctx.saved_tensors
        grad = None
        if ctx.needs_input_grad[0]:
            grad = ops.dflash_backward(x, xt, scale, lzq, lzp, tgt, dloss, ctx.kind)
        return grad, None, None, None, None, None, None, None


def dflash_loss(logits, target_logits, loss_mask=None, gamma: float = 4.0,
                sample_from_anchor: bool = False, kind: str = "kl",
                block_size: int | None = None):
    """DFlash loss for torch tensors, with autograd.

    logits / target_logits: [N,B,V] float32 (or bfloat16) cuda. loss_mask: [N,B] bool/float or None.
    kind="kl" (speculators default) or "ce" (hard argmax(target) labels).
    """
    return DFlashLoss.apply(logits, target_logits, loss_mask, gamma, sample_from_anchor, kind,
                            block_size)
