"""The DFlash drafter's own layers on this library's kernels.

- ``rms_norm(x, weight, eps)``: RMSNorm over the last dimension (fp32 or bf16
  input, fp32 weight), forward and backward kernels of libspecdec.so; the
  weight gradient is reduced in a fixed order (bitwise repeatable).
- ``dflash_attention(q, k, v, n_ctx, scale)``: multi-head attention under the
  DFlash mask (query t < n_ctx sees keys j <= t, later queries see every key)
  for bf16 q, k, v of shape [B, T, H, 64] -- the projections' own layout.
  Forward and backward run on the tensor cores (tcgen05: products in tensor
  memory); the backward recomputes the probabilities from the forward's
  log-sum-exp and accumulates dq, dk, dv in a fixed order.

Reference: models/dflash/model.py:25-53 (DFlashAttention), :56-73 (the
pre-norm layer, torch.nn.RMSNorm), :123-131 (the mask).
``ENABLED`` switches the drafter modules between these kernels and plain
torch (for comparison); the kernels run only on CUDA tensors of the shapes and
dtypes above.
"""
from __future__ import annotations

import torch

from . import _lib

ENABLED = True


def set_enabled(enabled: bool) -> None:
    global ENABLED
    ENABLED = bool(enabled)


_DTYPES = {torch.float32: 0, torch.bfloat16: 1}


def _stream(t: torch.Tensor) -> int:
    return _lib.stream_handle(t.device)


def _status(dev: torch.device) -> int:
    """The stream's sticky drafter status word: the attention kernels set it
    when a bounded wait expires (their failed rows are then NaN); the next
    synchronising check (specdec.ops.check_backward, a validating D-PACE
    forward, GraphedStep.check) raises RuntimeError and clears it."""
    return _lib.status_words(dev)[_lib.STATUS_DRAFTER:].data_ptr()


class _RMSNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, eps):
        lib = _lib.load()
        D = x.shape[-1]
        x2 = x.contiguous().view(-1, D)
        w = weight.detach().float().contiguous()
        y = torch.empty_like(x2)
        rstd = torch.empty(x2.shape[0], dtype=torch.float32, device=x.device)
        with _lib.on_device(x.device):
            _lib.check(lib.specdec_rmsnorm_forward(x2.data_ptr(), w.data_ptr(), y.data_ptr(), rstd.data_ptr(),
                                                   x2.shape[0], D, float(eps), _DTYPES[x.dtype], _stream(x)),
                       "specdec_rmsnorm_forward")
        ctx.save_for_backward(x2, w, rstd)
        ctx.wdtype = weight.dtype
        return y.view(x.shape)

    @staticmethod
    def backward(ctx, dy):
        lib = _lib.load()
        x2, w, rstd = ctx.saved_tensors
        D = x2.shape[-1]
        dy2 = dy.to(x2.dtype).contiguous().view(-1, D)
        dx = torch.empty_like(x2)
        dw = torch.empty(D, dtype=torch.float32, device=x2.device)
        with _lib.on_device(x2.device):
            ws_bytes = lib.specdec_rmsnorm_workspace_bytes(x2.shape[0], D, x2.device.index)
            ws = torch.empty(ws_bytes, dtype=torch.uint8, device=x2.device)
            _lib.check(lib.specdec_rmsnorm_backward(x2.data_ptr(), w.data_ptr(), rstd.data_ptr(), dy2.data_ptr(),
                                                    dx.data_ptr(), dw.data_ptr(), x2.shape[0], D, _DTYPES[x2.dtype],
                                                    ws.data_ptr(), ws_bytes, _stream(x2)),
                       "specdec_rmsnorm_backward")
        return dx.view(dy.shape), dw.to(ctx.wdtype), None


def rms_norm_supported(x: torch.Tensor, weight: torch.Tensor | None) -> bool:
    return (ENABLED and x.is_cuda and x.dtype in _DTYPES and weight is not None
            and weight.dtype == torch.float32 and x.shape[-1] == weight.numel() and x.numel() > 0)


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float | None = None) -> torch.Tensor:
    """RMSNorm of the last dimension; eps None = finfo(x.dtype).eps (torch's default)."""
    e = torch.finfo(x.dtype).eps if eps is None else float(eps)
    return _RMSNorm.apply(x, weight, e)


class _DFlashAttention(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, n_ctx, scale):
        lib = _lib.load()
        B, T, H, Dh = q.shape
        q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
        o = torch.empty_like(q)
        lse = torch.empty(B, H, T, dtype=torch.float32, device=q.device)
        with _lib.on_device(q.device):
            _lib.check(lib.specdec_dflash_attention_forward(
                q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), lse.data_ptr(), B, T, H, Dh,
                int(n_ctx), float(scale), _status(q.device), _stream(q)), "specdec_dflash_attention_forward")
        ctx.save_for_backward(q, k, v, o, lse)
        ctx.n_ctx, ctx.scale = int(n_ctx), float(scale)
        return o

    @staticmethod
    def backward(ctx, do):
        lib = _lib.load()
        q, k, v, o, lse = ctx.saved_tensors
        B, T, H, Dh = q.shape
        do = do.to(q.dtype).contiguous()
        dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
        with _lib.on_device(q.device):
            ws_bytes = lib.specdec_dflash_attention_workspace_bytes(B, T, H)
            ws = torch.empty(ws_bytes, dtype=torch.uint8, device=q.device)
            _lib.check(lib.specdec_dflash_attention_backward(
                q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), lse.data_ptr(), do.data_ptr(),
                dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), B, T, H, Dh, ctx.n_ctx, ctx.scale, _status(q.device),
                ws.data_ptr(), ws_bytes, _stream(q)), "specdec_dflash_attention_backward")
        return dq, dk, dv, None, None


def attention_supported(q: torch.Tensor) -> bool:
    return (ENABLED and q.is_cuda and q.dtype == torch.bfloat16 and q.dim() == 4 and q.shape[-1] == 64
            and q.shape[1] <= 65535 * 128)


def dflash_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, n_ctx: int,
                     scale: float | None = None) -> torch.Tensor:
    """Attention under the DFlash mask; q, k, v bf16 [B, T, H, 64] -> o [B, T, H, 64]."""
    s = q.shape[-1] ** -0.5 if scale is None else float(scale)
    return _DFlashAttention.apply(q, k, v, n_ctx, s)
