"""Tensor-level wrappers over the C ABI: allocate outputs with torch, pass raw
pointers and the current CUDA stream, map status codes to exceptions.

Shape/dtype validation that mirrors the reference's host checks lives in the
reference-facing modules (losses.dpace, models.dflash.loss); these wrappers
assume validated, contiguous CUDA inputs.
"""
from __future__ import annotations

import torch

from . import _lib

DPACE_LOSS_TYPES = {
    "dpace": 0,
    "dpace-cumulative-confidence-only": 1,
    "dpace-continuation-value-only": 2,
}
DFLASH_KINDS = {"kl": 0, "ce": 1}

# When True (default, the reference's behaviour) the D-PACE forward raises
# ValueError for target ids outside [0, V), which costs one 4-byte
# device-to-host read per call. The kernel never reads out of bounds either
# way; with validation off an out-of-range id contributes ce = 0.
VALIDATE_TARGETS = True


def set_target_validation(enabled: bool) -> None:
    global VALIDATE_TARGETS
    VALIDATE_TARGETS = bool(enabled)


# When True the autograd path of D-PACE computes the gradient in its forward
# with specdec_dpace_forward_backward (the forward and backward kernels in one
# call, dloss = 1; the backward then only applies dloss, with no pass at all
# when dloss is 1). False (default): the backward kernel runs in the autograd
# backward with the real dloss, as in the reference.
FUSED_BACKWARD = False


def set_fused_backward(enabled: bool) -> None:
    global FUSED_BACKWARD
    FUSED_BACKWARD = bool(enabled)


# Element types of the logits the kernels take; the gradient has the logits'
# type. bf16 calls go to the *_bf16 entry points (fp32 arithmetic inside).
LOGIT_DTYPES = (torch.float32, torch.bfloat16)


def _entry(lib, name: str, t: torch.Tensor):
    return getattr(lib, name + "_bf16") if t.dtype == torch.bfloat16 else getattr(lib, name)


def _aligned(t: torch.Tensor | None) -> torch.Tensor | None:
    """bf16 tensors must start on a 16-byte boundary (the bulk copies need it);
    a view that does not is copied once."""
    if t is None or t.dtype != torch.bfloat16 or t.data_ptr() % 16 == 0:
        return t
    return t.clone()


_ATTN_TIMEOUT_MSG = ("an earlier drafter attention launch on this stream had a bounded wait expire; the rows "
                     "of its outputs that the failed part owned hold NaN")
_BWD_TIMEOUT_MSG = ("an earlier backward launch on this stream had a bounded wait expire; the blocks of "
                    "its gradient that the failed part left unfinished hold NaN")


def _capturing() -> bool:
    """True while the current stream is being captured into a CUDA graph: no
    read-back then (the status word stays on the device; see
    specdec.graphs.GraphedStep.check)."""
    return torch.cuda.is_current_stream_capturing()


def _read_status(dev: torch.device, what: str, V: int) -> None:
    """One device-to-host read of this stream's status words, after a D-PACE
    forward: raises ValueError for an out-of-range target (the reference's
    check), RuntimeError for an expired wait in this forward or in an earlier
    backward on the stream (reported here, at the next synchronising call, so
    that the autograd backward itself never synchronises)."""
    words = _lib.status_words(dev)
    st = words[:4].tolist()
    if st[_lib.STATUS_DPACE_BWD] or st[_lib.STATUS_DFLASH_BWD]:
        words[1:3].zero_()
        raise RuntimeError(_BWD_TIMEOUT_MSG)
    if st[_lib.STATUS_DRAFTER]:
        words[3:4].zero_()
        raise RuntimeError(_ATTN_TIMEOUT_MSG)
    if st[_lib.STATUS_DPACE_FWD] == _lib.ERR_TARGET_RANGE:
        raise ValueError(f"targets out of range [0, {V})")
    if st[_lib.STATUS_DPACE_FWD] == _lib.ERR_CUDA:  # counters are in an unknown state
        _lib.workspace("dpace", dev).reset_counters()
        raise RuntimeError(f"{what}: a bulk-copy wait timed out")


def check_backward(device: torch.device | int | None = None) -> None:
    """Synchronise with the current stream of `device` and raise RuntimeError
    if a D-PACE or DFlash backward, or a drafter attention kernel, launched on
    it since the last check had a bounded wait expire (its outputs then hold
    NaN where the failed part wrote). Every D-PACE forward that validates its
    targets performs this check as well."""
    dev = torch.device("cuda", torch.cuda.current_device() if device is None else
                       (device if isinstance(device, int) else device.index))
    words = _lib.status_words(dev)
    st = words[:4].tolist()
    if st[_lib.STATUS_DPACE_BWD] or st[_lib.STATUS_DFLASH_BWD]:
        words[1:3].zero_()
        raise RuntimeError(_BWD_TIMEOUT_MSG)
    if st[_lib.STATUS_DRAFTER]:
        words[3:4].zero_()
        raise RuntimeError(_ATTN_TIMEOUT_MSG)


def _dpace_forward(logits: torch.Tensor, targets: torch.Tensor, mask: torch.Tensor | None,
                  alpha: float, loss_type: int, n_global: int | None = None,
                  want_loss_n: bool = False, validate: bool | None = None):
    """Returns (loss 0-d, lse [N,B], scale [N,B], loss_n [N] or None)."""
    lib = _lib.load()
    N, B, V = logits.shape
    dev = logits.device
    n_global = N if n_global is None else int(n_global)
    loss = torch.empty((), dtype=torch.float32, device=dev)
    lse = torch.empty((N, B), dtype=torch.float32, device=dev)
    scale = torch.empty((N, B), dtype=torch.float32, device=dev)
    loss_n = torch.empty((N,), dtype=torch.float32, device=dev) if want_loss_n else None
    status = _lib.status_words(dev)[_lib.STATUS_DPACE_FWD:]
    ws = _lib.workspace("dpace", dev)
    sb = lib.specdec_dpace_scratch_bytes(N, B, V, dev.index)
    cb = lib.specdec_dpace_counter_bytes(N, B)
    scratch, counters = ws.ensure(dev, sb, cb)
    logits = _aligned(logits)
    code = _entry(lib, "specdec_dpace_forward", logits)(
        logits.data_ptr(), targets.data_ptr(), _lib.ptr(mask), N, B, V, float(alpha),
        int(loss_type), n_global, loss.data_ptr(), _lib.ptr(loss_n), lse.data_ptr(),
        scale.data_ptr(), status.data_ptr(), scratch.data_ptr(), scratch.numel(),
        counters.data_ptr(), counters.numel(), _lib.stream_handle(dev))
    _lib.check(code, "specdec_dpace_forward")
    if (VALIDATE_TARGETS if validate is None else validate) and N * B > 0 and not _capturing():
        _read_status(dev, "specdec_dpace_forward", V)
    return loss, lse, scale, loss_n


def _dpace_forward_backward(logits: torch.Tensor, targets: torch.Tensor, mask: torch.Tensor | None,
                            alpha: float, loss_type: int, n_global: int | None = None,
                            want_loss_n: bool = False, validate: bool | None = None,
                            out: torch.Tensor | None = None):
    """Loss and gradient (dloss = 1) in one call: the forward and backward
    kernels back to back on the current stream. Returns (loss 0-d, dlogits,
    lse [N,B], scale [N,B], loss_n or None)."""
    lib = _lib.load()
    N, B, V = logits.shape
    dev = logits.device
    n_global = N if n_global is None else int(n_global)
    logits = _aligned(logits)
    loss = torch.empty((), dtype=torch.float32, device=dev)
    lse = torch.empty((N, B), dtype=torch.float32, device=dev)
    scale = torch.empty((N, B), dtype=torch.float32, device=dev)
    loss_n = torch.empty((N,), dtype=torch.float32, device=dev) if want_loss_n else None
    dlogits = torch.empty_like(logits) if out is None else out
    status = _lib.status_words(dev)[_lib.STATUS_DPACE_FWD:]
    ws = _lib.workspace("dpace", dev)
    sb = lib.specdec_dpace_scratch_bytes(N, B, V, dev.index)
    cb = lib.specdec_dpace_counter_bytes(N, B)
    scratch, counters = ws.ensure(dev, sb, cb)
    code = _entry(lib, "specdec_dpace_forward_backward", logits)(
        logits.data_ptr(), targets.data_ptr(), _lib.ptr(mask), N, B, V, float(alpha),
        int(loss_type), n_global, loss.data_ptr(), _lib.ptr(loss_n), lse.data_ptr(),
        scale.data_ptr(), dlogits.data_ptr(), status.data_ptr(), scratch.data_ptr(), scratch.numel(),
        counters.data_ptr(), counters.numel(), _lib.stream_handle(dev))
    _lib.check(code, "specdec_dpace_forward_backward")
    if (VALIDATE_TARGETS if validate is None else validate) and N * B > 0 and not _capturing():
        _read_status(dev, "specdec_dpace_forward_backward", V)
    return loss, dlogits, lse, scale, loss_n


def _scale_inplace(x: torch.Tensor, factor: torch.Tensor) -> torch.Tensor:
    """x *= factor (a 1-element device tensor); no pass over x when factor == 1."""
    lib = _lib.load()
    f = factor.detach().to(device=x.device, dtype=torch.float32).reshape(1).contiguous()
    code = _entry(lib, "specdec_scale_inplace", x)(x.data_ptr(), x.numel(), f.data_ptr(),
                                                    _lib.stream_handle(x.device))
    _lib.check(code, "specdec_scale_inplace")
    return x


def _dpace_backward(logits: torch.Tensor, targets: torch.Tensor, lse: torch.Tensor,
                   scale: torch.Tensor, dloss: torch.Tensor | None,
                   out: torch.Tensor | None = None) -> torch.Tensor:
    lib = _lib.load()
    N, B, V = logits.shape
    dev = logits.device
    logits = _aligned(logits)
    dlogits = torch.empty_like(logits) if out is None else out
    if dloss is not None:
        dloss = dloss.detach().to(device=dev, dtype=torch.float32).contiguous()
    cb = lib.specdec_backward_counter_bytes()
    _, counters = _lib.workspace("dpace_bwd", dev).ensure(dev, 256, cb)
    status = _lib.status_words(dev)[_lib.STATUS_DPACE_BWD:]
    code = _entry(lib, "specdec_dpace_backward", logits)(
        logits.data_ptr(), targets.data_ptr(), lse.data_ptr(), scale.data_ptr(),
        _lib.ptr(dloss), dlogits.data_ptr(), N, B, V, status.data_ptr(), counters.data_ptr(),
        counters.numel(), _lib.stream_handle(dev))
    _lib.check(code, "specdec_dpace_backward")
    return dlogits


def _dflash_forward(logits: torch.Tensor, target_logits: torch.Tensor, mask: torch.Tensor | None,
                   gamma: float, sample_from_anchor: bool, kind: int, block_size: int,
                   n_global: int | None = None):
    """Returns (loss 0-d, loss_rows [N,B], scale [N,B], logzq [N,B], logzp [N,B], tgt [N,B] or None)."""
    lib = _lib.load()
    N, B, V = logits.shape
    dev = logits.device
    n_global = N if n_global is None else int(n_global)
    loss = torch.empty((), dtype=torch.float32, device=dev)
    loss_rows = torch.empty((N, B), dtype=torch.float32, device=dev)
    scale = torch.empty((N, B), dtype=torch.float32, device=dev)
    logzq = torch.empty((N, B), dtype=torch.float32, device=dev)
    logzp = torch.empty((N, B), dtype=torch.float32, device=dev)
    tgt = torch.empty((N, B), dtype=torch.int64, device=dev) if kind == 1 else None
    ws = _lib.workspace("dflash", dev)
    sb = lib.specdec_dflash_scratch_bytes(N, B, V, dev.index)
    cb = lib.specdec_dflash_counter_bytes(N, B)
    scratch, counters = ws.ensure(dev, sb, cb)
    logits, target_logits = _aligned(logits), _aligned(target_logits)
    code = _entry(lib, "specdec_dflash_forward", logits)(
        logits.data_ptr(), target_logits.data_ptr(), _lib.ptr(mask), N, B, V, int(block_size),
        float(gamma), int(bool(sample_from_anchor)), int(kind), n_global, loss.data_ptr(),
        loss_rows.data_ptr(), scale.data_ptr(), logzq.data_ptr(), logzp.data_ptr(),
        _lib.ptr(tgt), scratch.data_ptr(), scratch.numel(), counters.data_ptr(),
        counters.numel(), _lib.stream_handle(dev))
    _lib.check(code, "specdec_dflash_forward")
    return loss, loss_rows, scale, logzq, logzp, tgt


def _dflash_backward(logits: torch.Tensor, target_logits: torch.Tensor | None, scale: torch.Tensor,
                    logzq: torch.Tensor, logzp: torch.Tensor, tgt: torch.Tensor | None,
                    dloss: torch.Tensor | None, kind: int,
                    out: torch.Tensor | None = None) -> torch.Tensor:
    lib = _lib.load()
    N, B, V = logits.shape
    dev = logits.device
    logits, target_logits = _aligned(logits), _aligned(target_logits)
    dlogits = torch.empty_like(logits) if out is None else out
    if dloss is not None:
        dloss = dloss.detach().to(device=dev, dtype=torch.float32).contiguous()
    cb = lib.specdec_backward_counter_bytes()
    _, counters = _lib.workspace("dflash_bwd", dev).ensure(dev, 256, cb)
    status = _lib.status_words(dev)[_lib.STATUS_DFLASH_BWD:]
    code = _entry(lib, "specdec_dflash_backward", logits)(
        logits.data_ptr(), _lib.ptr(target_logits), scale.data_ptr(), logzq.data_ptr(),
        logzp.data_ptr(), _lib.ptr(tgt), _lib.ptr(dloss), dlogits.data_ptr(), N, B, V, int(kind),
        status.data_ptr(), counters.data_ptr(), counters.numel(), _lib.stream_handle(dev))
    _lib.check(code, "specdec_dflash_backward")
    return dlogits


def _on_device(fn):
    def wrapped(logits, *args, **kwargs):
        with _lib.on_device(logits.device):
            return fn(logits, *args, **kwargs)
    wrapped.__name__ = fn.__name__.lstrip("_")
    wrapped.__doc__ = fn.__doc__
    return wrapped


# Launches go to the tensors' device (and that device's current stream),
# whatever the caller's current device is.
dpace_forward = _on_device(_dpace_forward)
dpace_backward = _on_device(_dpace_backward)
dpace_forward_backward = _on_device(_dpace_forward_backward)
scale_inplace = _on_device(_scale_inplace)
dflash_forward = _on_device(_dflash_forward)
dflash_backward = _on_device(_dflash_backward)
