"""ctypes binding of libspecdec.so, the C ABI declared in include/specdec.h.

This module is the only place that touches the shared library. It maps the
library's status codes onto the exceptions the reference raises
(AssertionError for shape/dtype/contract violations, ValueError for values out
of domain), and keeps one workspace (scratch + zero-initialised counters) per
(device, stream, kernel family) so repeated calls allocate nothing.

There is no fallback: if the library is missing, every entry point raises.
"""
from __future__ import annotations

import contextlib
import ctypes
import os
import threading

import torch

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libspecdec.so")

OK = 0
ERR_ARGUMENT = 1
ERR_VALUE = 2
ERR_TARGET_RANGE = 3
ERR_WORKSPACE = 4
ERR_CUDA = 5

KERNEL_DPACE_FWD = 0
KERNEL_DPACE_BWD = 1
KERNEL_DFLASH_FWD = 2
KERNEL_DFLASH_BWD = 3
SHAPE_DEFAULT = -1  # set_launch_shape: the built-in choice per kernel and dtype

_c_i32 = ctypes.c_int32
_c_i64 = ctypes.c_int64
_c_f32 = ctypes.c_float
_c_sz = ctypes.c_size_t
_c_p = ctypes.c_void_p

# name -> (restype, argtypes); mirrors include/specdec.h
_SIGNATURES = {
    "specdec_version": (ctypes.c_int, []),
    "specdec_last_error": (ctypes.c_char_p, []),
    "specdec_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "specdec_dpace_scratch_bytes": (_c_sz, [_c_i64, _c_i32, _c_i64, ctypes.c_int]),
    "specdec_dpace_counter_bytes": (_c_sz, [_c_i64, _c_i32]),
    "specdec_dpace_forward": (ctypes.c_int, [
        _c_p, _c_p, _c_p, _c_i64, _c_i32, _c_i64, _c_f32, _c_i32, _c_i64,
        _c_p, _c_p, _c_p, _c_p, _c_p, _c_p, _c_sz, _c_p, _c_sz, _c_p]),
    "specdec_dpace_forward_noalloc": (ctypes.c_int, [
        _c_p, _c_p, _c_p, _c_i64, _c_i32, _c_i64, _c_f32, _c_i32, _c_i64,
        _c_p, _c_p, _c_p, _c_p, _c_p, _c_p]),
    "specdec_backward_counter_bytes": (_c_sz, []),
    "specdec_dpace_backward": (ctypes.c_int, [
        _c_p, _c_p, _c_p, _c_p, _c_p, _c_p, _c_i64, _c_i32, _c_i64, _c_p, _c_p, _c_sz, _c_p]),
    "specdec_dflash_scratch_bytes": (_c_sz, [_c_i64, _c_i32, _c_i64, ctypes.c_int]),
    "specdec_dflash_counter_bytes": (_c_sz, [_c_i64, _c_i32]),
    "specdec_dflash_forward": (ctypes.c_int, [
        _c_p, _c_p, _c_p, _c_i64, _c_i32, _c_i64, _c_i32, _c_f32, _c_i32, _c_i32, _c_i64,
        _c_p, _c_p, _c_p, _c_p, _c_p, _c_p, _c_p, _c_sz, _c_p, _c_sz, _c_p]),
    "specdec_dflash_backward": (ctypes.c_int, [
        _c_p, _c_p, _c_p, _c_p, _c_p, _c_p, _c_p, _c_p, _c_i64, _c_i32, _c_i64, _c_i32, _c_p, _c_p,
        _c_sz, _c_p]),
    "specdec_set_launch_shape": (ctypes.c_int, [_c_i32, _c_i32, _c_i32]),
    "specdec_launch_ctas": (_c_i64, [_c_i32, _c_i64, _c_i64, ctypes.c_int]),
    "specdec_set_block_queue": (ctypes.c_int, [_c_i32]),
    "specdec_test_withhold_stage": (ctypes.c_int, [_c_i32]),
    "specdec_dpace_forward_backward": (ctypes.c_int, [
        _c_p, _c_p, _c_p, _c_i64, _c_i32, _c_i64, _c_f32, _c_i32, _c_i64,
        _c_p, _c_p, _c_p, _c_p, _c_p, _c_p, _c_p, _c_sz, _c_p, _c_sz, _c_p]),
    "specdec_scale_inplace": (ctypes.c_int, [_c_p, _c_i64, _c_p, _c_p]),
    "specdec_rmsnorm_forward": (ctypes.c_int, [_c_p, _c_p, _c_p, _c_p, _c_i64, _c_i32, _c_f32, _c_i32, _c_p]),
    "specdec_rmsnorm_workspace_bytes": (_c_sz, [_c_i64, _c_i32, ctypes.c_int]),
    "specdec_rmsnorm_backward": (ctypes.c_int, [
        _c_p, _c_p, _c_p, _c_p, _c_p, _c_p, _c_i64, _c_i32, _c_i32, _c_p, _c_sz, _c_p]),
    "specdec_dflash_attention_forward": (ctypes.c_int, [
        _c_p, _c_p, _c_p, _c_p, _c_p, _c_i32, _c_i32, _c_i32, _c_i32, _c_i32, _c_f32, _c_p, _c_p]),
    "specdec_dflash_attention_workspace_bytes": (_c_sz, [_c_i32, _c_i32, _c_i32]),
    "specdec_dflash_attention_backward": (ctypes.c_int, [
        _c_p, _c_p, _c_p, _c_p, _c_p, _c_p, _c_p, _c_p, _c_p, _c_i32, _c_i32, _c_i32, _c_i32, _c_i32, _c_f32,
        _c_p, _c_p, _c_sz, _c_p]),
}
# bf16 entry points take the same arguments as their fp32 counterparts
for _name in ("specdec_dpace_forward", "specdec_dpace_backward", "specdec_dflash_forward",
              "specdec_dflash_backward", "specdec_dpace_forward_backward", "specdec_scale_inplace"):
    _SIGNATURES[_name + "_bf16"] = _SIGNATURES[_name]

_lib = None
_lib_lock = threading.Lock()


def load() -> ctypes.CDLL:
    """Load libspecdec.so once and attach the C signatures. Raises if absent."""
    global _lib
    if _lib is not None:
        return _lib
    with _lib_lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise ImportError(
                    f"libspecdec.so is not built ({LIB_PATH}); build it with "
                    "`make -C cuda-spec-decode_b200/csrc` or __graft_entry__.build()")
            lib = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in _SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def exported_symbols() -> list[str]:
    return list(_SIGNATURES)


def last_error() -> str:
    return load().specdec_last_error().decode()


def check(code: int, what: str) -> None:
    """Raise the reference's exception type for a non-OK status."""
    if code == OK:
        return
    msg = last_error() or load().specdec_status_string(code).decode()
    if code == ERR_ARGUMENT:
        raise AssertionError(msg)
    if code in (ERR_VALUE, ERR_TARGET_RANGE):
        raise ValueError(msg)
    raise RuntimeError(f"{what}: {msg}")


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def on_device(device: torch.device):
    """Context that makes `device` current: a no-op when it already is (the
    common case; entering torch.cuda.device costs host time on every call)."""
    if device.index is None or device.index == torch.cuda.current_device():
        return contextlib.nullcontext()
    return torch.cuda.device(device)


def stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def set_launch_shape(kernel: int, shape: int, ctas_per_sm: int = 0) -> None:
    check(load().specdec_set_launch_shape(kernel, shape, ctas_per_sm), "set_launch_shape")
    _workspaces.clear()


def set_block_queue(dynamic: bool) -> None:
    """Ring kernels: atomic block queue (True, default) or static interleave."""
    check(load().specdec_set_block_queue(1 if dynamic else 0), "set_block_queue")


class Workspace:
    """Scratch + counters for one (device, stream, family).

    The counters must be zero before the first call; every completed call
    leaves them zero, so they are zeroed only when (re)allocated.
    """

    __slots__ = ("scratch", "counters")

    def __init__(self):
        self.scratch = None
        self.counters = None

    def ensure(self, device: torch.device, scratch_bytes: int, counter_bytes: int):
        if self.scratch is None or self.scratch.numel() < scratch_bytes:
            self.scratch = torch.empty(max(scratch_bytes, 256), dtype=torch.uint8, device=device)
        if self.counters is None or self.counters.numel() < counter_bytes:
            self.counters = torch.zeros(max(counter_bytes, 256), dtype=torch.uint8, device=device)
        return self.scratch, self.counters

    def reset_counters(self):
        if self.counters is not None:
            self.counters.zero_()


_workspaces: dict = {}


def workspace(family: str, device: torch.device) -> Workspace:
    key = (family, device.index, torch.cuda.current_stream(device).cuda_stream)
    ws = _workspaces.get(key)
    if ws is None:
        ws = _workspaces[key] = Workspace()
    return ws


# Device status words per (device, stream), written by the kernels:
STATUS_DPACE_FWD = 0   # the D-PACE forward (and forward_backward): 0, ERR_TARGET_RANGE or ERR_CUDA
STATUS_DPACE_BWD = 1   # the last D-PACE backward: 0 or ERR_CUDA
STATUS_DFLASH_BWD = 2  # the last DFlash backward: 0 or ERR_CUDA
STATUS_DRAFTER = 3     # the drafter's attention kernels, sticky: 0, or ERR_CUDA once any wait expired
_status: dict = {}


def status_words(device: torch.device) -> torch.Tensor:
    """int32[4] on `device` for the current stream, zero-initialised once; the
    entry points write their status word into it on the device."""
    key = (device.index, torch.cuda.current_stream(device).cuda_stream)
    t = _status.get(key)
    if t is None:
        t = _status[key] = torch.zeros(4, dtype=torch.int32, device=device)
    return t
