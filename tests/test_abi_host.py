"""C-ABI library and host-side logic, without a GPU: the library loads, exports
every function include/specdec.h declares, and rejects bad arguments with the
documented status codes before touching the device; the Python glue raises
the reference's exception types."""
import ctypes
import os
import re

import pytest
import torch

from specdec import _lib

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(REPO, "include", "specdec.h")


def _declared():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(specdec_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    declared = _declared()
    assert declared, "no declarations parsed"
    for name in declared:
        assert hasattr(lib, name), f"{name} missing from libspecdec.so"
    assert set(declared) == set(_lib.exported_symbols())


def test_version_and_status_strings():
    lib = _lib.load()
    assert lib.specdec_version() >= 100
    assert lib.specdec_status_string(0) == b"ok"
    assert lib.specdec_status_string(3) == b"target id out of range"


def test_counter_bytes_are_host_only():
    lib = _lib.load()
    assert lib.specdec_dpace_counter_bytes(64, 16) >= 16 + 64 * 4
    assert lib.specdec_backward_counter_bytes() >= 16
    assert lib.specdec_dflash_counter_bytes(64, 16) >= 16 + 64 * 16 * 4
    assert lib.specdec_dpace_counter_bytes(64, 16) % 256 == 0


def _dpace_call(lib, B=16, alpha=0.5, loss_type=0, N=4, V=100):
    fake = ctypes.c_void_p(256)  # never dereferenced: argument checks fail first
    return lib.specdec_dpace_forward(fake, fake, None, N, B, V, alpha, loss_type, N, fake, None,
                                     fake, fake, None, fake, 1 << 20, fake, 1 << 20, None)


def test_dpace_argument_checks_without_gpu():
    lib = _lib.load()
    assert _dpace_call(lib, B=33) == _lib.ERR_ARGUMENT
    assert b"block_size <= 32" in lib.specdec_last_error()
    assert _dpace_call(lib, B=0) == _lib.ERR_ARGUMENT
    assert _dpace_call(lib, alpha=1.5) == _lib.ERR_VALUE
    assert _dpace_call(lib, alpha=float("nan")) == _lib.ERR_VALUE
    assert _dpace_call(lib, loss_type=3) == _lib.ERR_VALUE
    assert _dpace_call(lib, V=0) == _lib.ERR_TARGET_RANGE


def test_dflash_argument_checks_without_gpu():
    lib = _lib.load()
    fake = ctypes.c_void_p(256)

    def call(block_size=8, gamma=4.0, kind=0, B=8):
        return lib.specdec_dflash_forward(fake, fake, None, 4, B, 100, block_size, gamma, 0, kind,
                                          4, fake, None, fake, fake, fake, None, fake, 1 << 20,
                                          fake, 1 << 20, None)

    assert call(block_size=9) == _lib.ERR_ARGUMENT
    assert call(block_size=0) == _lib.ERR_ARGUMENT
    assert call(gamma=0.0) == _lib.ERR_VALUE
    assert call(gamma=-1.0) == _lib.ERR_VALUE
    assert call(kind=2) == _lib.ERR_VALUE


def test_status_to_exception_mapping():
    with pytest.raises(AssertionError):
        _lib.check(_lib.ERR_ARGUMENT, "x")
    with pytest.raises(ValueError):
        _lib.check(_lib.ERR_VALUE, "x")
    with pytest.raises(ValueError):
        _lib.check(_lib.ERR_TARGET_RANGE, "x")
    with pytest.raises(RuntimeError):
        _lib.check(_lib.ERR_CUDA, "x")
    _lib.check(_lib.OK, "x")


# ---- reference-facing host checks (losses/dpace.py:157-173, loss.py:178-191) ----

def test_dpace_host_checks():
    from losses.dpace import _check

    x = torch.zeros(2, 4, 8)
    t = torch.zeros(2, 4, dtype=torch.int64)
    _check(x, t, None, 0.5, "dpace")
    with pytest.raises(AssertionError):
        _check(x.double(), t, None, 0.5, "dpace")
    with pytest.raises(AssertionError):
        _check(x, t.int(), None, 0.5, "dpace")
    with pytest.raises(AssertionError):
        _check(torch.zeros(2, 33, 8), torch.zeros(2, 33, dtype=torch.int64), None, 0.5, "dpace")
    with pytest.raises(AssertionError):
        _check(x, t, torch.zeros(2, 3), 0.5, "dpace")
    with pytest.raises(ValueError):
        _check(x, t, None, 1.5, "dpace")
    with pytest.raises(ValueError):
        _check(x, t, None, 0.5, "topk_mask")
    with pytest.raises(ValueError):
        _check(torch.zeros(2, 4, 0), t, None, 0.5, "dpace")


def test_dflash_host_checks():
    from models.dflash.loss import _check

    x = torch.zeros(2, 8, 16)
    _check(x, x, None, 4.0, "kl", None)
    _check(x, x, None, 4.0, "ce", 3)
    with pytest.raises(AssertionError):
        _check(x, x, None, 4.0, "kl", 9)
    with pytest.raises(AssertionError):
        _check(x, torch.zeros(2, 8, 4), None, 4.0, "kl", None)
    with pytest.raises(ValueError):
        _check(x, x, None, 0.0, "kl", None)
    with pytest.raises(ValueError):
        _check(x, x, None, 4.0, "tv", None)


def test_entry_points_reject_cpu_tensors():
    from losses import dpace_loss, fused_dpace_loss
    from models.dflash import dflash_loss, fused_dflash_loss

    x = torch.zeros(2, 4, 8)
    t = torch.zeros(2, 4, dtype=torch.int64)
    for fn in (lambda: dpace_loss(x, t), lambda: fused_dpace_loss(x, t),
               lambda: dflash_loss(x, x), lambda: fused_dflash_loss(x, x)):
        with pytest.raises(AssertionError):
            fn()


def test_dflash_objective_binds_target_logits():
    from models.dflash import dflash_objective

    seen = {}

    import models.dflash.loss as L
    orig = L.dflash_loss
    try:
        L.dflash_loss = lambda lg, tl, **kw: seen.update(lg=lg, tl=tl, kw=kw) or 0.0
        fn = dflash_objective("VERIFIER", gamma=2.0, kind="ce")
        fn("DRAFT", "TOKENS")
    finally:
        L.dflash_loss = orig
    assert seen == {"lg": "DRAFT", "tl": "VERIFIER", "kw": {"gamma": 2.0, "kind": "ce"}}
