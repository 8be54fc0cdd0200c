"""Parity cases shared by the golden-vector generator and the tests.

Inputs are regenerated from per-case seeds with numpy's PCG64 Generator; each
fixture records the SHA-256 of the generated input bytes, so a change in the
generator stream shows up as a test failure rather than a silent mismatch.
The case list mirrors the reference's own checks
(losses/tests/test_dpace.py:66-81, models/dflash/tests/test_loss.py:77-95)
plus reduced-N versions of the benchmark workloads (same V, B, value
distribution and mask rule).
"""
from __future__ import annotations

import hashlib

import numpy as np

FULL_GRAD_MAX = 16384   # store the whole gradient up to this many elements
N_PROBES = 256          # otherwise store the gradient at this many random positions

DPACE_TYPES = ("dpace", "dpace-cumulative-confidence-only", "dpace-continuation-value-only")


def _c(name, N, B, V, seed, **kw):
    d = dict(name=name, N=N, B=B, V=V, seed=seed, sigma=1.0, shift=0.0, mask="none",
             alpha=0.5, loss_type="dpace")
    d.update(kw)
    return d


DPACE_CASES = [
    _c("nomask_N8_B4_V1024", 8, 4, 1024, 1),
    _c("bern.5_N8_B8_V1024", 8, 8, 1024, 2, mask=("bern", 0.5)),
    _c("bern.2_N8_B8_V1024", 8, 8, 1024, 3, mask=("bern", 0.2)),
    _c("bern.05_N8_B16_V1024", 8, 16, 1024, 4, mask=("bern", 0.05)),
    _c("B1_N8_V1024", 8, 1, 1024, 5, mask=("bern", 0.5)),
    _c("B32_N8_V1024", 8, 32, 1024, 6, mask=("bern", 0.5)),
    _c("V7_N6_B8", 6, 8, 7, 7, mask=("bern", 0.5)),
    _c("V1000_N6_B8", 6, 8, 1000, 8, mask=("bern", 0.5)),
    _c("V32000_N4_B8", 4, 8, 32000, 9, mask=("bern", 0.5)),
    _c("V151936_N2_B8", 2, 8, 151936, 10, mask=("bern", 0.5)),
    _c("shift-20_N8_B4_V1024", 8, 4, 1024, 11, mask=("bern", 0.5), shift=-20.0),
    _c("alpha0_N4_B8_V2048", 4, 8, 2048, 12, mask=("bern", 0.5), alpha=0.0),
    _c("alpha.1_N4_B8_V2048", 4, 8, 2048, 13, mask=("bern", 0.5), alpha=0.1),
    _c("alpha.9_N4_B8_V2048", 4, 8, 2048, 14, mask=("bern", 0.5), alpha=0.9),
    _c("alpha1_N4_B8_V2048", 4, 8, 2048, 15, mask=("bern", 0.5), alpha=1.0),
    _c("type_P_N4_B8_V1024", 4, 8, 1024, 16, mask=("bern", 0.5),
       loss_type="dpace-cumulative-confidence-only"),
    _c("type_SP_N4_B8_V1024", 4, 8, 1024, 17, mask=("bern", 0.5),
       loss_type="dpace-continuation-value-only"),
    _c("allmasked_N4_B8_V512", 4, 8, 512, 18, mask=("zeros",)),
    _c("seq0masked_N4_B8_V512", 4, 8, 512, 19, mask=("seq0",)),
    _c("fracmask_N4_B8_V512", 4, 8, 512, 20, mask=("frac",)),
    _c("col3masked_N2_B8_V256", 2, 8, 256, 21, mask=("col", 3)),
    _c("N3_B8_V7_masked", 3, 8, 7, 22, mask=("bern", 0.5)),
    # workload shapes (N reduced so the CPU oracle finishes in seconds)
    _c("ws1_N8_B16_V32000_sd2", 8, 16, 32000, 101, sigma=2.0),
    _c("ws2_N4_B16_V128256_sd2_prefix4", 4, 16, 128256, 102, sigma=2.0, mask=("prefix", 4)),
    _c("ws2P_N2_B16_V128256_sd2_prefix4", 2, 16, 128256, 103, sigma=2.0, mask=("prefix", 4),
       loss_type="dpace-cumulative-confidence-only"),
    _c("ws2SP_N2_B16_V128256_sd2_prefix4", 2, 16, 128256, 104, sigma=2.0, mask=("prefix", 4),
       loss_type="dpace-continuation-value-only"),
    _c("ws4_N2_B32_V151936_sd3_prefix8", 2, 32, 151936, 105, sigma=3.0, mask=("prefix", 8)),
]


def _f(name, N, B, V, seed, **kw):
    d = dict(name=name, N=N, B=B, V=V, seed=seed, sigma=1.0, noise=None, mask="none",
             gamma=4.0, sfa=False, kind="kl", block_size=None)
    d.update(kw)
    return d


DFLASH_CASES = [
    _f("kl_N8_B4_V1024", 8, 4, 1024, 201),
    _f("ce_N8_B4_V1024", 8, 4, 1024, 202, kind="ce"),
    _f("kl_bern.5_N8_B8_V1024", 8, 8, 1024, 203, mask=("bern", 0.5)),
    _f("ce_bern.5_N8_B8_V1024", 8, 8, 1024, 204, mask=("bern", 0.5), kind="ce"),
    _f("kl_B1_N8_V1024", 8, 1, 1024, 205),
    _f("kl_B32_N8_V1024", 8, 32, 1024, 206, mask=("bern", 0.7)),
    _f("kl_V7_N6_B8", 6, 8, 7, 207, mask=("bern", 0.7)),
    _f("kl_V1000_N6_B8", 6, 8, 1000, 208, mask=("bern", 0.7)),
    _f("kl_V32000_N4_B8", 4, 8, 32000, 209, mask=("bern", 0.7)),
    _f("kl_V151936_N2_B8", 2, 8, 151936, 210, mask=("bern", 0.7)),
    _f("kl_N64_B8_V4096", 64, 8, 4096, 211, mask=("bern", 0.7)),
    _f("kl_gamma1_N4_B8_V2048", 4, 8, 2048, 212, mask=("bern", 0.7), gamma=1.0),
    _f("kl_gamma10_N4_B8_V2048", 4, 8, 2048, 213, mask=("bern", 0.7), gamma=10.0),
    _f("kl_gamma100_N4_B8_V2048", 4, 8, 2048, 214, mask=("bern", 0.7), gamma=100.0),
    _f("kl_sfa_N4_B8_V1024", 4, 8, 1024, 215, mask=("bern", 0.7), sfa=True),
    _f("ce_sfa_N4_B8_V1024", 4, 8, 1024, 216, mask=("bern", 0.7), sfa=True, kind="ce"),
    _f("kl_bs4_N4_B16_V1024", 4, 16, 1024, 217, mask=("bern", 0.7), block_size=4),
    _f("ce_bs4_N4_B16_V1024", 4, 16, 1024, 218, mask=("bern", 0.7), block_size=4, kind="ce"),
    _f("kl_bs3_N4_B12_V512", 4, 12, 512, 219, block_size=3),
    _f("kl_bs3_N3_B8_V256_ragged", 3, 8, 256, 220, block_size=3, mask=("bern", 0.7)),
    _f("kl_allmasked_N4_B8_V512", 4, 8, 512, 221, mask=("zeros",)),
    _f("kl_fracmask_N4_B8_V512", 4, 8, 512, 222, mask=("frac",)),
    _f("ce_ties_N4_B8_V64", 4, 8, 64, 223, kind="ce", ties=True),
    # workload shape: verifier = draft + N(0, 1), draft ~ N(0, 2^2)
    _f("ws3_kl_N4_B16_V128256_sd2_corr", 4, 16, 128256, 301, sigma=2.0, noise=1.0),
    _f("ws3_ce_N2_B16_V128256_sd2_corr", 2, 16, 128256, 302, sigma=2.0, noise=1.0, kind="ce"),
]


def make_mask(rng: np.random.Generator, spec, N: int, B: int):
    if spec == "none":
        return None
    kind = spec[0]
    if kind == "bern":
        return (rng.random((N, B)) < spec[1]).astype(np.float32)
    if kind == "prefix":
        m = np.ones((N, B), np.float32)
        k = rng.integers(0, spec[1] + 1, N)
        for n in range(N):
            m[n, :k[n]] = 0.0
        return m
    if kind == "zeros":
        return np.zeros((N, B), np.float32)
    if kind == "seq0":
        m = np.ones((N, B), np.float32)
        m[0] = 0.0
        return m
    if kind == "col":
        m = np.ones((N, B), np.float32)
        m[:, spec[1]] = 0.0
        return m
    if kind == "frac":
        m = rng.random((N, B)).astype(np.float32)
        m[m < 0.3] = 0.0
        return m
    raise ValueError(spec)


def dpace_inputs(case):
    rng = np.random.default_rng(case["seed"])
    N, B, V = case["N"], case["B"], case["V"]
    x = (rng.normal(0.0, case["sigma"], (N, B, V)) + case["shift"]).astype(np.float32)
    t = rng.integers(0, V, (N, B), dtype=np.int64)
    m = make_mask(rng, case["mask"], N, B)
    return x, t, m


def dflash_inputs(case):
    rng = np.random.default_rng(case["seed"])
    N, B, V = case["N"], case["B"], case["V"]
    x = rng.normal(0.0, case["sigma"], (N, B, V)).astype(np.float32)
    if case["noise"] is None:
        y = rng.normal(0.0, case["sigma"], (N, B, V)).astype(np.float32)
    else:
        y = (x + rng.normal(0.0, case["noise"], (N, B, V))).astype(np.float32)
    if case.get("ties"):
        # integer-valued verifier logits: repeated maxima exercise the first-index argmax
        y = np.round(y * 2.0).astype(np.float32)
    m = make_mask(rng, case["mask"], N, B)
    return x, y, m


def digest(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        if a is not None:
            h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def probe_indices(case, total: int) -> np.ndarray:
    rng = np.random.default_rng(case["seed"] + 7919)
    return np.sort(rng.choice(total, size=min(N_PROBES, total), replace=False)).astype(np.int64)
