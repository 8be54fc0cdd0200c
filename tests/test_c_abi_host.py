"""The C ABI from a pure C host (tests/c/abi_host.c: include/specdec.h, the CUDA
runtime and libspecdec.so, no Python): the header compiles as C11 and links
(CPU); on the GPU the program's loss and gradient equal the oracle's on
golden-case inputs (loss 1e-5 relative, gradient 1e-6 absolute)."""
import os
import struct
import subprocess

import numpy as np
import pytest
import torch

import cases
from oracle import dflash as odf
from oracle import dpace as odp

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIBDIR = os.path.join(REPO, "cuda-spec-decode_b200", "specdec")
CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")


def _build(tmp_path) -> str:
    exe = str(tmp_path / "abi_host")
    cmd = ["gcc", "-std=c11", "-O2", "-Wall", "-Werror", "-I", os.path.join(REPO, "include"),
           "-I", os.path.join(CUDA_HOME, "include"), os.path.join(REPO, "tests", "c", "abi_host.c"),
           "-L", LIBDIR, "-lspecdec", "-L", os.path.join(CUDA_HOME, "lib64"), "-lcudart",
           f"-Wl,-rpath,{LIBDIR}", f"-Wl,-rpath,{os.path.join(CUDA_HOME, 'lib64')}", "-o", exe]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    return exe


def test_header_compiles_and_links_from_c(tmp_path):
    if not os.path.exists(os.path.join(LIBDIR, "libspecdec.so")):
        pytest.skip("libspecdec.so not built")
    assert os.path.exists(_build(tmp_path))


def _run(exe, tmp_path, header: bytes, *arrays):
    src, dst = tmp_path / "in.bin", tmp_path / "out.bin"
    with open(src, "wb") as f:
        f.write(header)
        for a in arrays:
            f.write(np.ascontiguousarray(a).tobytes())
    r = subprocess.run([exe, str(src), str(dst)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, (r.returncode, r.stderr)
    out = np.fromfile(dst, dtype=np.float32)
    return float(out[0]), out[1:]


DPACE = [c for c in cases.DPACE_CASES if c["N"] * c["B"] * c["V"] <= 4_000_000][:8]
DFLASH = [c for c in cases.DFLASH_CASES if c["N"] * c["B"] * c["V"] <= 4_000_000
          and c["block_size"] in (None,) and not c["sfa"] and c["mask"] == "none"][:6]


@pytest.mark.gpu
@pytest.mark.parametrize("case", DPACE, ids=lambda c: c["name"])
def test_c_host_dpace_matches_oracle(cuda, tmp_path, case):
    exe = _build(tmp_path)
    x, t, m = cases.dpace_inputs(case)
    N, B, V = x.shape
    lt = {"dpace": 0, "dpace-cumulative-confidence-only": 1, "dpace-continuation-value-only": 2}[case["loss_type"]]
    mm = np.ones((N, B), np.float32) if m is None else m.astype(np.float32)
    header = struct.pack("<iqiqif", 0, N, B, V, lt, case["alpha"])
    loss, g = _run(exe, tmp_path, header, x.astype(np.float32), t.astype(np.int64), mm)
    want, g_ref = odp.dpace_fwd_bwd_torch(torch.from_numpy(x), torch.from_numpy(t), case["alpha"],
                                          None if m is None else torch.from_numpy(m), case["loss_type"])
    assert abs(loss - float(want)) <= 1e-5 * abs(float(want)) + 1e-12
    np.testing.assert_allclose(g.reshape(x.shape), g_ref.numpy(), rtol=0, atol=1e-6)


@pytest.mark.gpu
@pytest.mark.parametrize("case", DFLASH, ids=lambda c: c["name"])
def test_c_host_dflash_matches_oracle(cuda, tmp_path, case):
    exe = _build(tmp_path)
    x, y, m = cases.dflash_inputs(case)
    assert m is None
    N, B, V = x.shape
    kind = {"kl": 0, "ce": 1}[case["kind"]]
    header = struct.pack("<iqiqif", 1, N, B, V, kind, case["gamma"])
    loss, g = _run(exe, tmp_path, header, x.astype(np.float32), y.astype(np.float32))
    want, g_ref = odf.dflash_fwd_bwd_torch(torch.from_numpy(x), torch.from_numpy(y), None, case["gamma"],
                                           False, case["kind"])
    assert abs(loss - float(want)) <= 1e-5 * abs(float(want)) + 1e-12
    np.testing.assert_allclose(g.reshape(x.shape), g_ref.numpy(), rtol=0, atol=1e-6)
