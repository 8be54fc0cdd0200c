"""Generate the golden vectors in tests/golden/ from the REFERENCE's own oracles.

Runs only where a checkout of the reference exists; its path is the required
argument (or $SPECDEC_REF). It evaluates, on the CPU and in float32:
  - losses/dpace_ref.py::d_pace_loss (loaded by file path: the package
    __init__ imports cupy), with torch autograd for the gradient;
  - the specforge oracle _naive_dpace_weight / oracle_loss and the speculators
    oracle EPS / dflash_loss_decay / kl_div_loss / ce_loss / loss_function,
    lifted out of the reference's test scripts by AST (those scripts import
    cupy and run their checks at import time, so they cannot be imported);
on the seeded inputs of tests/golden/cases.py, and writes
dpace_golden.npz / dflash_golden.npz (+ a readable golden_summary.json).

    python tests/golden/make_golden.py <path of the reference checkout>
"""
from __future__ import annotations

import ast
import importlib.util
import json
import os
import sys

import numpy as np
import torch
import torch.nn.functional as F

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import cases  # noqa: E402

REF = None  # the reference checkout: argv[1] or $SPECDEC_REF


def load_module_by_path(name: str, path: str):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def lift_definitions(path: str, names: set[str]) -> dict:
    """Execute only the named top-level defs/assignments of a script."""
    tree = ast.parse(open(path).read(), filename=path)
    keep = []
    for node in tree.body:
        if isinstance(node, ast.FunctionDef) and node.name in names:
            keep.append(node)
        elif isinstance(node, ast.Assign) and any(
                isinstance(t, ast.Name) and t.id in names for t in node.targets):
            keep.append(node)
    found = {n.name if isinstance(n, ast.FunctionDef) else n.targets[0].id for n in keep}
    missing = names - found
    if missing:
        raise RuntimeError(f"{path}: definitions not found: {sorted(missing)}")
    ns = {"torch": torch, "F": F, "np": np}
    exec(compile(ast.Module(body=keep, type_ignores=[]), path, "exec"), ns)
    return ns


def store_grad(out: dict, key: str, case: dict, grad: np.ndarray) -> None:
    flat = grad.reshape(-1)
    if flat.size <= cases.FULL_GRAD_MAX:
        out[f"{key}/grad"] = grad.astype(np.float32)
    else:
        idx = cases.probe_indices(case, flat.size)
        out[f"{key}/probe_idx"] = idx
        out[f"{key}/probe_val"] = flat[idx].astype(np.float32)
    out[f"{key}/grad_abs_sum"] = np.array(np.abs(grad.astype(np.float64)).sum())


def main() -> None:
    torch.set_num_threads(os.cpu_count() or 1)
    ref_dpace = load_module_by_path("ref_dpace_ref", os.path.join(REF, "losses", "dpace_ref.py"))
    spec_dpace = lift_definitions(os.path.join(REF, "losses", "tests", "test_dpace.py"),
                                  {"_naive_dpace_weight", "oracle_loss"})
    spec_dflash = lift_definitions(os.path.join(REF, "models", "dflash", "tests", "test_loss.py"),
                                   {"EPS", "dflash_loss_decay", "kl_div_loss", "ce_loss",
                                    "loss_function"})
    summary = {"dpace": {}, "dflash": {}}

    out = {}
    for case in cases.DPACE_CASES:
        x, t, m = cases.dpace_inputs(case)
        key = case["name"]
        xt = torch.from_numpy(x).requires_grad_(True)
        tt = torch.from_numpy(t)
        mt = None if m is None else torch.from_numpy(m)
        loss = ref_dpace.d_pace_loss(xt, tt, case["alpha"], mt, case["loss_type"])
        loss.backward()
        with torch.no_grad():
            loss_spec = spec_dpace["oracle_loss"](torch.from_numpy(x), tt, case["alpha"], mt,
                                                  case["loss_type"])
        out[f"{key}/sha256"] = np.array(cases.digest(x, t, m))
        out[f"{key}/loss"] = np.array(float(loss.detach()), dtype=np.float32)
        out[f"{key}/loss_spec"] = np.array(float(loss_spec), dtype=np.float32)
        store_grad(out, key, case, xt.grad.numpy())
        summary["dpace"][key] = {"loss": float(loss.detach()), "loss_spec": float(loss_spec)}
        print(f"dpace  {key:40s} loss={float(loss.detach()):.7g} spec={float(loss_spec):.7g}")
    np.savez_compressed(os.path.join(HERE, "dpace_golden.npz"), **out)

    out = {}
    kind_fn = {"kl": spec_dflash["kl_div_loss"], "ce": spec_dflash["ce_loss"]}
    for case in cases.DFLASH_CASES:
        x, y, m = cases.dflash_inputs(case)
        key = case["name"]
        N, B, V = x.shape
        bs = B if case["block_size"] is None else case["block_size"]
        xt = torch.from_numpy(x).requires_grad_(True)
        yt = torch.from_numpy(y)
        mt = torch.ones((N, B)) if m is None else torch.from_numpy(m)
        pos = torch.arange(B).view(1, -1) % bs
        loss = spec_dflash["loss_function"](xt, yt, mt, pos, kind_fn[case["kind"]], case["gamma"],
                                            case["sfa"])
        loss.backward()
        out[f"{key}/sha256"] = np.array(cases.digest(x, y, m))
        out[f"{key}/loss"] = np.array(float(loss.detach()), dtype=np.float32)
        store_grad(out, key, case, xt.grad.numpy())
        summary["dflash"][key] = {"loss": float(loss.detach())}
        print(f"dflash {key:40s} loss={float(loss.detach()):.7g}")
    np.savez_compressed(os.path.join(HERE, "dflash_golden.npz"), **out)

    with open(os.path.join(HERE, "golden_summary.json"), "w") as f:
        json.dump(summary, f, indent=1, sort_keys=True)


if __name__ == "__main__":
    REF = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("SPECDEC_REF")
    if not REF or not os.path.isdir(REF):
        sys.exit("usage: make_golden.py <path of the reference checkout> (or set SPECDEC_REF)")
    main()
