"""Runs the reference's own CUDA kernels on the BASELINE-size cases and saves their outputs.

Usage (on a machine with a GPU and the reference's Python package installed somewhere):

    OEQ_REFERENCE_PKG=<dir holding the openequivariance package> \\
        python tests/golden/make_golden_refgpu.py --out <dir>

The reference package is used as shipped, through its public API (``oeq.TPProblem``,
``oeq.TensorProduct``, ``oeq.TensorProductConv``) and its JIT route
(``OEQ_JIT_EXTENSION=1``: ``torch.utils.cpp_extension.load`` of its torch extension,
``_torch/extlib/__init__.py:83-201``, then NVRTC per problem for the device's architecture,
``extension/backend/backend_cuda.hpp:199-301``).  That extension registers the
``libtorch_tp_jit`` operators, as this repository's shim does, so this script never imports
``openequivariance_b200``.

For every case of ``refgpu_cases`` it writes ``refgpu_<case>.npz``: the forward output, the
gradients of a seeded upstream gradient (and, for ``DOUBLE_BACKWARD`` cases, the double
backward), each summarised by ``refgpu_cases.summarise``; plus the device name and the
reference version.  The convolution case also stores the graph's digest.
"""

from __future__ import annotations

import argparse
import os
import sys
import time
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
import refgpu_cases as R  # noqa: E402


def _import_reference():
    pkg = os.environ.get("OEQ_REFERENCE_PKG")
    if not pkg:
        sys.exit("set OEQ_REFERENCE_PKG to the directory that holds the reference's "
                 "openequivariance package")
    os.environ["OEQ_JIT_EXTENSION"] = "1"
    sys.path.insert(0, str(Path(pkg).resolve()))
    import openequivariance as oeq

    return oeq


def _problem(oeq, case, dtype):
    in1, in2, out, ins, mode, shared = case[:6]
    return oeq.TPProblem(in1, in2, out, [(i, j, k, mode, True) for i, j, k in ins],
                         shared_weights=shared, internal_weights=False,
                         irrep_dtype=dtype, weight_dtype=dtype)


def run_tp(oeq, torch, name, outdir):
    case = R.TP_CASES[name]
    dt = np.float32 if case[6] == "float32" else np.float64
    tdt = torch.float32 if dt == np.float32 else torch.float64
    tp = oeq.TensorProduct(_problem(oeq, case, dt), torch_op=True)
    X, Y, W, dZ, ddX, ddY, ddW = (torch.tensor(a, dtype=tdt, device="cuda") for a in R.tp_inputs(name))
    x, y, w = (t.clone().requires_grad_(True) for t in (X, Y, W))
    z = tp(x, y, w)
    gx, gy, gw = torch.autograd.grad(z, (x, y, w), dZ, create_graph=name in R.DOUBLE_BACKWARD)
    res = {}
    R.summarise("Z", z.detach().cpu().numpy(), res)
    R.summarise("dX", gx.detach().cpu().numpy(), res)
    R.summarise("dY", gy.detach().cpu().numpy(), res)
    R.summarise("dW", gw.detach().cpu().numpy(), res)
    if name in R.DOUBLE_BACKWARD:
        # Double backward through the reference's autograd: the gradient of
        # <dX, ddX> + <dY, ddY> + <dW, ddW> with respect to x, y, w and dZ.
        g = torch.tensor(R.tp_inputs(name)[3], dtype=tdt, device="cuda").requires_grad_(True)
        z2 = tp(x, y, w)
        hx, hy, hw = torch.autograd.grad(z2, (x, y, w), g, create_graph=True)
        s = (hx * ddX).sum() + (hy * ddY).sum() + (hw * ddW).sum()
        ax, ay, aw, ag = torch.autograd.grad(s, (x, y, w, g))
        R.summarise("ddbl:X", ax.cpu().numpy(), res)
        R.summarise("ddbl:Y", ay.cpu().numpy(), res)
        R.summarise("ddbl:W", aw.cpu().numpy(), res)
        R.summarise("ddbl:dZ", ag.cpu().numpy(), res)
    return res


def run_conv(oeq, torch, outdir):
    rows, cols, tperm = R.c3_graph()
    assert rows.size == R.C3_EDGES, rows.size
    X, Y, W, dZ = R.conv_inputs(rows.size)
    prob = _problem(oeq, R.CONV_CASE, np.float32)
    dev = lambda a: torch.tensor(a, device="cuda")  # noqa: E731
    r, c, t = dev(rows), dev(cols), dev(tperm)
    res = {"graph_digest": np.array(R.graph_digest(rows, cols))}
    for mode in ("atomic", "deterministic"):
        conv = oeq.TensorProductConv(prob, deterministic=mode == "deterministic", torch_op=True)
        x, y, w = (dev(a).requires_grad_(True) for a in (X, Y, W))
        z = conv(x, y, w, r, c, t if mode == "deterministic" else None)
        gx, gy, gw = torch.autograd.grad(z, (x, y, w), dev(dZ))
        R.summarise(f"{mode}:Z", z.detach().cpu().numpy(), res)
        R.summarise(f"{mode}:dX", gx.cpu().numpy(), res)
        R.summarise(f"{mode}:dY", gy.cpu().numpy(), res)
        R.summarise(f"{mode}:dW", gw.cpu().numpy(), res)
    return res


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", required=True)
    ap.add_argument("--cases", default="c1,c2,c2ml,c4_f32,c4_f64,c3")
    args = ap.parse_args()
    oeq = _import_reference()
    import torch

    outdir = Path(args.out)
    outdir.mkdir(parents=True, exist_ok=True)
    meta = {"device": np.array(torch.cuda.get_device_name(0)),
            "reference_version": np.array(getattr(oeq, "__version__", "0.7.0"))}
    for name in args.cases.split(","):
        t0 = time.time()
        res = run_conv(oeq, torch, outdir) if name == "c3" else run_tp(oeq, torch, name, outdir)
        torch.cuda.synchronize()
        res.update(meta)
        np.savez_compressed(outdir / f"refgpu_{name}.npz", **res)
        print(f"{name}: {len(res)} arrays in {time.time() - t0:.1f} s", flush=True)


if __name__ == "__main__":
    main()
