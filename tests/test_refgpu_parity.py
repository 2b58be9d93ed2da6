"""Parity at the BASELINE configurations' own sizes.

Two anchors:

* the reference's own CUDA kernels: ``tests/golden/refgpu_<case>.npz`` hold their outputs
  (made by ``tests/golden/make_golden_refgpu.py`` on a B200 through the reference's public
  API and JIT route); the inputs are regenerated here from the seeds in
  ``tests/golden/refgpu_cases.py``;
* the fp64 CPU oracle, for C1 literal (1000 rows, seed 0) and the full C3 graph (5,000 nodes,
  839,872 edges), as ``tests/batch_test.py:63-130`` and ``tests/conv_test.py:102-160`` of
  the reference do with e3nn.

Bounds: normalised max error 1e-5 (float32) and 1e-12 (float64), on every element of the
small outputs and, for the large ones, on seeded sample rows and on two sketches that touch
every element (``refgpu_cases.summarise``).
"""

import sys

import numpy as np
import pytest
import torch

from conftest import GOLDEN

sys.path.insert(0, str(GOLDEN))
import refgpu_cases as R  # noqa: E402
import tp_oracle as O  # noqa: E402

pytestmark = pytest.mark.gpu

TOL = {"float32": 1e-5, "float64": 1e-12}


def _fixture(name):
    path = GOLDEN / f"refgpu_{name}.npz"
    if not path.exists():
        pytest.skip(f"{path.name} not generated")
    with np.load(path, allow_pickle=False) as f:
        return {k: f[k] for k in f.files}


def _problem(case, dtype):
    from openequivariance_b200.irreps import TPProblem

    in1, in2, out, ins, mode, shared = case[:6]
    return TPProblem(in1, in2, out, [(i, j, k, mode, True) for i, j, k in ins],
                     shared_weights=shared, internal_weights=False, irrep_dtype=dtype,
                     weight_dtype=dtype)


def _check(key, got, fx, tol):
    err = R.compare(key, got.detach().double().cpu().numpy(), fx)
    assert err <= tol, f"{key}: normalised max error {err:.3e} > {tol:.0e}"
    return err


@pytest.mark.parametrize("name", sorted(R.TP_CASES))
def test_tp_matches_reference_kernels(name, cuda_device):
    import openequivariance_b200 as oeq

    fx = _fixture(name)
    case = R.TP_CASES[name]
    dt = np.float32 if case[6] == "float32" else np.float64
    tdt = torch.float32 if dt == np.float32 else torch.float64
    tol = TOL[case[6]]
    tp = oeq.TensorProduct(_problem(case, dt))
    X, Y, W, dZ, ddX, ddY, ddW = (torch.tensor(a, dtype=tdt, device="cuda")
                                  for a in R.tp_inputs(name))
    x, y, w = (t.clone().requires_grad_(True) for t in (X, Y, W))
    dbl = name in R.DOUBLE_BACKWARD
    z = tp(x, y, w)
    _check("Z", z, fx, tol)
    g = dZ.clone().requires_grad_(dbl)
    gx, gy, gw = torch.autograd.grad(z, (x, y, w), g, create_graph=dbl)
    _check("dX", gx, fx, tol)
    _check("dY", gy, fx, tol)
    _check("dW", gw, fx, tol)
    if dbl:
        s = (gx * ddX).sum() + (gy * ddY).sum() + (gw * ddW).sum()
        ax, ay, aw, ag = torch.autograd.grad(s, (x, y, w, g))
        _check("ddbl:X", ax, fx, tol)
        _check("ddbl:Y", ay, fx, tol)
        _check("ddbl:W", aw, fx, tol)
        _check("ddbl:dZ", ag, fx, tol)


@pytest.fixture(scope="module")
def c3():
    rows, cols, tperm = R.c3_graph()
    return rows, cols, tperm, R.conv_inputs(rows.size)


@pytest.mark.parametrize("mode", ["atomic", "deterministic"])
def test_c3_conv_matches_reference_kernels(mode, c3, cuda_device):
    import openequivariance_b200 as oeq

    fx = _fixture("c3")
    rows, cols, tperm, (X, Y, W, dZ) = c3
    assert str(fx["graph_digest"]) == R.graph_digest(rows, cols)
    conv = oeq.TensorProductConv(_problem(R.CONV_CASE, np.float32),
                                 deterministic=mode == "deterministic")
    dev = lambda a: torch.tensor(a, device="cuda")  # noqa: E731
    x, y, w = (dev(a).requires_grad_(True) for a in (X, Y, W))
    z = conv(x, y, w, dev(rows), dev(cols), dev(tperm) if mode == "deterministic" else None)
    _check(f"{mode}:Z", z, fx, 1e-5)
    gx, gy, gw = torch.autograd.grad(z, (x, y, w), dev(dZ))
    _check(f"{mode}:dX", gx, fx, 1e-5)
    _check(f"{mode}:dY", gy, fx, 1e-5)
    _check(f"{mode}:dW", gw, fx, 1e-5)


def test_c1_literal_vs_oracle(cuda_device):
    """C1 exactly as BASELINE states it: 1000 rows, uniform[0, 1) from seed 0, float32."""
    import openequivariance_b200 as oeq

    case = R.TP_CASES["c1"]
    X, Y, W, dZ, *_ = R.tp_inputs("c1")
    op = O.make_problem(case[0], case[1], case[2], [(0, 0, 0, "uvu", True)])
    tp = oeq.TensorProduct(_problem(case, np.float32))
    x, y, w = (torch.tensor(a, device="cuda", requires_grad=True) for a in (X, Y, W))
    z = tp(x, y, w)
    X64, Y64, W64, G64 = (a.astype(np.float64) for a in (X, Y, W, dZ))
    assert O.normalized_max_error(z.detach().double().cpu().numpy(),
                                  O.forward(op, X64, Y64, W64)) <= 1e-5
    z.backward(torch.tensor(dZ, device="cuda"))
    want = O.backward(op, X64, Y64, W64, G64)
    for got, ref in zip((x.grad, y.grad, w.grad), want):
        assert O.normalized_max_error(got.double().cpu().numpy(), ref) <= 1e-5


@pytest.mark.parametrize("mode", ["atomic", "deterministic"])
def test_c3_full_graph_vs_oracle(mode, c3, cuda_device):
    """The whole C3 graph (839,872 edges) against the fp64 oracle, forward and backward."""
    import openequivariance_b200 as oeq

    rows, cols, tperm, (X, Y, W, dZ) = c3
    op = O.make_problem(*R.CONV_CASE[:3], [(0, 0, 0, "uvu", True)])
    conv = oeq.TensorProductConv(_problem(R.CONV_CASE, np.float32),
                                 deterministic=mode == "deterministic")
    dev = lambda a: torch.tensor(a, device="cuda")  # noqa: E731
    x, y, w = (dev(a).requires_grad_(True) for a in (X, Y, W))
    z = conv(x, y, w, dev(rows), dev(cols), dev(tperm) if mode == "deterministic" else None)
    X64, Y64, W64, G64 = (a.astype(np.float64) for a in (X, Y, W, dZ))
    assert O.normalized_max_error(z.detach().double().cpu().numpy(),
                                  O.conv_forward(op, X64, Y64, W64, rows, cols)) <= 1e-5
    z.backward(dev(dZ))
    want = O.conv_backward(op, X64, Y64, W64, G64, rows, cols)
    for what, got, ref in zip(("dX", "dY", "dW"), (x.grad, y.grad, w.grad), want):
        e = O.normalized_max_error(got.double().cpu().numpy(), ref)
        assert e <= 1e-5, f"{what}: {e:.3e}"


def test_c3_graph_built_on_device_matches(cuda_device):
    """The device radius graph (cell list, receiver sort, transpose permutation) gives the
    same C3 edge list as scipy's periodic KD-tree, in the reference's ``CoordGraph`` order."""
    from openequivariance_b200.graph import radius_graph

    rows, cols, tperm = R.c3_graph()
    rng = np.random.default_rng(0)
    pos = torch.tensor(rng.uniform(0.0, R.C3_BOX, size=(R.C3_NODES, 3)), device="cuda")
    r, c, t, _ = radius_graph(pos, R.C3_BOX, R.C3_CUTOFF)
    assert r.numel() == R.C3_EDGES
    assert R.graph_digest(r.cpu().numpy(), c.cpu().numpy()) == R.graph_digest(rows, cols)
    assert np.array_equal(t.cpu().numpy(), tperm)
