"""SymmetricContraction module: reference parity on CPU (torch formulation) and on the GPU
(fused kernels), group_gemm against a dense evaluation, gradients of every order."""

import glob
import os
import sys

import numpy as np
import pytest
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
sys.path.insert(0, os.path.join(os.path.dirname(HERE), "oracle"))

import openequivariance_b200 as oeq  # noqa: E402
import sc_oracle as SO  # noqa: E402

FIXTURES = sorted(glob.glob(os.path.join(HERE, "golden", "sc_*.npz")))
IDS = [os.path.basename(p)[3:-4] for p in FIXTURES]


def _module(d, dtype=torch.float64):
    corr, ne = (int(v) for v in d["meta"])
    torch.manual_seed(12345)  # the reference fixture's seed: weights must come out identical
    return oeq.SymmetricContraction(str(d["irreps_in"]), str(d["irreps_out"]), correlation=corr,
                                    num_elements=ne, dtype=dtype)


def _run(mod, d, device, dtype):
    x = torch.tensor(d["x"], dtype=dtype, device=device, requires_grad=True)
    ne = int(d["meta"][1])
    y = torch.nn.functional.one_hot(torch.tensor(d["labels"]), num_classes=ne).to(dtype).to(device)
    out = mod(x, y)
    params = []
    for c in mod.contractions:
        params += [c.weights_max] + list(c.weights)
    g = torch.tensor(d["grad_out"], dtype=dtype, device=device)
    grads = torch.autograd.grad((out * g).sum(), [x] + params)
    return out, grads


def _nerr(a, b):
    a = np.asarray(a.detach().cpu().double().numpy() if torch.is_tensor(a) else a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return np.abs(a - b).max() / max(np.abs(b).max(), 1e-30)


def _check(d, out, grads, tol):
    """Normalised max error (max |a - b| / max |b|) of the output and every gradient."""
    pairs = [("out", out, d["out"]), ("grad_x", grads[0], d["grad_x"])]
    corr = int(d["meta"][0])
    gi = 1
    for ci in range((len(grads) - 1) // corr):
        pairs.append((f"c{ci}.weights_max", grads[gi], d[f"c{ci}_grad_weights_max"]))
        gi += 1
        for i in range(corr - 1):
            pairs.append((f"c{ci}.weights[{i}]", grads[gi], d[f"c{ci}_grad_weights_{i}"]))
            gi += 1
    for what, got, want in pairs:
        e = _nerr(got, want)
        assert e <= tol, f"{what}: normalised max error {e:.3e} > {tol:.0e}"


@pytest.mark.parametrize("path", FIXTURES, ids=IDS)
def test_seeded_weights_and_buffers_match_reference(path):
    d = np.load(path)
    mod = _module(d)
    for ci, c in enumerate(mod.contractions):
        np.testing.assert_array_equal(c.weights_max.detach().numpy(), d[f"c{ci}_weights_max"])
        for i, w in enumerate(c.weights):
            np.testing.assert_array_equal(w.detach().numpy(), d[f"c{ci}_weights_{i}"])
        for nu in range(1, c.correlation + 1):
            np.testing.assert_allclose(c.U_tensors(nu).numpy(), d[f"c{ci}_U{nu}"], atol=1e-12)


@pytest.mark.parametrize("path", FIXTURES, ids=IDS)
def test_cpu_monomial_formulation_matches_reference(path):
    """The weight folding onto monomials (``coefficients``), evaluated by the differentiable
    torch form of the polynomial on the CPU, reproduces the reference module's outputs and
    every gradient.  (The module itself runs only the fused GPU kernels.)"""
    from openequivariance_b200.symmetric_contraction import _torch_contraction

    d = np.load(path)
    mod = _module(d)
    x = torch.tensor(d["x"], dtype=torch.float64, requires_grad=True)
    ne = int(d["meta"][1])
    elem = torch.tensor(d["labels"])
    out = _torch_contraction(mod, x, mod.coefficients(), elem)
    params = []
    for c in mod.contractions:
        params += [c.weights_max] + list(c.weights)
    g = torch.tensor(d["grad_out"], dtype=torch.float64)
    grads = torch.autograd.grad((out * g).sum(), [x] + params)
    assert ne == mod.num_elements
    _check(d, out, grads, 1e-10)


def test_module_refuses_cpu_tensors():
    d = np.load(FIXTURES[0])
    mod = _module(d)
    x = torch.tensor(d["x"], dtype=torch.float64)
    y = torch.nn.functional.one_hot(torch.tensor(d["labels"]), num_classes=int(d["meta"][1]))
    with pytest.raises(RuntimeError, match="is not on the GPU"):
        mod(x, y.double())


# ------------------------------------------------------------------------------- GPU

def _normalized_err(a, b):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return np.abs(a - b).max() / max(np.abs(b).max(), 1e-30)


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float64, torch.float32], ids=["f64", "f32"])
@pytest.mark.parametrize("path", FIXTURES, ids=IDS)
def test_gpu_fused_matches_reference(path, dtype):
    d = np.load(path)
    mod = _module(d, torch.float64).to(dtype).cuda()
    assert mod.fused_ok, "fixture shapes are in the fused kernels' range"
    out, grads = _run(mod, d, "cuda", dtype)
    tol = 1e-10 if dtype == torch.float64 else 1e-5
    _check(d, out, grads, tol)


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float64, torch.float32], ids=["f64", "f32"])
def test_gpu_mace_shape_against_oracle(dtype):
    """128x0e+128x1o+128x2e -> 128x0e+128x1o, correlation 3, 10 elements (C5 shape)."""
    n, ne = 2000, 10
    prob = SO.ScProblem("128x0e+128x1o+128x2e", "128x0e+128x1o", 3, ne)
    torch.manual_seed(7)
    mod = oeq.SymmetricContraction("128x0e+128x1o+128x2e", "128x0e+128x1o", correlation=3,
                                   num_elements=ne, dtype=torch.float64)
    g = torch.Generator().manual_seed(11)
    x = torch.randn(n, 128, 9, dtype=torch.float64, generator=g)
    labels = torch.randint(0, ne, (n,), generator=g)
    weights = [[c.weights_max.detach().clone().requires_grad_(True)] +
               [w.detach().clone().requires_grad_(True) for w in c.weights]
               for c in mod.contractions]
    xo = x.clone().requires_grad_(True)
    want = SO.forward(prob, weights, xo, labels)
    G = torch.randn(want.shape, dtype=torch.float64, generator=g)
    flat = [w for ws in weights for w in ws]
    want_grads = torch.autograd.grad((want * G).sum(), [xo] + flat)
    modg = mod.to(dtype).cuda()
    y = torch.nn.functional.one_hot(labels, ne).to(dtype).cuda()
    xg = x.to(dtype).cuda().requires_grad_(True)
    got = modg(xg, y)
    params = [p for c in modg.contractions for p in [c.weights_max] + list(c.weights)]
    got_grads = torch.autograd.grad((got * G.to(dtype).cuda()).sum(), [xg] + params)
    tol = 1e-12 if dtype == torch.float64 else 1e-5
    assert _normalized_err(got.detach().cpu().numpy(), want.detach().numpy()) <= tol
    # Gradients of x and of every weight tensor (weights_max and the lower correlations of
    # both output irreps) at the C5 shape.
    for i, (a, b) in enumerate(zip(got_grads, want_grads)):
        e = _normalized_err(a.cpu().numpy(), b.numpy())
        assert e <= tol, f"gradient {i}: normalised max error {e:.3e}"


@pytest.mark.gpu
def test_gpu_backward_deterministic():
    torch.manual_seed(3)
    mod = oeq.SymmetricContraction("16x0e+16x1o+16x2e", "16x0e+16x1o", correlation=3,
                                   num_elements=4).cuda()
    x = torch.randn(500, 16, 9, device="cuda", requires_grad=True)
    y = torch.nn.functional.one_hot(torch.randint(0, 4, (500,)), 4).float().cuda()
    runs = []
    for _ in range(2):
        out = mod(x, y)
        gx, gw = torch.autograd.grad(out.square().sum(), [x, mod.contractions[1].weights_max])
        runs.append((out, gx, gw))
    for a, b in zip(runs[0], runs[1]):
        assert torch.equal(a, b)


@pytest.mark.gpu
def test_gpu_double_backward_gradcheck():
    torch.manual_seed(5)
    mod = oeq.SymmetricContraction("2x0e+2x1o", "2x0e+2x1o", correlation=2, num_elements=3,
                                   dtype=torch.float64).cuda()
    x = torch.randn(7, 2, 4, dtype=torch.float64, device="cuda", requires_grad=True)
    y = torch.nn.functional.one_hot(torch.tensor([0, 2, 1, 1, 0, 2, 2]), 3).double().cuda()
    w = mod.contractions[0].weights_max
    f = lambda xx, ww: mod(xx, y)  # noqa: E731
    assert torch.autograd.gradcheck(lambda xx: mod(xx, y), (x,))
    assert torch.autograd.gradgradcheck(lambda xx: mod(xx, y), (x,))
    del f, w


@pytest.mark.gpu
@pytest.mark.parametrize("inner", [0, 1])
@pytest.mark.parametrize("dtype", [torch.float64, torch.float32], ids=["f64", "f32"])
def test_group_gemm_op(inner, dtype):
    from openequivariance_b200 import _ops

    _ops.ensure_registered()
    g = torch.Generator().manual_seed(1)
    counts = torch.tensor([3, 0, 5, 2], dtype=torch.int64)
    R, G, b, m, k = int(counts.sum()), 4, 6, 7, 5
    off = np.concatenate([[0], np.cumsum(counts.numpy())])
    if inner == 0:
        A = torch.randn(G, b, m, k, dtype=dtype, generator=g)
        B = torch.randn(R, b, k, dtype=dtype, generator=g)
        want = torch.zeros(R, b, m, dtype=torch.float64)
        for i in range(G):
            want[off[i]:off[i + 1]] = torch.einsum("bmk,rbk->rbm", A[i].double(), B[off[i]:off[i + 1]].double())
    else:
        A = torch.randn(R, b, m, dtype=dtype, generator=g)
        B = torch.randn(R, b, k, dtype=dtype, generator=g)
        want = torch.zeros(G, b, m, k, dtype=torch.float64)
        for i in range(G):
            want[i] = torch.einsum("rbm,rbk->bmk", A[off[i]:off[i + 1]].double(), B[off[i]:off[i + 1]].double())
    got = torch.ops.libtorch_tp_jit.group_gemm(A.cuda(), B.cuda(), counts, G, b, m, k, inner)
    tol = 1e-12 if dtype == torch.float64 else 1e-5
    assert _normalized_err(got.cpu(), want) <= tol
