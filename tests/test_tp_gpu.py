"""Batch tensor product on the GPU vs the reference fixtures and the CPU oracle."""

import numpy as np
import pytest
import torch

import tp_oracle as O
from conftest import golden_names, load_golden, oracle_problem, product_problem
from gpu_util import TOL, assert_close, nerr, to_dev

pytestmark = pytest.mark.gpu

DTYPES = [np.float32, np.float64]


def _tp(g, dtype, layout="mul_ir"):
    import openequivariance_b200 as oeq

    return oeq.TensorProduct(product_problem(g, dtype=dtype, layout=layout))


@pytest.mark.parametrize("dtype", DTYPES, ids=["f32", "f64"])
@pytest.mark.parametrize("name", golden_names("tp"))
def test_forward_backward_vs_reference(name, dtype, cuda_device):
    g = load_golden(name)
    tp = _tp(g, dtype)
    perm = g["perm"]
    Z = tp(to_dev(g["X"], dtype), to_dev(g["Y"], dtype), to_dev(g["W_e3nn"][..., perm], dtype))
    assert_close(Z, g["Z"], dtype, "forward")
    x = to_dev(g["bX"], dtype).requires_grad_()
    y = to_dev(g["bY"], dtype).requires_grad_()
    w = to_dev(g["bW_e3nn"][..., perm], dtype).requires_grad_()
    tp(x, y, w).backward(to_dev(g["G"], dtype))
    assert_close(x.grad, g["gX"], dtype, "dX")
    assert_close(y.grad, g["gY"], dtype, "dY")
    assert_close(w.grad, g["gW_oeq"], dtype, "dW")


@pytest.mark.parametrize("dtype", DTYPES, ids=["f32", "f64"])
@pytest.mark.parametrize("name", golden_names("tp"))
def test_double_backward_vs_oracle(name, dtype, cuda_device):
    g = load_golden(name)
    p = oracle_problem(g)
    tp = _tp(g, dtype)
    perm = g["perm"]
    inv = np.argsort(perm)
    rng = np.random.default_rng(5)
    X, Y, W, G = g["bX"], g["bY"], g["bW_e3nn"], g["G"]
    a, b, c = rng.uniform(size=X.shape), rng.uniform(size=Y.shape), rng.uniform(size=W.shape)
    gX, gY, gW, gG = O.double_backward(p, X, Y, W, G, a, b, c)
    ops = torch.ops.libtorch_tp_jit
    out = ops.jit_tp_double_backward(
        tp.kernel, tp.hash, to_dev(X, dtype), to_dev(Y, dtype), to_dev(W[..., perm], dtype),
        to_dev(G, dtype), to_dev(a, dtype), to_dev(b, dtype), to_dev(c[..., perm], dtype))
    assert_close(out[0], gX, dtype, "ddX")
    assert_close(out[1], gY, dtype, "ddY")
    assert_close(out[2].detach().cpu().numpy()[..., inv], gW, dtype, "ddW")
    assert_close(out[3], gG, dtype, "ddZ")


@pytest.mark.parametrize("name", ["tp_mace_large.npz", "tp_uvu_16x40_l111.npz",
                                  "tp_uvu_33_l222.npz", "tp_uvu_l725.npz"])
def test_ir_mul_layout(name, cuda_device):
    from openequivariance_b200.utils import transpose_irrep_layout

    g = load_golden(name)
    dtype = np.float64
    p = product_problem(g, dtype=dtype)
    tp = _tp(g, dtype, layout="ir_mul")
    X = transpose_irrep_layout(g["X"], p.irreps_in1, "mul_ir", "ir_mul")
    Y = transpose_irrep_layout(g["Y"], p.irreps_in2, "mul_ir", "ir_mul")
    Z = tp(to_dev(X, dtype), to_dev(Y, dtype), to_dev(g["W_e3nn"][..., g["perm"]], dtype))
    Zm = transpose_irrep_layout(Z.cpu().numpy(), p.irreps_out, "ir_mul", "mul_ir")
    assert nerr(Zm, g["Z"]) <= TOL[dtype]
    x = to_dev(transpose_irrep_layout(g["bX"], p.irreps_in1, "mul_ir", "ir_mul"), dtype)
    y = to_dev(transpose_irrep_layout(g["bY"], p.irreps_in2, "mul_ir", "ir_mul"), dtype)
    w = to_dev(g["bW_e3nn"][..., g["perm"]], dtype)
    G = to_dev(transpose_irrep_layout(g["G"], p.irreps_out, "mul_ir", "ir_mul"), dtype)
    x.requires_grad_(), y.requires_grad_(), w.requires_grad_()
    tp(x, y, w).backward(G)
    gx = transpose_irrep_layout(x.grad.cpu().numpy(), p.irreps_in1, "ir_mul", "mul_ir")
    gy = transpose_irrep_layout(y.grad.cpu().numpy(), p.irreps_in2, "ir_mul", "mul_ir")
    assert nerr(gx, g["gX"]) <= TOL[dtype]
    assert nerr(gy, g["gY"]) <= TOL[dtype]
    assert nerr(w.grad, g["gW_oeq"]) <= TOL[dtype]


def test_triple_backward_matches_finite_difference(cuda_device):
    """Third derivative through autograd (create_graph twice) vs the oracle's algebra."""
    g = load_golden("tp_uvu_33_l222.npz")
    dtype = np.float64
    tp = _tp(g, dtype)
    rng = np.random.default_rng(11)
    B = 3
    X = to_dev(rng.normal(size=(B, g["X"].shape[1])), dtype).requires_grad_()
    Y = to_dev(rng.normal(size=(B, g["Y"].shape[1])), dtype).requires_grad_()
    W = to_dev(rng.normal(size=(B, int(g["weight_numel"]))), dtype).requires_grad_()
    ok = torch.autograd.gradcheck(lambda a, b, c: tp(a, b, c), (X, Y, W), eps=1e-6, atol=1e-8)
    assert ok
    ok = torch.autograd.gradgradcheck(lambda a, b, c: tp(a, b, c), (X, Y, W), eps=1e-6,
                                      atol=1e-7)
    assert ok

    def grads(a, b, c):
        out = tp(a, b, c)
        ga, gb, gc = torch.autograd.grad(out.pow(2).sum(), (a, b, c), create_graph=True)
        return ga.pow(2).sum() + gb.pow(2).sum() + gc.pow(2).sum()

    ok = torch.autograd.gradcheck(grads, (X, Y, W), eps=1e-6, atol=1e-6)
    assert ok


def test_shared_weights_and_to_dtype(cuda_device):
    g = load_golden("tp_mace_medium_shared.npz")
    tp = _tp(g, np.float32)
    tp.to(torch.float64)
    Z = tp(to_dev(g["X"], np.float64), to_dev(g["Y"], np.float64),
           to_dev(g["W_e3nn"][g["perm"]], np.float64))
    assert nerr(Z, g["Z"]) <= TOL[np.float64]


def test_empty_batch(cuda_device):
    g = load_golden("tp_c1.npz")
    tp = _tp(g, np.float32)
    Z = tp(torch.zeros(0, 5, device="cuda"), torch.zeros(0, 7, device="cuda"),
           torch.zeros(0, 1, device="cuda"))
    assert Z.shape == (0, 5)


def test_input_validation_messages(cuda_device):
    g = load_golden("tp_c1.npz")
    tp = _tp(g, np.float32)
    X, Y, W = (torch.rand(10, 5, device="cuda"), torch.rand(10, 7, device="cuda"),
               torch.rand(10, 1, device="cuda"))
    tp(X, Y, W)
    with pytest.raises(RuntimeError, match="Shape mismatch"):
        tp(X.unsqueeze(1), Y, W)
    with pytest.raises(RuntimeError, match="Shape mismatch"):
        tp(X, torch.rand(10, 8, device="cuda"), W)
    with pytest.raises(RuntimeError, match="is not on the GPU"):
        tp(X, Y.cpu(), W)
    with pytest.raises(RuntimeError, match="Dtype mismatch"):
        tp(X, Y, W.to(torch.bfloat16))


def _kernel_names(fn):
    from torch.profiler import ProfilerActivity, profile

    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        fn()
        torch.cuda.synchronize()
    return {e.name for e in prof.events() if e.device_type.name == "CUDA"}


@pytest.mark.parametrize("name", ["tp_c2_literal.npz", "tp_mace_medium_shared.npz"])
def test_lockstep_many_rows(name, cuda_device):
    """The C2-shape forward and backward over 997 rows (ragged for every row-block size), so
    the kernels' rings of W / dZ slots wrap many times and both row buffers are reused, vs the
    fp64 oracle."""
    g = load_golden(name)
    p = oracle_problem(g)
    dtype = np.float32
    tp = _tp(g, dtype)
    perm = g["perm"]
    inv = np.argsort(perm)
    rng = np.random.default_rng(3)
    B = 997
    X = rng.normal(size=(B, g["X"].shape[1]))
    Y = rng.normal(size=(B, g["Y"].shape[1]))
    shared = bool(g["shared_weights"])
    W = rng.normal(size=(int(g["weight_numel"]),) if shared else (B, int(g["weight_numel"])))
    G = rng.normal(size=(B, g["Z"].shape[1]))
    gX, gY, gW = O.backward(p, X, Y, W[..., inv], G)
    Zref = O.forward(p, X, Y, W[..., inv])
    xs, ys, ws = to_dev(X, dtype), to_dev(Y, dtype), to_dev(W, dtype)
    out = {}
    names = _kernel_names(lambda: out.update(Z=tp(xs, ys, ws)))
    if name == "tp_c2_literal.npz":
        assert any("tp_fwd_lk" in n for n in names), sorted(names)
    assert_close(out["Z"], Zref, dtype, "Z")
    x = to_dev(X, dtype).requires_grad_()
    y = to_dev(Y, dtype).requires_grad_()
    w = to_dev(W, dtype).requires_grad_()
    names = _kernel_names(lambda: tp(x, y, w).backward(to_dev(G, dtype)))
    assert any("tp_bwd_lk" in n for n in names), sorted(names)
    assert_close(x.grad, gX, dtype, "dX")
    assert_close(y.grad, gY, dtype, "dY")
    assert_close(w.grad.cpu().numpy()[..., inv], gW, dtype, "dW")
