"""Shared-weight uvw problems (BASELINE config C4 shape) vs the CPU oracle.

The forward of the NequIP-shaped problem (32 channels per irrep, l <= 2, shared weights,
float32) runs on the tensor cores (``tp_uvw_tc_fwd``); the backward of this class (float32
and float64) runs on ``tp_uvw_sw_dxy`` / ``tp_uvw_sw_dw``.  Results must stay within the
bounds (normalised max error 1e-5 fp32, 1e-12 fp64) on partial tiles, many tiles, and
problems whose output irreps are ordered differently or receive no instruction.
"""

import numpy as np
import pytest
import torch

import tp_oracle as O
from gpu_util import TOL, nerr, to_dev

pytestmark = pytest.mark.gpu


def _fc(in1, in2, out):
    from openequivariance_b200.problems import fully_connected_tpp

    return fully_connected_tpp(in1, in2, out, shared_weights=True, internal_weights=False,
                               irrep_dtype=np.float32, weight_dtype=np.float32)


def _oracle(p):
    ins = [(i.i_in1, i.i_in2, i.i_out, i.connection_mode, True) for i in p.instructions]
    return O.make_problem(str(p.irreps_in1), str(p.irreps_in2), str(p.irreps_out), ins,
                          shared_weights=True)


def _kernel_names(fn):
    from torch.profiler import ProfilerActivity, profile

    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        fn()
        torch.cuda.synchronize()
    return [e.name for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA]


C4 = ("32x0e+32x0o+32x1e+32x1o+32x2e+32x2o", "1x0e+1x1o+1x2e",
      "32x0e+32x0o+32x1e+32x1o+32x2e+32x2o")


@pytest.mark.parametrize("dtype", [np.float32, np.float64], ids=["f32", "f64"])
@pytest.mark.parametrize("rows", [1, 6, 127, 128, 129, 1000])
def test_c4_forward_vs_oracle(rows, dtype, cuda_device):
    """float32: tcgen05 kernel; float64: the CUDA-core kernel of the same class."""
    import openequivariance_b200 as oeq
    from openequivariance_b200.problems import fully_connected_tpp

    p = fully_connected_tpp(*C4, shared_weights=True, internal_weights=False,
                            irrep_dtype=dtype, weight_dtype=dtype)
    op = _oracle(p)
    perm = O.oeq_permutation(op)
    rng = np.random.default_rng(rows)
    X = rng.normal(size=(rows, p.irreps_in1.dim))
    Y = rng.normal(size=(rows, p.irreps_in2.dim))
    W = rng.normal(size=(p.weight_numel,)) / np.sqrt(32 * 5)
    tp = oeq.TensorProduct(p)
    xs, ys, ws = to_dev(X, dtype), to_dev(Y, dtype), to_dev(W[perm], dtype)
    names = _kernel_names(lambda: tp(xs, ys, ws))
    want = "tp_uvw_tc_fwd" if dtype == np.float32 else "tp_uvw_sw_fwd"
    assert any(want in n for n in names), names
    e = nerr(tp(xs, ys, ws), O.forward(op, X, Y, W))
    assert e <= TOL[dtype], f"normalised max error {e:.3e}"


def test_c4_forward_runs_on_tensor_cores_and_matches_fp64(cuda_device):
    """Full C4 batch (20,000 rows) against the float64 kernels on the same inputs."""
    import openequivariance_b200 as oeq
    from openequivariance_b200.problems import baseline_problem

    p32, p64 = baseline_problem("c4", np.float32), baseline_problem("c4", np.float64)
    B = 20000
    g = torch.Generator(device="cuda").manual_seed(3)
    X = torch.randn(B, p32.irreps_in1.dim, device="cuda", dtype=torch.float64, generator=g)
    Y = torch.randn(B, p32.irreps_in2.dim, device="cuda", dtype=torch.float64, generator=g)
    W = torch.randn(p32.weight_numel, device="cuda", dtype=torch.float64, generator=g) / 12.6
    tp32, tp64 = oeq.TensorProduct(p32), oeq.TensorProduct(p64)
    Z64 = tp64(X, Y, W)
    X32, Y32, W32 = X.float(), Y.float(), W.float()
    names = _kernel_names(lambda: tp32(X32, Y32, W32))
    assert any("tp_uvw_tc_fwd" in n for n in names), names
    Z32 = tp32(X32, Y32, W32)
    e = nerr(Z32, Z64.cpu().numpy())
    assert e <= TOL[np.float32], f"normalised max error {e:.3e}"
    # Same inputs, same result (the schedule is fixed).
    assert torch.equal(Z32, tp32(X32, Y32, W32))


def test_unfed_output_irrep_and_mixed_order(cuda_device):
    """Outputs in non-sorted order, one of them (2e) fed by no instruction: zeros there."""
    import openequivariance_b200 as oeq

    p = _fc("32x1o+32x0e", "1x1o", "32x2o+32x1o+32x0e+32x2e+32x1e")
    # 1o x 1o -> 0e, 1e, 2e; 0e x 1o -> 1o.  Keep every instruction except the one into 2e.
    keep = [(i.i_in1, i.i_in2, i.i_out, "uvw", True) for i in p.instructions
            if str(p.irreps_out[i.i_out][1]) != "2e"]
    from openequivariance_b200.irreps import TPProblem

    p = TPProblem(p.irreps_in1, p.irreps_in2, p.irreps_out, keep, shared_weights=True,
                  internal_weights=False, irrep_dtype=np.float32, weight_dtype=np.float32)
    op = _oracle(p)
    perm = O.oeq_permutation(op)
    rng = np.random.default_rng(9)
    rows = 333
    X = rng.normal(size=(rows, p.irreps_in1.dim))
    Y = rng.normal(size=(rows, p.irreps_in2.dim))
    W = rng.normal(size=(p.weight_numel,))
    tp = oeq.TensorProduct(p)
    xs, ys, ws = to_dev(X, np.float32), to_dev(Y, np.float32), to_dev(W[perm], np.float32)
    names = _kernel_names(lambda: tp(xs, ys, ws))
    assert any("tp_uvw_tc_fwd" in n for n in names), names
    Z = tp(xs, ys, ws)
    want = O.forward(op, X, Y, W)
    assert nerr(Z, want) <= TOL[np.float32]
    off = p.irreps_out.slices()[3]
    assert torch.count_nonzero(Z[:, off]).item() == 0
    # Backward of the same problem (every input irrep is read; the 2e output gets no path).
    G = rng.normal(size=(rows, p.irreps_out.dim))
    x, y, w = (t.clone().requires_grad_() for t in (xs, ys, ws))
    tp(x, y, w).backward(to_dev(G, np.float32))
    gX, gY, gW = O.backward(op, X, Y, W, G)
    assert nerr(x.grad, gX) <= TOL[np.float32]
    assert nerr(y.grad, gY) <= TOL[np.float32]
    assert nerr(w.grad, gW[perm]) <= TOL[np.float32]


@pytest.mark.parametrize("dtype", [np.float32, np.float64], ids=["f32", "f64"])
@pytest.mark.parametrize("rows", [1, 33, 1000])
def test_c4_backward_vs_oracle(rows, dtype, cuda_device):
    import openequivariance_b200 as oeq
    from openequivariance_b200.problems import fully_connected_tpp

    p = fully_connected_tpp(*C4, shared_weights=True, internal_weights=False,
                            irrep_dtype=dtype, weight_dtype=dtype)
    op = _oracle(p)
    perm = O.oeq_permutation(op)
    rng = np.random.default_rng(100 + rows)
    X = rng.normal(size=(rows, p.irreps_in1.dim))
    Y = rng.normal(size=(rows, p.irreps_in2.dim))
    W = rng.normal(size=(p.weight_numel,)) / np.sqrt(32 * 5)
    G = rng.normal(size=(rows, p.irreps_out.dim))
    tp = oeq.TensorProduct(p)
    x = to_dev(X, dtype).requires_grad_()
    y = to_dev(Y, dtype).requires_grad_()
    w = to_dev(W[perm], dtype).requires_grad_()
    names = _kernel_names(lambda: tp(x, y, w).backward(to_dev(G, dtype)))
    assert any("tp_uvw_sw_dxy" in n for n in names) and any("tp_uvw_sw_dw" in n for n in names)
    gX, gY, gW = O.backward(op, X, Y, W, G)
    for got, want, what in ((x.grad, gX, "dX"), (y.grad, gY, "dY"), (w.grad, gW[perm], "dW")):
        e = nerr(got, want)
        assert e <= TOL[dtype], f"{what}: normalised max error {e:.3e}"
