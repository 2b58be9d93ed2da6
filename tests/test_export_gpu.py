"""Deployment paths of the operators: torch.save/load, torch.compile, torch.export, AOTInductor
(Python and a C++ loader), submodule ``.to(dtype)``, and the convolution's triple backward.

Follows the reference's ``tests/export_test.py:19-233`` (same problem, 32x5e (x) 1x3e -> 32x5e
uvu, and the same three module kinds: batch, deterministic conv, atomic conv),
``tests/batch_test.py:395-460`` (submodule dtype conversion) and ``tests/conv_test.py:149``
(conv triple backward).  The C++ loader is this repository's own (``tests/aoti_loader.cpp``),
built with g++ against libtorch and ``libtorch_oeqb200.so``.
"""

import functools
import os
import subprocess
import sys
import tempfile

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.fixture(scope="module")
def problem():
    import openequivariance_b200 as oeq

    return oeq.TPProblem("32x5e", "1x3e", "32x5e", [(0, 0, 0, "uvu", True)],
                         shared_weights=False, internal_weights=False,
                         irrep_dtype=np.float32, weight_dtype=np.float32)


def _graph():
    """Receiver / sender indices of a 3-node path graph (both directions), receiver-sorted,
    with the sender-order permutation."""
    rows = torch.tensor([0, 1, 1, 2], device="cuda")
    cols = torch.tensor([1, 0, 2, 1], device="cuda")
    perm = torch.argsort(cols * 3 + rows)
    return rows, cols, perm


@pytest.fixture(params=["batch", "conv_det", "conv_atomic"], scope="module")
def tp_and_inputs(request, problem, cuda_device):
    import openequivariance_b200 as oeq

    gen = torch.Generator(device="cuda").manual_seed(0)
    if request.param == "batch":
        B = 1000
        X = torch.rand(B, problem.irreps_in1.dim, device="cuda", generator=gen)
        Y = torch.rand(B, problem.irreps_in2.dim, device="cuda", generator=gen)
        W = torch.rand(B, problem.weight_numel, device="cuda", generator=gen)
        return oeq.TensorProduct(problem), (X, Y, W)
    rows, cols, perm = _graph()
    X = torch.rand(3, problem.irreps_in1.dim, device="cuda", generator=gen)
    Y = torch.rand(4, problem.irreps_in2.dim, device="cuda", generator=gen)
    W = torch.rand(4, problem.weight_numel, device="cuda", generator=gen)
    if request.param == "conv_atomic":
        return oeq.TensorProductConv(problem, deterministic=False), (X, Y, W, rows, cols)
    return oeq.TensorProductConv(problem, deterministic=True), (X, Y, W, rows, cols, perm)


def test_torch_save_load(tp_and_inputs):
    tp, inputs = tp_and_inputs
    want = tp(*inputs)
    with tempfile.NamedTemporaryFile(suffix=".pt") as f:
        torch.save(tp, f.name)
        loaded = torch.load(f.name)
    torch.testing.assert_close(loaded(*inputs), want, atol=1e-5, rtol=0)


def test_torch_compile(tp_and_inputs):
    tp, inputs = tp_and_inputs
    want = tp(*inputs)
    got = torch.compile(tp)(*inputs)
    torch.testing.assert_close(got, want, atol=1e-5, rtol=0)


def test_torch_compile_backward(tp_and_inputs):
    """Gradients through a compiled module (fake kernels + registered autograd)."""
    tp, inputs = tp_and_inputs
    leaf = [t.clone().requires_grad_(True) for t in inputs[:3]]
    leaf2 = [t.clone().requires_grad_(True) for t in inputs[:3]]
    tp(*leaf, *inputs[3:]).square().sum().backward()
    torch.compile(tp)(*leaf2, *inputs[3:]).square().sum().backward()
    for a, b in zip(leaf, leaf2):
        torch.testing.assert_close(b.grad, a.grad, atol=1e-4, rtol=1e-5)


def test_torch_export(tp_and_inputs):
    tp, inputs = tp_and_inputs
    want = tp(*inputs)
    ep = torch.export.export(tp, args=inputs, strict=False)
    torch.testing.assert_close(ep.module()(*inputs), want, atol=1e-5, rtol=0)


@functools.lru_cache(maxsize=None)
def _has_openmp(cxx):
    with tempfile.TemporaryDirectory() as d:
        src = os.path.join(d, "t.cpp")
        with open(src, "w") as f:
            f.write("int main() { return 0; }\n")
        r = subprocess.run([cxx, "-fopenmp", src, "-o", os.path.join(d, "t")],
                           capture_output=True)
    return r.returncode == 0


@pytest.fixture(autouse=True)
def _inductor_compiler(monkeypatch):
    """AOTInductor builds its wrapper with OpenMP.  Where the host compiler it finds first
    cannot link OpenMP, it is pointed at the system g++ if that one can; without any such
    compiler the tests that need it are skipped (a build without OpenMP loads incorrectly)."""
    import torch._inductor.config as ic
    import torch._inductor.cpp_builder as cb

    if _has_openmp(cb.get_cpp_compiler()):
        return
    alt = "/usr/bin/g++"
    if os.path.exists(alt) and _has_openmp(alt):
        monkeypatch.setattr(ic.cpp, "cxx", (None, alt))
    else:
        pytest.skip("no host C++ compiler with OpenMP for AOTInductor")


def test_aoti_python(tp_and_inputs):
    tp, inputs = tp_and_inputs
    want = tp(*inputs)
    ep = torch.export.export(tp, args=inputs, strict=False)
    with tempfile.TemporaryDirectory() as d:
        path = torch._inductor.aoti_compile_and_package(ep, package_path=os.path.join(d, "m.pt2"))
        model = torch._inductor.aoti_load_package(path)
        torch.testing.assert_close(model(*inputs), want, atol=1e-5, rtol=0)


def test_aoti_cpp_loader(problem, cuda_device):
    """An AOTI package of the batch TP, run from C++ (libtorch + libtorch_oeqb200.so)."""
    import openequivariance_b200 as oeq
    from torch.utils.cpp_extension import include_paths, library_paths

    tp = oeq.TensorProduct(problem)
    B = 1000
    gen = torch.Generator(device="cuda").manual_seed(0)
    X = torch.rand(B, problem.irreps_in1.dim, device="cuda", generator=gen)
    Y = torch.rand(B, problem.irreps_in2.dim, device="cuda", generator=gen)
    W = torch.rand(B, problem.weight_numel, device="cuda", generator=gen)
    want = tp(X, Y, W).cpu().numpy()
    ep = torch.export.export(tp, args=(X, Y, W), strict=False)
    with tempfile.TemporaryDirectory() as d:
        pkg = torch._inductor.aoti_compile_and_package(ep, package_path=os.path.join(d, "m.pt2"))
        for name, t in (("x", X), ("y", Y), ("w", W)):
            t.cpu().numpy().astype(np.float32).tofile(os.path.join(d, f"{name}.bin"))
        exe = os.path.join(d, "aoti_loader")
        libs = library_paths("cuda")
        cmd = (["g++", "-O1", "-std=c++17", os.path.join(HERE, "aoti_loader.cpp"), "-o", exe,
                "-D_GLIBCXX_USE_CXX11_ABI=" + str(int(torch.compiled_with_cxx11_abi()))]
               + [f"-I{p}" for p in include_paths("cuda")]
               + [f"-L{p}" for p in libs] + [f"-Wl,-rpath,{p}" for p in libs]
               + ["-Wl,--no-as-needed", oeq.torch_ext_so_path(), "-ltorch", "-ltorch_cpu",
                  "-ltorch_cuda", "-lc10", "-lc10_cuda"])
        r = subprocess.run(cmd, capture_output=True, text=True)
        assert r.returncode == 0, r.stderr[-3000:]
        r = subprocess.run([exe, pkg, d, str(B), str(problem.irreps_in1.dim),
                            str(problem.irreps_in2.dim), str(problem.weight_numel),
                            str(problem.irreps_out.dim)], capture_output=True, text=True)
        assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-3000:]
        got = np.fromfile(os.path.join(d, "z.bin"), dtype=np.float32).reshape(want.shape)
    np.testing.assert_allclose(got, want, atol=1e-5, rtol=0)


@pytest.mark.parametrize("start", ["float32", "float64"])
def test_submodule_dtype_conversion(start, cuda_device):
    import openequivariance_b200 as oeq

    dt = {"float32": (np.float32, torch.float32), "float64": (np.float64, torch.float64)}
    npdt, tdt = dt[start]
    prob = oeq.TPProblem("8x1o+8x2e", "1x0e+1x1o", "8x1o+8x2e",
                         [(0, 0, 0, "uvu", True), (1, 1, 0, "uvu", True), (1, 0, 1, "uvu", True)],
                         shared_weights=False, internal_weights=False,
                         irrep_dtype=npdt, weight_dtype=npdt)

    class Parent(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.tp = oeq.TensorProduct(prob)

        def forward(self, x, y, w):
            return self.tp(x, y, w)

    parent = Parent()
    g = torch.Generator(device="cuda").manual_seed(1)
    args = [torch.rand(10, n, device="cuda", generator=g, dtype=tdt)
            for n in (prob.irreps_in1.dim, prob.irreps_in2.dim, prob.weight_numel)]
    assert parent(*args).dtype == tdt
    other = torch.float64 if tdt == torch.float32 else torch.float32
    parent.to(other)
    args2 = [a.to(other) for a in args]
    out = parent(*args2)
    assert out.dtype == other
    onp = np.float64 if other == torch.float64 else np.float32
    fresh = oeq.TensorProduct(oeq.TPProblem(
        "8x1o+8x2e", "1x0e+1x1o", "8x1o+8x2e",
        [(0, 0, 0, "uvu", True), (1, 1, 0, "uvu", True), (1, 0, 1, "uvu", True)],
        shared_weights=False, internal_weights=False, irrep_dtype=onp, weight_dtype=onp))
    torch.testing.assert_close(out, fresh(*args2))


def test_conv_triple_backward(cuda_device):
    """Third derivatives of the convolution through autograd (gradcheck, float64)."""
    import openequivariance_b200 as oeq

    prob = oeq.TPProblem("2x0e+2x1o", "1x0e+1x1o", "2x0e+2x1o",
                         [(0, 0, 0, "uvu", True), (1, 1, 0, "uvu", True),
                          (0, 1, 1, "uvu", True), (1, 0, 1, "uvu", True)],
                         shared_weights=False, internal_weights=False,
                         irrep_dtype=np.float64, weight_dtype=np.float64)
    n = 5
    rows = torch.tensor([0, 0, 1, 2, 2, 3, 4, 4], device="cuda")
    cols = torch.tensor([1, 4, 0, 1, 3, 2, 0, 3], device="cuda")
    perm = torch.argsort(cols * n + rows)
    E = rows.numel()
    g = torch.Generator(device="cuda").manual_seed(3)
    for det in (False, True):
        conv = oeq.TensorProductConv(prob, deterministic=det)
        X = torch.randn(n, prob.irreps_in1.dim, device="cuda", dtype=torch.float64,
                        generator=g).requires_grad_()
        Y = torch.randn(E, prob.irreps_in2.dim, device="cuda", dtype=torch.float64,
                        generator=g).requires_grad_()
        W = torch.randn(E, prob.weight_numel, device="cuda", dtype=torch.float64,
                        generator=g).requires_grad_()

        def f(a, b, c):
            return conv(a, b, c, rows, cols, perm if det else None)

        assert torch.autograd.gradcheck(f, (X, Y, W), eps=1e-6, atol=1e-8)
        assert torch.autograd.gradgradcheck(f, (X, Y, W), eps=1e-6, atol=1e-7)

        def grads(a, b, c):
            out = f(a, b, c)
            ga, gb, gc = torch.autograd.grad(out.pow(2).sum(), (a, b, c), create_graph=True)
            return ga.pow(2).sum() + gb.pow(2).sum() + gc.pow(2).sum()

        assert torch.autograd.gradcheck(grads, (X, Y, W), eps=1e-6, atol=1e-6)
