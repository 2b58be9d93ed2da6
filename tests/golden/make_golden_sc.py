"""Generates the symmetric-contraction golden fixtures (``sc_*.npz``) from the reference.

Run where a checkout of the reference is available, naming it in ``OEQ_REFERENCE_ROOT``:
``OEQ_REFERENCE_ROOT=<checkout> python tests/golden/make_golden_sc.py``.

The reference module ``_torch/symmetric_contraction/SymmetricContraction.py`` imports e3nn
and the compiled extension, neither of which exists in this container.  The module file is
loaded unchanged with three stand-ins placed in ``sys.modules`` first:

* ``e3nn.o3``: ``Irreps``/``Irrep`` from the reference's own ``core/e3nn_lite.py`` (which is
  e3nn 0.5 code, ``e3nn_lite.py:1-12``) and ``wigner_3j`` wrapping ``e3nn_lite.wigner_3j``
  as a torch tensor; ``e3nn.util`` decorators as no-ops;
* ``openequivariance._torch.extlib``: a module attribute stub (``DEVICE_TYPE``);
* ``torch.ops.libtorch_tp_jit.group_gemm``: a CPU implementation of the documented
  semantics of ``extension/group_mm.hpp:38-141`` (per element i and channel b,
  ``C[r,b,:] = A[i,b] @ B[r,b,:]`` over the element's rows when ``ragged_inner == 0``;
  ``C[i,b] = sum_r A[r,b,:] (x) B[r,b,:]`` otherwise).

Everything else (``_wigner_nj``, ``U_matrix_real``, ``Contraction.forward``, the
sort/unsort of ``SymmetricContraction.forward`` and the group_gemm autograd formulas of
``register_autograd``) runs as written in the reference.
Fixtures hold the U matrices, the module's seeded parameters, inputs, outputs, a seeded
upstream gradient and the gradients of the inputs and of every weight.
"""

from __future__ import annotations

import importlib.util
import os
import sys
import types
from pathlib import Path

import numpy as np

OUT = Path(__file__).resolve().parent
if "OEQ_REFERENCE_ROOT" not in os.environ:
    sys.exit("set OEQ_REFERENCE_ROOT to a checkout of the reference (the directory that holds "
             "openequivariance/openequivariance)")
REF = Path(os.environ["OEQ_REFERENCE_ROOT"]) / "openequivariance"

os.environ["OEQ_NOTORCH"] = "1"
sys.path.insert(0, str(REF))

import torch  # noqa: E402

import openequivariance.core.e3nn_lite as el  # noqa: E402


def _install_stubs():
    e3nn = types.ModuleType("e3nn")
    o3 = types.ModuleType("e3nn.o3")
    o3.Irreps = el.Irreps
    o3.Irrep = el.Irrep

    def wigner_3j(l1, l2, l3, dtype=None):
        return torch.tensor(el.wigner_3j(l1, l2, l3), dtype=dtype or torch.float64)

    o3.wigner_3j = wigner_3j
    util = types.ModuleType("e3nn.util")
    codegen = types.ModuleType("e3nn.util.codegen")
    codegen.CodeGenMixin = type("CodeGenMixin", (), {})
    jit = types.ModuleType("e3nn.util.jit")
    jit.compile_mode = lambda mode: (lambda cls: cls)
    e3nn.o3, e3nn.util, util.codegen, util.jit = o3, util, codegen, jit
    sys.modules.update({"e3nn": e3nn, "e3nn.o3": o3, "e3nn.util": util,
                        "e3nn.util.codegen": codegen, "e3nn.util.jit": jit})
    extlib = types.ModuleType("openequivariance._torch.extlib")
    extlib.DEVICE_TYPE = "cpu"
    extlib.BUILT_EXTENSION = False
    sys.modules["openequivariance._torch.extlib"] = extlib
    import openequivariance._torch as t

    t.extlib = extlib

    lib = torch.library.Library("libtorch_tp_jit", "DEF")
    lib.define("group_gemm(Tensor A, Tensor B, Tensor ragged_counts, int num_W, int batch_size, "
               "int m, int k, int ragged_inner) -> Tensor")

    def group_gemm(A, B, counts, num_W, batch_size, m, k, ragged_inner):
        off = 0
        if ragged_inner == 0:
            C = A.new_zeros(B.shape[0], batch_size, m)
            for i in range(num_W):
                n = int(counts[i])
                C[off:off + n] = torch.einsum("bmk,rbk->rbm", A[i], B[off:off + n])
                off += n
        else:
            C = A.new_zeros(num_W, batch_size, m, k)
            for i in range(num_W):
                n = int(counts[i])
                C[i] = torch.einsum("rbm,rbk->bmk", A[off:off + n], B[off:off + n])
                off += n
        return C

    lib.impl("group_gemm", group_gemm, "CPU")
    return lib


_LIB = _install_stubs()


def _load_reference_sc():
    path = REF / "openequivariance" / "_torch" / "symmetric_contraction" / "SymmetricContraction.py"
    spec = importlib.util.spec_from_file_location("ref_symmetric_contraction", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


SC = _load_reference_sc()
# The reference registers the group_gemm backward (itself a group_gemm) only when its extension
# is built; register it here so gradients flow through the top correlation as in the reference.
SC.register_autograd()

# (name, irreps_in, irreps_out, correlation, num_elements, labels); the first three are the
# configurations of tests/symmetric_contraction_test.py, the last is the MACE/C5 shape with
# fewer channels and nodes.
CONFIGS = [
    ("t1", "2x0e + 2x1o", "2x0e + 2x1o", 2, 4, [0, 2, 3, 2, 0, 0, 2, 3, 2, 2]),
    ("t2", "1x0e + 1x1o + 1x2e", "1x0e + 1x1o", 3, 3, [0, 1, 2, 0, 1, 2, 0, 1]),
    ("t3", "4x0e + 4x1o", "4x0e", 2, 5, [0, 1, 2, 3, 4, 0, 1, 2, 3, 4]),
    ("c5s", "8x0e + 8x1o + 8x2e", "8x0e + 8x1o", 3, 10,
     [3, 7, 1, 0, 9, 2, 2, 5, 8, 4, 6, 1, 0, 3, 9, 9, 4, 7, 5, 6]),
]


def main():
    for name, ii, io, corr, ne, labels in CONFIGS:
        torch.manual_seed(12345)
        irr_in = el.Irreps(ii)
        mod = SC.SymmetricContraction(irr_in, el.Irreps(io), correlation=corr, num_elements=ne,
                                      dtype=torch.float64)
        gen = torch.Generator().manual_seed(2468)
        nf = irr_in.count(el.Irrep("0e"))
        x = torch.randn(len(labels), nf, irr_in.dim // nf, dtype=torch.float64, generator=gen,
                        requires_grad=True)
        y = torch.nn.functional.one_hot(torch.tensor(labels), num_classes=ne).to(torch.float64)
        out = mod(x, y)
        g = torch.randn(out.shape, dtype=torch.float64, generator=gen)
        params = []
        for c in mod.contractions:
            params += [c.weights_max] + list(c.weights)
        grads = torch.autograd.grad((out * g).sum(), [x] + params)
        arrays = {"x": x.detach().numpy(), "labels": np.array(labels), "out": out.detach().numpy(),
                  "grad_out": g.numpy(), "grad_x": grads[0].numpy(), "meta": np.array([corr, ne])}
        gi = 1
        for ci, c in enumerate(mod.contractions):
            arrays[f"c{ci}_weights_max"] = c.weights_max.detach().numpy()
            arrays[f"c{ci}_grad_weights_max"] = grads[gi].numpy()
            gi += 1
            for wi, w in enumerate(c.weights):
                arrays[f"c{ci}_weights_{wi}"] = w.detach().numpy()
                arrays[f"c{ci}_grad_weights_{wi}"] = grads[gi].numpy()
                gi += 1
            for nu in range(1, corr + 1):
                arrays[f"c{ci}_U{nu}"] = c.U_tensors(nu).numpy()
        np.savez_compressed(OUT / f"sc_{name}.npz", irreps_in=np.array(ii), irreps_out=np.array(io),
                            **arrays)
        print(name, tuple(out.shape), float(out.detach().abs().max()))


if __name__ == "__main__":
    main()
