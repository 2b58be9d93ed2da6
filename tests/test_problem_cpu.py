"""Host-side logic of the package against the reference-generated fixtures (no GPU)."""

import ctypes
import re
from pathlib import Path

import numpy as np
import pytest

from conftest import ROOT, golden_names, load_golden, product_problem
from openequivariance_b200 import cg, plan
from openequivariance_b200.irreps import Irrep, Irreps, TPProblem


def test_product_cg_matches_reference():
    g = load_golden("cg_wigner3j.npz")
    for key, table in g.items():
        l1, l2, l3 = map(int, key.split("_"))
        np.testing.assert_allclose(cg.real_wigner_3j(l1, l2, l3), table, rtol=0, atol=1e-14)
        dense = np.zeros_like(table)
        for i, j, k, v in cg.sparse_cg(l1, l2, l3):
            dense[i, j, k] = v
        np.testing.assert_allclose(dense, table, rtol=0, atol=1e-12)


@pytest.mark.parametrize("name", golden_names("tp"))
def test_product_problem_matches_reference(name):
    g = load_golden(name)
    p = product_problem(g)
    np.testing.assert_allclose([i.path_weight for i in p.instructions], g["path_weights"],
                               rtol=1e-15, atol=0)
    assert p.weight_numel == int(g["weight_numel"])
    np.testing.assert_array_equal(plan.oeq_weight_permutation(p), g["perm"])
    w = np.arange(p.weight_numel, dtype=np.float64)[None, :].repeat(2, 0)
    fwd = plan.reorder_weights(p, w, "forward")
    np.testing.assert_array_equal(fwd[0], g["perm"])
    np.testing.assert_array_equal(plan.reorder_weights(p, fwd, "backward"), w)


def test_irreps_parsing_and_api():
    ir = Irreps("128x0e+128x1o + 2x2e")
    assert ir.dim == 128 + 384 + 10 and ir.num_irreps == 258 and ir.lmax == 2
    assert [s.start for s in ir.slices()] == [0, 128, 512]
    assert repr(Irreps("2x1o+1x1o").simplify()) == "3x1o"
    assert Irrep("3y") == Irrep(3, -1)
    assert list(Irrep("1o") * Irrep("1o")) == [Irrep("0e"), Irrep("1e"), Irrep("2e")]
    srt = Irreps("1x1o+1x0e").sort()
    assert repr(srt.irreps) == "1x0e+1x1o" and srt.p == (1, 0)
    with pytest.raises(ValueError):
        Irreps("3x")


def test_support_gate_messages():
    p = TPProblem("5x5e", "1x3e", "5x5e", [(0, 0, 0, "uvw", True)], shared_weights=False,
                  internal_weights=False, layout="ir_mul")
    with pytest.raises(AssertionError, match="layout='ir_mul'"):
        plan.analyze_problem(p)
    p = TPProblem("1x1e", "1x1e", "1x1e", [(0, 0, 0, "uvu", False)], shared_weights=False)
    with pytest.raises(AssertionError, match="trainable weights"):
        plan.analyze_problem(p)
    p = TPProblem("1x1e", "1x1e", "1x1e", [(0, 0, 0, "uvu", True)], shared_weights=False,
                  irrep_dtype=np.float32, weight_dtype=np.float64)
    with pytest.raises(AssertionError, match="irrep_dtype and weight_dtype"):
        plan.analyze_problem(p)


def test_descriptor_layout():
    g = load_golden("tp_mace_large.npz")
    p = product_problem(g, dtype=np.float32)
    d = plan.pack_descriptor(p, deterministic=True, kahan=True)
    h = np.frombuffer(d[:128], dtype="<i8")
    assert h[0] == plan.MAGIC and h[1] == 1 and h[2] == 1 and h[4] == 0
    assert (h[6], h[7], h[8], h[9]) == (3, 4, 17, 17)
    assert (h[10], h[11], h[12], h[13]) == (1152, 16, 9088, 2176)
    assert h[15] == 3
    n = 128 + (3 + 4 + 17) * 24 + 17 * 56 + int(h[14]) * 32
    assert len(d) == n
    assert plan.descriptor_hash(d) == plan.descriptor_hash(bytes(d))


def _header_functions():
    text = (ROOT / "include" / "oeqb200.h").read_text()
    return sorted(set(re.findall(r"^(?:const char\*|int|size_t)\s+(oeqb_\w+)\(", text, re.M)))


def test_cabi_library_exports_every_declared_symbol():
    from openequivariance_b200 import _ext

    lib = _ext.cabi()
    names = _header_functions()
    assert len(names) >= 10
    for name in names:
        assert hasattr(lib, name), name
    assert lib.oeqb_version().startswith(b"oeqb200")


def test_cabi_rejects_bad_descriptors_without_gpu():
    from openequivariance_b200 import _ext

    lib = _ext.cabi()
    out = ctypes.c_void_p()
    bad = bytes(64)
    assert lib.oeqb_plan_create(bad, len(bad), 0, ctypes.byref(out)) == 1
    assert b"short" in lib.oeqb_last_error()
    g = load_golden("tp_c1.npz")
    d = bytearray(plan.pack_descriptor(product_problem(g)))
    d[0] ^= 0xFF
    assert lib.oeqb_plan_create(bytes(d), len(d), 0, ctypes.byref(out)) == 1
    assert b"magic" in lib.oeqb_last_error()
    d = plan.pack_descriptor(product_problem(g))
    assert lib.oeqb_plan_create(d[:-8], len(d) - 8, 0, ctypes.byref(out)) == 1
    assert b"truncated" in lib.oeqb_last_error()


def test_torch_ops_registered():
    import torch

    from openequivariance_b200 import _ops

    _ops.ensure_registered()
    for name in ("jit_tp_forward", "jit_tp_backward", "jit_tp_double_backward",
                 "jit_conv_forward", "jit_conv_backward", "jit_conv_double_backward"):
        assert hasattr(torch.ops.libtorch_tp_jit, name)


def test_refgpu_cases_match_baseline_problems():
    """The BASELINE-size parity cases (run on the reference's kernels by
    ``tests/golden/make_golden_refgpu.py``) are the package's BASELINE problems."""
    import sys

    from conftest import GOLDEN
    from openequivariance_b200.problems import baseline_problem

    sys.path.insert(0, str(GOLDEN))
    import refgpu_cases as R

    for case, base in (("c1", "c1"), ("c2", "c2"), ("c2ml", "c2ml"), ("c4_f32", "c4")):
        in1, in2, out, ins, mode, shared = R.TP_CASES[case][:6]
        p = baseline_problem(base)
        assert (str(p.irreps_in1), str(p.irreps_in2), str(p.irreps_out)) == (in1, in2, out)
        assert [(i.i_in1, i.i_in2, i.i_out) for i in p.instructions] == ins
        assert {i.connection_mode for i in p.instructions} == {mode}
        assert p.shared_weights == shared
        assert p.weight_numel == R.weight_numel(R.TP_CASES[case])
    rows, cols, tperm = R.c3_graph()
    assert rows.size == R.C3_EDGES
    assert np.all(np.diff(rows * R.C3_NODES + cols) > 0)
    assert np.all(np.diff(cols[tperm] * R.C3_NODES + rows[tperm]) > 0)
