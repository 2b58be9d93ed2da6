"""The allocation-free forward entry point, called through the C ABI.

Some callers cannot allocate device memory (a custom call inside another runtime's
allocator, a fixed-arena server); ``oeqb_tp_forward_noalloc`` serves them from a static
device array.  This test compares it with the regular plan-based entry point on two
consecutive calls (the array keeps the previous call's contents, so the second call checks
that stale state does not leak into the result).  It lives in its own file, collected last.
"""

import ctypes

import numpy as np
import pytest

from conftest import load_golden, product_problem

pytestmark = pytest.mark.gpu


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr())


# tp_c4_nequip_uvw is the shared-weight uvw class: the plan path runs its dedicated
# kernels (tensor cores in float32), the allocation-free call runs the table kernel.
@pytest.mark.parametrize("name,dtype", [("tp_mace_large.npz", np.float32),
                                        ("tp_c1.npz", np.float64),
                                        ("tp_c4_nequip_uvw.npz", np.float32),
                                        ("tp_c4_nequip_uvw.npz", np.float64)])
def test_noalloc_forward_matches_plan_forward(name, dtype, cuda_device):
    import torch

    from openequivariance_b200 import _ext, plan

    lib = _ext.cabi()
    g = load_golden(name)
    prob = product_problem(g, dtype=dtype)
    desc = plan.pack_descriptor(prob)
    tdt = torch.float32 if dtype == np.float32 else torch.float64
    handle = ctypes.c_void_p()
    assert lib.oeqb_plan_create(desc, len(desc), 0, ctypes.byref(handle)) == 0, lib.oeqb_last_error()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    try:
        gen = torch.Generator(device="cuda").manual_seed(7)
        for call in range(2):
            B = 300 + 77 * call
            X = torch.randn(B, prob.irreps_in1.dim, dtype=tdt, device="cuda", generator=gen)
            Y = torch.randn(B, prob.irreps_in2.dim, dtype=tdt, device="cuda", generator=gen)
            wshape = (prob.weight_numel,) if prob.shared_weights else (B, prob.weight_numel)
            W = torch.randn(*wshape, dtype=tdt, device="cuda", generator=gen)
            Z_ref = torch.empty(B, prob.irreps_out.dim, dtype=tdt, device="cuda")
            Z = torch.full_like(Z_ref, float("nan"))
            assert lib.oeqb_tp_forward(handle, ctypes.c_int64(B), _ptr(X), _ptr(Y), _ptr(W),
                                       _ptr(Z_ref), stream) == 0, lib.oeqb_last_error()
            assert lib.oeqb_tp_forward_noalloc(desc, len(desc), 0, ctypes.c_int64(B), _ptr(X),
                                               _ptr(Y), _ptr(W), _ptr(Z), stream) == 0, \
                lib.oeqb_last_error()
            torch.cuda.synchronize()
            tol = 1e-5 if dtype == np.float32 else 1e-12
            err = (Z - Z_ref).abs().max().item() / max(Z_ref.abs().max().item(), 1e-30)
            assert err <= tol, f"call {call}: normalised max error {err:.3e}"
    finally:
        lib.oeqb_plan_destroy(handle)


def test_noalloc_rejects_oversized_problem(cuda_device):
    from openequivariance_b200 import _ext, plan
    from openequivariance_b200.irreps import TPProblem

    lib = _ext.cabi()
    # 1100 instructions x 64 bytes of instruction table alone exceed the 64 KiB array.
    ins = [(0, 0, 0, "uvu", True)] * 1100
    prob = TPProblem("4x1e", "1x1e", "4x1e", ins, shared_weights=False, internal_weights=False)
    desc = plan.pack_descriptor(prob)
    rc = lib.oeqb_tp_forward_noalloc(desc, len(desc), 0, ctypes.c_int64(1), None, None, None,
                                     None, None)
    assert rc == 2
    assert b"at most 65536" in lib.oeqb_last_error()
