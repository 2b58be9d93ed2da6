"""Bad graph inputs reach the caller as errors (device checks on).

The reference's kernels index without checks, so a bad ``rows``/``cols``/``sender_perm``
entry faults the GPU or silently gives wrong sums (its C++ layer exits on driver errors,
``extension/backend/backend_cuda.hpp:15-45``).  Here, with the device checks on
(``set_device_checks(True)``, or ``OEQB_DEVICE_CHECKS=1`` which ``conftest.py`` sets for the
test session), every convolution call validates its graph on the device before launching
and raises ``RuntimeError`` naming the defect; the convolution kernels never see the bad
graph.  The error is injected on the host side only (bad index values in valid memory).
"""

import ctypes

import numpy as np
import pytest
import torch

from conftest import load_golden, product_problem

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _checks_on():
    import openequivariance_b200 as oeq

    prev = oeq.set_device_checks(True)
    yield
    oeq.set_device_checks(prev)


def _graph():
    """A valid receiver-sorted ring graph with its transpose permutation."""
    n = 40
    rows = np.repeat(np.arange(n), 3)
    cols = np.stack([(np.arange(n) - 1) % n, (np.arange(n) + 1) % n, (np.arange(n) + 7) % n], 1).ravel()
    order = np.lexsort((cols, rows))
    rows, cols = rows[order], cols[order]
    tperm = np.lexsort((rows, cols))
    return n, rows, cols, tperm


def _run(deterministic, rows, cols, tperm, n, backward=False):
    import openequivariance_b200 as oeq

    g = load_golden("conv_c1.npz")
    prob = product_problem(g, dtype=np.float32)
    conv = oeq.TensorProductConv(prob, deterministic=deterministic)
    E = len(rows)
    rng = np.random.default_rng(0)
    dev = lambda a, **k: torch.tensor(a, device="cuda", **k)  # noqa: E731
    x = dev(rng.normal(size=(n, prob.irreps_in1.dim)).astype(np.float32), requires_grad=True)
    y = dev(rng.normal(size=(E, prob.irreps_in2.dim)).astype(np.float32), requires_grad=True)
    w = dev(rng.normal(size=(E, prob.weight_numel)).astype(np.float32), requires_grad=True)
    z = conv(x, y, w, dev(rows), dev(cols), dev(tperm) if deterministic else None)
    if backward:
        z.backward(torch.ones_like(z))
    torch.cuda.synchronize()
    return z


@pytest.mark.parametrize("deterministic", [False, True])
@pytest.mark.parametrize("where", ["cols_high", "cols_negative", "rows_high"])
def test_out_of_range_index_raises(deterministic, where, cuda_device):
    n, rows, cols, tperm = _graph()
    rows, cols = rows.copy(), cols.copy()
    if where == "cols_high":
        cols[17] = n + 3
    elif where == "cols_negative":
        cols[5] = -1
    else:
        rows[-1] = n  # still sorted, but past the last node
    with pytest.raises(RuntimeError, match="edge index out of range"):
        _run(deterministic, rows, cols, tperm, n)


def test_unsorted_rows_raise_in_deterministic_mode(cuda_device):
    n, rows, cols, tperm = _graph()
    rows = rows.copy()
    rows[[10, 50]] = rows[[50, 10]]
    with pytest.raises(RuntimeError, match="rows are not sorted"):
        _run(True, rows, cols, tperm, n)
    # The atomic mode accepts any edge order.
    _run(False, rows, cols, tperm, n)


@pytest.mark.parametrize("defect,message", [
    ("duplicate", "not a permutation"),
    ("identity", "sender \\(cols\\) order"),
    ("out_of_range", "transpose_perm entry out of range"),
])
def test_bad_sender_perm_raises_in_backward(defect, message, cuda_device):
    n, rows, cols, tperm = _graph()
    tperm = tperm.copy()
    if defect == "duplicate":
        tperm[31] = tperm[30]
    elif defect == "identity":
        tperm = np.arange(len(rows))
    else:
        tperm[0] = len(rows) + 10
    # The forward pass does not read the permutation; the backward pass must refuse it.
    z = _run(True, rows, cols, tperm, n)
    assert torch.isfinite(z).all()
    with pytest.raises(RuntimeError, match=message):
        _run(True, rows, cols, tperm, n, backward=True)


def test_valid_graph_passes_and_status_is_clean(cuda_device):
    import openequivariance_b200 as oeq

    n, rows, cols, tperm = _graph()
    z_on = _run(True, rows, cols, tperm, n, backward=True)
    oeq.check_device_status()
    oeq.set_device_checks(False)
    z_off = _run(True, rows, cols, tperm, n, backward=True)
    oeq.check_device_status()
    assert torch.equal(z_on, z_off)


def test_validate_through_the_c_abi(cuda_device):
    from openequivariance_b200 import _ext

    lib = _ext.cabi()
    lib.oeqb_conv_validate_scratch_bytes.restype = ctypes.c_size_t
    n, rows, cols, tperm = _graph()
    E = len(rows)
    need = lib.oeqb_conv_validate_scratch_bytes(ctypes.c_int64(E))
    assert need >= 16 + 4 * ((E + 31) // 32)
    scratch = torch.zeros(need, dtype=torch.uint8, device="cuda")
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    p = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    r, c, t = (torch.tensor(a, device="cuda") for a in (rows, cols, tperm))
    args = (ctypes.c_int64(E), ctypes.c_int64(n), 1, p(scratch), ctypes.c_size_t(need), stream)
    assert lib.oeqb_conv_validate(p(r), p(c), p(t), *args) == 0, lib.oeqb_last_error()
    c[3] = n
    assert lib.oeqb_conv_validate(p(r), p(c), p(t), *args) == 1
    assert b"edge index out of range" in lib.oeqb_last_error()
    # Too little scratch is refused before anything runs.
    assert lib.oeqb_conv_validate(p(r), p(c), p(t), ctypes.c_int64(E), ctypes.c_int64(n), 1,
                                  p(scratch), ctypes.c_size_t(8), stream) == 1
    assert b"scratch" in lib.oeqb_last_error()


def _clear_status():
    """Reads every plan's flag until none is set (a flag left by an earlier test is not this
    test's concern)."""
    import openequivariance_b200 as oeq

    for _ in range(1000):
        try:
            oeq.check_device_status()
            return
        except RuntimeError:
            continue
    raise AssertionError("device status flags keep being set")


@pytest.mark.parametrize("deterministic", [False, True])
def test_kernels_drop_and_flag_bad_edges_with_checks_off(deterministic, cuda_device):
    """With the device checks off the bad graph reaches the single-path (C3-class) kernels.
    They skip the bad edge, raise the plan's status flag, and ``check_device_status`` reports
    it.  The other edges' results equal the oracle on the graph without that edge."""
    import openequivariance_b200 as oeq
    import tp_oracle as O
    from gpu_util import assert_close

    oeq.set_device_checks(False)
    _clear_status()
    n, rows, cols, tperm = _graph()
    bad = 17
    cols = cols.copy()
    cols[bad] = n + 3
    prob = oeq.TPProblem("1x2e", "1x3e", "1x2e", [(0, 0, 0, "uvu", True)],
                         shared_weights=False, internal_weights=False)
    conv = oeq.TensorProductConv(prob, deterministic=deterministic)
    E = len(rows)
    rng = np.random.default_rng(3)
    X, Y = rng.normal(size=(n, 5)), rng.normal(size=(E, 7))
    W, G = rng.normal(size=(E, 1)), rng.normal(size=(n, 5))
    dev = lambda a: torch.tensor(a, device="cuda")  # noqa: E731
    x, y, w = (dev(a.astype(np.float32)).requires_grad_() for a in (X, Y, W))
    z = conv(x, y, w, dev(rows), dev(cols), dev(tperm) if deterministic else None)
    z.backward(dev(G.astype(np.float32)))
    torch.cuda.synchronize()
    with pytest.raises(RuntimeError, match="edge index out of range"):
        oeq.check_device_status()
    oeq.check_device_status()  # reading the flag cleared it
    keep = np.arange(E) != bad
    p = O.make_problem("1x2e", "1x3e", "1x2e", [(0, 0, 0, "uvu", True)])
    r, c = rows[keep], cols[keep]
    assert_close(z, O.conv_forward(p, X, Y[keep], W[keep], r, c), np.float32, "forward")
    gX, gY, gW = O.conv_backward(p, X, Y[keep], W[keep], G, r, c)
    assert_close(x.grad, gX, np.float32, "dX")
    assert_close(y.grad[torch.from_numpy(keep).cuda()], gY, np.float32, "dY")
    assert_close(w.grad[torch.from_numpy(keep).cuda()], gW, np.float32, "dW")


def test_band_pass_flags_bad_permutation_entry_with_checks_off(cuda_device):
    """An out-of-range transpose_perm entry reaches the deterministic backward's pass B with
    the checks off: the position is skipped and status 2 is reported."""
    import openequivariance_b200 as oeq

    oeq.set_device_checks(False)
    _clear_status()
    n, rows, cols, tperm = _graph()
    tperm = tperm.copy()
    tperm[0] = len(rows) + 10
    prob = oeq.TPProblem("1x2e", "1x3e", "1x2e", [(0, 0, 0, "uvu", True)],
                         shared_weights=False, internal_weights=False)
    conv = oeq.TensorProductConv(prob, deterministic=True)
    E = len(rows)
    gen = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(n, 5, device="cuda", generator=gen, requires_grad=True)
    y = torch.randn(E, 7, device="cuda", generator=gen)
    w = torch.randn(E, 1, device="cuda", generator=gen)
    dev = lambda a: torch.tensor(a, device="cuda")  # noqa: E731
    z = conv(x, y, w, dev(rows), dev(cols), dev(tperm))
    z.backward(torch.ones_like(z))
    torch.cuda.synchronize()
    assert torch.isfinite(x.grad).all()
    with pytest.raises(RuntimeError, match="transpose_perm entry out of range"):
        oeq.check_device_status()
