"""Fused graph convolution on the GPU: atomic, deterministic and Kahan modes."""

import numpy as np
import pytest
import torch

import tp_oracle as O
from conftest import golden_names, load_golden, oracle_problem, product_problem
from gpu_util import TOL, assert_close, nerr, to_dev

pytestmark = pytest.mark.gpu

MODES = ["atomic", "deterministic", "kahan"]


def _conv(g, dtype, mode):
    import openequivariance_b200 as oeq

    return oeq.TensorProductConv(product_problem(g, dtype=dtype),
                                 deterministic=mode != "atomic", kahan=mode == "kahan")


def _idx(a):
    return torch.tensor(np.asarray(a), dtype=torch.int64, device="cuda")


def _cases():
    out = []
    for name in golden_names("conv"):
        for mode in MODES:
            for dtype in (np.float32, np.float64):
                if mode == "kahan" and dtype == np.float64:
                    continue
                out.append(pytest.param(name, mode, dtype, id=f"{name}-{mode}-{dtype.__name__}"))
    return out


@pytest.mark.parametrize("name,mode,dtype", _cases())
def test_conv_vs_reference(name, mode, dtype, cuda_device):
    g = load_golden(name)
    conv = _conv(g, dtype, mode)
    perm = g["perm"]
    rows, cols, tperm = _idx(g["rows"]), _idx(g["cols"]), _idx(g["transpose_perm"])
    sp = tperm if mode != "atomic" else None
    X = to_dev(g["X"], dtype).requires_grad_()
    Y = to_dev(g["Y"], dtype).requires_grad_()
    W = to_dev(g["W_e3nn"][..., perm], dtype).requires_grad_()
    Z = conv(X, Y, W, rows, cols, sp)
    assert_close(Z, g["Z"], dtype, "forward")
    Z.backward(to_dev(g["G"], dtype))
    assert_close(X.grad, g["gX"], dtype, "dX")
    assert_close(Y.grad, g["gY"], dtype, "dY")
    assert_close(W.grad, g["gW_oeq"], dtype, "dW")
    # double backward vs the oracle
    p = oracle_problem(g)
    rng = np.random.default_rng(2)
    a = rng.uniform(size=g["X"].shape)
    b = rng.uniform(size=g["Y"].shape)
    c = rng.uniform(size=g["W_e3nn"].shape)
    want = O.conv_double_backward(p, g["X"], g["Y"], g["W_e3nn"], g["G"], a, b, c,
                                  g["rows"], g["cols"])
    out = torch.ops.libtorch_tp_jit.jit_conv_double_backward(
        conv.kernel, conv.hash, to_dev(g["X"], dtype), to_dev(g["Y"], dtype),
        to_dev(g["W_e3nn"][..., perm], dtype), to_dev(g["G"], dtype), to_dev(a, dtype),
        to_dev(b, dtype), to_dev(c[..., perm], dtype), rows, cols, conv.workspace_buffer,
        tperm if mode != "atomic" else conv.dummy_transpose_perm)
    assert_close(out[0], want[0], dtype, "ddX")
    assert_close(out[1], want[1], dtype, "ddY")
    assert_close(out[2].cpu().numpy()[..., np.argsort(perm)], want[2], dtype, "ddW")
    assert_close(out[3], want[3], dtype, "ddZ")


def radius_graph(n, box, cutoff, seed):
    """Directed radius graph in a periodic box, receiver-sorted, with transpose perm."""
    from scipy.spatial import cKDTree

    rng = np.random.default_rng(seed)
    pos = rng.uniform(0, box, size=(n, 3))
    tree = cKDTree(pos, boxsize=box)
    pairs = tree.query_pairs(cutoff, output_type="ndarray")
    rows = np.concatenate([pairs[:, 0], pairs[:, 1]]).astype(np.int64)
    cols = np.concatenate([pairs[:, 1], pairs[:, 0]]).astype(np.int64)
    order = np.lexsort((cols, rows))
    rows, cols = rows[order], cols[order]
    tperm = np.lexsort((rows, cols)).astype(np.int64)
    vec = pos[cols] - pos[rows]
    vec -= box * np.round(vec / box)
    return pos, rows, cols, tperm, vec


@pytest.mark.parametrize("mode", MODES)
def test_radius_graph_c1_irreps_vs_oracle(mode, cuda_device):
    import openequivariance_b200 as oeq

    pos, rows, cols, tperm, _ = radius_graph(400, 12.0, 3.0, seed=0)
    dtype = np.float32
    prob = oeq.TPProblem("1x2e", "1x3e", "1x2e", [(0, 0, 0, "uvu", True)],
                         shared_weights=False, internal_weights=False)
    conv = oeq.TensorProductConv(prob, deterministic=mode != "atomic", kahan=mode == "kahan")
    p = O.make_problem("1x2e", "1x3e", "1x2e", [(0, 0, 0, "uvu", True)])
    rng = np.random.default_rng(1)
    X, Y = rng.normal(size=(400, 5)), rng.normal(size=(len(rows), 7))
    W, G = rng.normal(size=(len(rows), 1)), rng.normal(size=(400, 5))
    args = [_idx(rows), _idx(cols), _idx(tperm) if mode != "atomic" else None]
    x, y, w = (to_dev(X, dtype).requires_grad_(), to_dev(Y, dtype).requires_grad_(),
               to_dev(W, dtype).requires_grad_())
    Z = conv(x, y, w, *args)
    assert_close(Z, O.conv_forward(p, X, Y, W, rows, cols), dtype, "forward")
    Z.backward(to_dev(G, dtype))
    gX, gY, gW = O.conv_backward(p, X, Y, W, G, rows, cols)
    assert_close(x.grad, gX, dtype, "dX")
    assert_close(y.grad, gY, dtype, "dY")
    assert_close(w.grad, gW, dtype, "dW")


@pytest.mark.parametrize("dtype", [np.float32, np.float64], ids=["f32", "f64"])
@pytest.mark.parametrize("mode", ["atomic", "deterministic"])
def test_single_path_silent_senders_and_hub(mode, dtype, cuda_device):
    """C3-class conv on a graph where nodes 0-49 send no edge (their dX rows must be zero),
    nodes 50-59 receive none (zero Z rows), and node 60 sends to every receiver, so its run in
    transpose_perm order spans several 32-edge blocks.  float32 runs the pipelined kernels,
    float64 the generic ones (both with the banded pass B when deterministic)."""
    import openequivariance_b200 as oeq

    n = 300
    rng = np.random.default_rng(11)
    recv = np.setdiff1d(np.arange(n), np.arange(50, 60))
    r = rng.choice(recv, 6000)
    s = rng.integers(50, n, 6000)
    r = np.concatenate([r, recv])
    s = np.concatenate([s, np.full(len(recv), 60)])
    key = np.unique(r * n + s)
    rows, cols = key // n, key % n
    tperm = np.argsort(cols * n + rows, kind="stable")
    E = len(rows)
    prob = oeq.TPProblem("1x2e", "1x3e", "1x2e", [(0, 0, 0, "uvu", True)],
                         shared_weights=False, internal_weights=False, irrep_dtype=dtype,
                         weight_dtype=dtype)
    conv = oeq.TensorProductConv(prob, deterministic=mode != "atomic")
    p = O.make_problem("1x2e", "1x3e", "1x2e", [(0, 0, 0, "uvu", True)])
    X, Y = rng.normal(size=(n, 5)), rng.normal(size=(E, 7))
    W, G = rng.normal(size=(E, 1)), rng.normal(size=(n, 5))
    args = [_idx(rows), _idx(cols), _idx(tperm) if mode != "atomic" else None]
    x, y, w = (to_dev(X, dtype).requires_grad_(), to_dev(Y, dtype).requires_grad_(),
               to_dev(W, dtype).requires_grad_())
    Z = conv(x, y, w, *args)
    # Leave NaN behind in freed blocks of the caching allocator, so a dX row the kernels skip
    # does not read as zero by chance.
    junk = torch.full((64, n * 5), float("nan"), device="cuda", dtype=x.dtype)
    del junk
    Z.backward(to_dev(G, dtype))
    assert_close(Z, O.conv_forward(p, X, Y, W, rows, cols), dtype, "forward")
    gX, gY, gW = O.conv_backward(p, X, Y, W, G, rows, cols)
    assert torch.all(x.grad[:50] == 0)
    assert torch.all(Z[50:60] == 0)
    assert_close(x.grad, gX, dtype, "dX")
    assert_close(y.grad, gY, dtype, "dY")
    assert_close(w.grad, gW, dtype, "dW")


@pytest.mark.parametrize("kahan", [False, True])
def test_deterministic_mode_is_bitwise_reproducible(kahan, cuda_device):
    import openequivariance_b200 as oeq

    _, rows, cols, tperm, _ = radius_graph(2000, 20.0, 3.5, seed=4)
    prob = oeq.TPProblem("32x0e+32x1o", "1x0e+1x1o", "32x0e+32x1o+32x1e",
                         [(0, 0, 0, "uvu", True), (0, 1, 1, "uvu", True), (1, 0, 1, "uvu", True),
                          (1, 1, 0, "uvu", True), (1, 1, 2, "uvu", True)],
                         shared_weights=False, internal_weights=False)
    conv = oeq.TensorProductConv(prob, deterministic=True, kahan=kahan)
    gen = torch.Generator(device="cuda").manual_seed(0)
    X = torch.rand(2000, prob.irreps_in1.dim, device="cuda", generator=gen, requires_grad=True)
    Y = torch.rand(len(rows), prob.irreps_in2.dim, device="cuda", generator=gen)
    W = torch.rand(len(rows), prob.weight_numel, device="cuda", generator=gen)
    G = torch.rand(2000, prob.irreps_out.dim, device="cuda", generator=gen)
    r, c, t = _idx(rows), _idx(cols), _idx(tperm)
    outs = []
    for _ in range(3):
        X.grad = None
        Z = conv(X, Y, W, r, c, t)
        Z.backward(G)
        outs.append((Z.detach().clone(), X.grad.clone()))
    for Z, gx in outs[1:]:
        assert torch.equal(Z, outs[0][0])
        assert torch.equal(gx, outs[0][1])


def test_shared_weights_atomic(cuda_device):
    g = load_golden("conv_c1.npz")
    import openequivariance_b200 as oeq

    p = product_problem(g, dtype=np.float64)
    p.shared_weights = True
    conv = oeq.TensorProductConv(p, deterministic=False)
    op = O.make_problem("1x2e", "1x3e", "1x2e", [(0, 0, 0, "uvu", True)], shared_weights=True)
    W = np.array([0.7])
    x, y, w = (to_dev(t, np.float64).requires_grad_() for t in (g["X"], g["Y"], W))
    Z = conv(x, y, w, _idx(g["rows"]), _idx(g["cols"]))
    assert nerr(Z, O.conv_forward(op, g["X"], g["Y"], W, g["rows"], g["cols"])) <= 1e-12
    Z.backward(to_dev(g["G"], np.float64))
    gX, gY, gW = O.conv_backward(op, g["X"], g["Y"], W, g["G"], g["rows"], g["cols"])
    assert nerr(x.grad, gX) <= 1e-12
    assert nerr(y.grad, gY) <= 1e-12
    assert nerr(w.grad, gW) <= 1e-12
    with pytest.raises(AssertionError, match="shared weights"):
        oeq.TensorProductConv(p, deterministic=True)


def test_conv_input_validation(cuda_device):
    g = load_golden("conv_c1.npz")
    conv = _conv(g, np.float32, "deterministic")
    X, Y = to_dev(g["X"], np.float32), to_dev(g["Y"], np.float32)
    W = to_dev(g["W_e3nn"], np.float32)
    rows, cols, tp = _idx(g["rows"]), _idx(g["cols"]), _idx(g["transpose_perm"])
    conv(X, Y, W, rows, cols, tp)
    with pytest.raises(RuntimeError, match="Shape mismatch"):
        conv(X, Y, W, rows, cols, tp[:-1])
    with pytest.raises(RuntimeError, match="is not on the GPU"):
        conv(X, Y, W, rows.cpu(), cols, tp)
    with pytest.raises(RuntimeError, match="Dtype mismatch"):
        conv(X, Y, W, rows.int(), cols, tp)


@pytest.mark.parametrize("dtype", [np.float32, np.float64], ids=["f32", "f64"])
def test_deterministic_single_path_dense_graph(dtype, cuda_device):
    """C3-class deterministic conv on a dense graph (~150 neighbours per node), so receiver and
    sender runs span several 32-edge blocks: forward, backward and bitwise repeatability."""
    import openequivariance_b200 as oeq

    pos, rows, cols, tperm, _ = radius_graph(300, 10.0, 4.5, seed=3)
    assert len(rows) / 300 > 100
    prob = oeq.TPProblem("1x2e", "1x3e", "1x2e", [(0, 0, 0, "uvu", True)],
                         shared_weights=False, internal_weights=False, irrep_dtype=dtype,
                         weight_dtype=dtype)
    conv = oeq.TensorProductConv(prob, deterministic=True)
    p = O.make_problem("1x2e", "1x3e", "1x2e", [(0, 0, 0, "uvu", True)])
    rng = np.random.default_rng(8)
    X, Y = rng.normal(size=(300, 5)), rng.normal(size=(len(rows), 7))
    W, G = rng.normal(size=(len(rows), 1)), rng.normal(size=(300, 5))
    r, c, t = _idx(rows), _idx(cols), _idx(tperm)
    outs = []
    for _ in range(2):
        x, y, w = (to_dev(X, dtype).requires_grad_(), to_dev(Y, dtype).requires_grad_(),
                   to_dev(W, dtype).requires_grad_())
        Z = conv(x, y, w, r, c, t)
        Z.backward(to_dev(G, dtype))
        outs.append([Z.detach(), x.grad, y.grad, w.grad])
    assert_close(outs[0][0], O.conv_forward(p, X, Y, W, rows, cols), dtype, "forward")
    gX, gY, gW = O.conv_backward(p, X, Y, W, G, rows, cols)
    assert_close(outs[0][1], gX, dtype, "dX")
    assert_close(outs[0][2], gY, dtype, "dY")
    assert_close(outs[0][3], gW, dtype, "dW")
    for a, b in zip(outs[0], outs[1]):
        assert torch.equal(a, b)
