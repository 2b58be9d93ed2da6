"""Pins the CPU oracle against fixtures generated from the reference (tests/golden)."""

import numpy as np
import pytest

import tp_oracle as O
from conftest import golden_names, load_golden, oracle_problem


def test_cg_tables_match_reference():
    g = load_golden("cg_wigner3j.npz")
    assert len(g) >= 60
    for key, table in g.items():
        l1, l2, l3 = map(int, key.split("_"))
        np.testing.assert_allclose(O.wigner_3j(l1, l2, l3), table, rtol=0, atol=1e-14)


@pytest.mark.parametrize("name", golden_names("tp"))
def test_problem_normalisation_and_weight_order(name):
    g = load_golden(name)
    p = oracle_problem(g)
    np.testing.assert_allclose(p.path_weights, g["path_weights"], rtol=1e-15, atol=0)
    assert p.weight_numel == int(g["weight_numel"])
    np.testing.assert_array_equal(O.oeq_permutation(p), g["perm"])


@pytest.mark.parametrize("name", golden_names("tp"))
def test_forward_backward_match_reference(name):
    g = load_golden(name)
    p = oracle_problem(g)
    Z = O.forward(p, g["X"], g["Y"], g["W_e3nn"])
    assert O.normalized_max_error(Z, g["Z"]) < 1e-13
    gX, gY, gW = O.backward(p, g["bX"], g["bY"], g["bW_e3nn"], g["G"])
    assert O.normalized_max_error(gX, g["gX"]) < 1e-13
    assert O.normalized_max_error(gY, g["gY"]) < 1e-13
    assert O.normalized_max_error(gW[..., g["perm"]], g["gW_oeq"]) < 1e-13


@pytest.mark.parametrize("name", golden_names("conv"))
def test_conv_matches_reference(name):
    g = load_golden(name)
    p = oracle_problem(g)
    rows, cols = g["rows"], g["cols"]
    assert np.all(np.diff(rows) >= 0), "golden graph is receiver-sorted"
    # transpose_perm lists edges in (sender, receiver) order.
    tp = g["transpose_perm"]
    keys = list(zip(cols[tp], rows[tp]))
    assert keys == sorted(keys)
    Z = O.conv_forward(p, g["X"], g["Y"], g["W_e3nn"], rows, cols)
    assert O.normalized_max_error(Z, g["Z"]) < 1e-13
    gX, gY, gW = O.conv_backward(p, g["X"], g["Y"], g["W_e3nn"], g["G"], rows, cols)
    assert O.normalized_max_error(gX, g["gX"]) < 1e-13
    assert O.normalized_max_error(gY, g["gY"]) < 1e-13
    assert O.normalized_max_error(gW[..., g["perm"]], g["gW_oeq"]) < 1e-13


def test_double_backward_identity():
    """<a,gX>+<b,gY>+<c,gW> = <G, d/dt f(X+ta, Y+tb, W+tc)> checked by finite differences."""
    rng = np.random.default_rng(3)
    p = O.make_problem("3x1e+2x0e", "1x1o+1x2e", "3x1o+3x2o+2x2e",
                       [(0, 0, 0, "uvu", True), (0, 1, 1, "uvu", True), (1, 1, 2, "uvu", True)])
    B = 4
    X, Y = rng.normal(size=(B, 13)), rng.normal(size=(B, 8))
    W = rng.normal(size=(B, p.weight_numel))
    G = rng.normal(size=(B, 9 + 15 + 10))
    a, b, c = rng.normal(size=X.shape), rng.normal(size=Y.shape), rng.normal(size=W.shape)
    gX, gY, gW, gG = O.double_backward(p, X, Y, W, G, a, b, c)
    # gG is the directional derivative of f along (a, b, c): f is trilinear, so the
    # central difference is exact up to the cubic term.
    h = 1e-4
    fd = (O.forward(p, X + h * a, Y + h * b, W + h * c) - O.forward(p, X - h * a, Y - h * b,
                                                                   W - h * c)) / (2 * h)
    np.testing.assert_allclose(gG, fd, rtol=1e-6, atol=1e-8)
    # gX = d/dX <G, directional derivative> etc.: check one random direction.
    d = rng.normal(size=X.shape)

    def s(Xv):
        bX, bY, bW = O.backward(p, Xv, Y, W, G)
        return np.sum(a * bX) + np.sum(b * bY) + np.sum(c * bW)

    fd_x = (s(X + h * d) - s(X - h * d)) / (2 * h)
    assert abs(fd_x - np.sum(gX * d)) < 1e-6 * max(1, abs(fd_x))
