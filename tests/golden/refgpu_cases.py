"""BASELINE-size parity cases shared by the reference-kernel fixture generator and the tests.

This module is plain numpy (plus scipy for the radius graph) so that two different processes
can import it:

* ``make_golden_refgpu.py`` runs the reference's own CUDA kernels on these cases (the
  reference registers the ``libtorch_tp_jit`` operators itself, so it runs in a process that
  never loads this package);
* ``tests/test_refgpu_parity.py`` runs this package's kernels on the same cases and compares.

Every input is regenerated from a seed, so the fixtures only hold the reference's outputs,
and of the large ones only a compact summary (see ``summarise``).

Cases (the TP problems equal ``openequivariance_b200.problems``'s
``baseline_problem``, which a CPU test checks):

* ``c1``: 1x2e (x) 1x3e -> 1x2e, one uvu path, 1000 rows, uniform[0, 1) inputs drawn from
  ``default_rng(0)`` in the order X, Y, W (the reference's ``get_random_buffers_forward``,
  ``benchmark/test_buffers.py:8-28``), float32.
* ``c2`` (literal reading, 24 paths) and ``c2ml`` (the reference's ``mace-large``, 17 paths):
  1000 rows, X, Y, W ~ N(0, 1), float32.
* ``c4``: NequIP uvw, 30 paths, shared weights, 20,000 rows, float32 and float64.
* ``c3``: the fused convolution on the BASELINE graph (5,000 nodes uniform in a periodic 25 A
  cube, 5 A cutoff: 839,872 directed edges, receiver-sorted as the reference's
  ``CoordGraph``, ``core/ConvolutionBase.py:57-82``), 1x2e (x) 1x3e -> 1x2e with per-edge
  weights, atomic and deterministic, float32.

Y rows are standard normal draws rather than spherical harmonics of the edge vectors: the
products are linear in Y, so parity does not depend on where its values come from.
"""

from __future__ import annotations

import hashlib

import numpy as np

C2_OUT = ("128x0e+128x0e+128x0e+128x1o+128x1o+128x1o+128x1o+128x1o+128x1e+128x1e+128x2o+"
          "128x2o+128x2o+128x2e+128x2e+128x2e+128x2e+128x2e+128x3o+128x3o+128x3o+128x3o+"
          "128x3e+128x3e")
C2_INS = [(0, 0, 0), (1, 1, 1), (2, 2, 2), (0, 1, 3), (1, 0, 4), (1, 2, 5), (2, 1, 6), (2, 3, 7),
          (1, 1, 8), (2, 2, 9), (1, 2, 10), (2, 1, 11), (2, 3, 12), (0, 2, 13), (1, 1, 14),
          (1, 3, 15), (2, 0, 16), (2, 2, 17), (0, 3, 18), (1, 2, 19), (2, 1, 20), (2, 3, 21),
          (1, 3, 22), (2, 2, 23)]
C2ML_OUT = ("128x0e+128x0e+128x0e+128x1o+128x1o+128x1o+128x1o+128x1o+128x2e+128x2e+128x2e+"
            "128x2e+128x2e+128x3o+128x3o+128x3o+128x3o")
C2ML_INS = [(0, 0, 0), (1, 1, 1), (2, 2, 2), (0, 1, 3), (1, 0, 4), (1, 2, 5), (2, 1, 6),
            (2, 3, 7), (0, 2, 8), (1, 1, 9), (1, 3, 10), (2, 0, 11), (2, 2, 12), (0, 3, 13),
            (1, 2, 14), (2, 1, 15), (2, 3, 16)]
C4_IR = "32x0e+32x0o+32x1e+32x1o+32x2e+32x2o"
C4_INS = [(0, 0, 0), (0, 1, 3), (0, 2, 4), (1, 0, 1), (1, 1, 2), (1, 2, 5), (2, 0, 2), (2, 1, 1),
          (2, 1, 3), (2, 1, 5), (2, 2, 2), (2, 2, 4), (3, 0, 3), (3, 1, 0), (3, 1, 2), (3, 1, 4),
          (3, 2, 3), (3, 2, 5), (4, 0, 4), (4, 1, 3), (4, 1, 5), (4, 2, 0), (4, 2, 2), (4, 2, 4),
          (5, 0, 5), (5, 1, 2), (5, 1, 4), (5, 2, 1), (5, 2, 3), (5, 2, 5)]

# name -> (irreps_in1, irreps_in2, irreps_out, [(i1, i2, i3)], mode, shared, dtype, rows)
TP_CASES = {
    "c1": ("1x2e", "1x3e", "1x2e", [(0, 0, 0)], "uvu", False, "float32", 1000),
    "c2": ("128x0e+128x1o+128x2e", "1x0e+1x1o+1x2e+1x3o", C2_OUT, C2_INS, "uvu", False,
           "float32", 1000),
    "c2ml": ("128x0e+128x1o+128x2e", "1x0e+1x1o+1x2e+1x3o", C2ML_OUT, C2ML_INS, "uvu", False,
             "float32", 1000),
    "c4_f32": (C4_IR, "1x0e+1x1o+1x2e", C4_IR, C4_INS, "uvw", True, "float32", 20000),
    "c4_f64": (C4_IR, "1x0e+1x1o+1x2e", C4_IR, C4_INS, "uvw", True, "float64", 20000),
}
# Cases whose double backward is also pinned (the others: forward and backward).
DOUBLE_BACKWARD = ("c1", "c4_f64")

CONV_CASE = ("1x2e", "1x3e", "1x2e", [(0, 0, 0)], "uvu", False, "float32")
C3_NODES, C3_BOX, C3_CUTOFF = 5000, 25.0, 5.0
C3_EDGES = 839_872

N_SAMPLE_ROWS = 8


def irreps_dim(s: str) -> int:
    d = 0
    for term in s.split("+"):
        mul, ir = term.split("x")
        d += int(mul) * (2 * int(ir[:-1]) + 1)
    return d


def weight_numel(case) -> int:
    in1, in2, out, ins, mode, shared = case[:6]

    def blocks(s):
        return [(int(t.split("x")[0]), int(t.split("x")[1][:-1])) for t in s.split("+")]

    b1, b2, b3 = blocks(in1), blocks(in2), blocks(out)
    n = 0
    for i, j, k in ins:
        n += b1[i][0] * b2[j][0] * (b3[k][0] if mode == "uvw" else 1)
    return n


def tp_inputs(name: str):
    """Seeded inputs of a TP case: X, Y, W, dZ and (double backward) ddX, ddY, ddW."""
    case = TP_CASES[name]
    in1, in2, out, _, _, shared, dt, rows = case
    wn = weight_numel(case)
    wshape = (wn,) if shared else (rows, wn)
    if name == "c1":
        rng = np.random.default_rng(0)
        X = rng.uniform(size=(rows, irreps_dim(in1)))
        Y = rng.uniform(size=(rows, irreps_dim(in2)))
        W = rng.uniform(size=wshape)
        dZ = rng.uniform(size=(rows, irreps_dim(out)))
    else:
        rng = np.random.default_rng(1 + sorted(TP_CASES).index(name))
        X = rng.standard_normal((rows, irreps_dim(in1)))
        Y = rng.standard_normal((rows, irreps_dim(in2)))
        W = rng.standard_normal(wshape) * (0.1 if shared else 1.0)
        dZ = rng.standard_normal((rows, irreps_dim(out)))
    ddX = rng.standard_normal(X.shape)
    ddY = rng.standard_normal(Y.shape)
    ddW = rng.standard_normal(W.shape)
    cast = np.float32 if dt == "float32" else np.float64
    return tuple(a.astype(cast) for a in (X, Y, W, dZ, ddX, ddY, ddW))


def c3_graph():
    """(rows, cols, transpose_perm): the BASELINE C3 radius graph, receiver-sorted.

    Positions uniform in [0, 25)^3 from ``default_rng(0)``; every ordered pair (receiver i,
    sender j), i != j, with minimum-image distance below 5; sorted by (receiver, sender);
    ``transpose_perm`` lists the sorted positions in (sender, receiver) order.
    """
    from scipy.spatial import cKDTree

    rng = np.random.default_rng(0)
    pos = rng.uniform(0.0, C3_BOX, size=(C3_NODES, 3))
    tree = cKDTree(pos, boxsize=C3_BOX)
    pairs = tree.query_pairs(C3_CUTOFF, output_type="ndarray")
    i = np.concatenate([pairs[:, 0], pairs[:, 1]]).astype(np.int64)
    j = np.concatenate([pairs[:, 1], pairs[:, 0]]).astype(np.int64)
    order = np.lexsort((j, i))
    rows, cols = i[order], j[order]
    tperm = np.lexsort((rows, cols)).astype(np.int64)
    return rows, cols, tperm


def graph_digest(rows: np.ndarray, cols: np.ndarray) -> str:
    h = hashlib.sha256()
    h.update(np.ascontiguousarray(rows, dtype=np.int64).tobytes())
    h.update(np.ascontiguousarray(cols, dtype=np.int64).tobytes())
    return h.hexdigest()


def conv_inputs(nnz: int):
    """Seeded inputs of the C3 convolution: X [nodes, 5], Y [E, 7], W [E, 1], dZ [nodes, 5]."""
    rng = np.random.default_rng(1234)
    X = rng.standard_normal((C3_NODES, 5)).astype(np.float32)
    Y = rng.standard_normal((nnz, 7)).astype(np.float32)
    W = rng.standard_normal((nnz, 1)).astype(np.float32)
    dZ = rng.standard_normal((C3_NODES, 5)).astype(np.float32)
    return X, Y, W, dZ


def summarise(key: str, a: np.ndarray, out: dict) -> None:
    """Stores a compact, size-independent summary of an output array under ``key``.

    Arrays of at most 64 Ki elements are stored whole.  Larger ones [R, D] are stored as
    ``N_SAMPLE_ROWS`` seeded sample rows plus two float64 sketches that touch every element:
    ``key:rowsk`` = A @ r (one value per row) and ``key:colsk`` = s @ A (one per column), with
    r, s seeded standard normal vectors.  A wrong element anywhere moves a sketch entry by
    about its own error, so sketches compared with the same normalised bound as the elements
    check the whole array.  Row sketches of more than ``ROW_BLOCKS`` rows are folded into
    blocks (``block_sketch``).
    """
    a = np.asarray(a)
    if a.size <= 65536:
        out[key] = a
        return
    a2 = a.reshape(a.shape[0], -1).astype(np.float64)
    rows = sample_rows(a2.shape[0])
    out[key + ":rows"] = a[rows]
    r, s = sketch_vectors(a2.shape[0], a2.shape[1])
    out[key + ":rowsk"] = block_sketch(a2 @ r)
    out[key + ":colsk"] = s @ a2


ROW_BLOCKS = 4096


def block_sketch(v: np.ndarray) -> np.ndarray:
    """Per-row sketch values folded into at most ``ROW_BLOCKS`` contiguous blocks, each a
    seeded random combination of its rows (so a change in any row moves its block)."""
    n = v.shape[0]
    if n <= ROW_BLOCKS:
        return v
    t = np.random.default_rng(11).standard_normal(n)
    starts = (np.arange(ROW_BLOCKS, dtype=np.int64) * n) // ROW_BLOCKS
    return np.add.reduceat(v * t, starts)


def sample_rows(n: int) -> np.ndarray:
    return np.sort(np.random.default_rng(99).choice(n, size=min(N_SAMPLE_ROWS, n), replace=False))


def sketch_vectors(nrows: int, ncols: int):
    rng = np.random.default_rng(7)
    return rng.standard_normal(ncols), rng.standard_normal(nrows)


def normalised_error(got, want) -> float:
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    return float(np.max(np.abs(got - want)) / max(np.max(np.abs(want)), 1e-30)) if want.size else 0.0


def compare(key: str, got: np.ndarray, fixture: dict) -> float:
    """Normalised max error of ``got`` against the summary stored under ``key``."""
    if key in fixture:
        return normalised_error(got, fixture[key])
    g2 = np.asarray(got).reshape(got.shape[0], -1).astype(np.float64)
    r, s = sketch_vectors(g2.shape[0], g2.shape[1])
    return max(normalised_error(np.asarray(got)[sample_rows(g2.shape[0])], fixture[key + ":rows"]),
               normalised_error(block_sketch(g2 @ r), fixture[key + ":rowsk"]),
               normalised_error(s @ g2, fixture[key + ":colsk"]))
