"""CPU oracle for the Clebsch-Gordan tensor-product hot path -- TEST INFRASTRUCTURE ONLY.

This module is the checker, never the product: only ``tests/``, ``__graft_entry__.smoke()``
and ``bench.py``'s CPU-baseline leg use it.  It restates, in plain numpy (float64), the
semantics the reference delegates to e3nn (its correctness oracle is
``_torch/E3NNTensorProduct.py:23-96`` / ``_torch/E3NNConv.py``, which are not installed
here), written independently of ``openequivariance_b200``:

* real-basis Wigner 3j in e3nn's convention (reference ``core/e3nn_lite.py:656-864``):
  SU(2) Clebsch-Gordan coefficients from Racah's sum, rotated to the real basis with the
  ``(-i)^l`` phase, normalised to unit Frobenius norm;
* path normalisation of ``TPProblem`` (``core/e3nn_lite.py:502-578``);
* ``uvu``/``uvw`` contractions with e3nn weight order ``[u,v]`` / ``[u,v,w]``
  (index roles as in ``templates/loop_unroll_tp.cuh:47-85``);
* the reference's "oeq" weight order (``core/ComputationSchedule.py:187-345,653-714``),
  restated by enumerating the 32-chunk child instructions explicitly;
* the fused convolution ``z[rows[e]] += TP(x[cols[e]], y[e], W[e])``
  (``core/ConvolutionBase.py:300-309``);
* the symmetric-gradient identities used for backward / double backward.

Parity pin: ``tests/test_oracle_golden.py`` checks every piece against fixtures generated
from the reference itself (``tests/golden/make_golden.py``).
"""

from __future__ import annotations

import functools
import math
from dataclasses import dataclass, field
from typing import List, Sequence, Tuple

import numpy as np

# --------------------------------------------------------------------------- CG tables


def _racah(j1, m1, j2, m2, j3, m3) -> float:
    if m1 + m2 != m3 or not abs(j1 - j2) <= j3 <= j1 + j2:
        return 0.0
    if abs(m1) > j1 or abs(m2) > j2 or abs(m3) > j3:
        return 0.0
    f = math.factorial
    norm = ((2 * j3 + 1) * f(j1 + j2 - j3) * f(j1 - j2 + j3) * f(-j1 + j2 + j3)
            / f(j1 + j2 + j3 + 1))
    norm *= f(j1 + m1) * f(j1 - m1) * f(j2 + m2) * f(j2 - m2) * f(j3 + m3) * f(j3 - m3)
    total = 0.0
    for k in range(0, j1 + j2 + j3 + 1):
        dens = (k, j1 + j2 - j3 - k, j1 - m1 - k, j2 + m2 - k, j3 - j2 + m1 + k,
                j3 - j1 - m2 + k)
        if min(dens) < 0:
            continue
        total += (-1) ** k / math.prod(f(d) for d in dens)
    return math.sqrt(norm) * total


def _q_entries(l):
    """Non-zero entries (complex_row, real_col, value) of e3nn's real->complex basis."""
    s = 1 / math.sqrt(2)
    phase = (-1j) ** l
    out = []
    for m in range(-l, l + 1):
        if m < 0:
            out += [(l + m, l - m, s * phase), (l + m, l + m, -1j * s * phase)]
        elif m == 0:
            out += [(l, l, phase)]
        else:
            out += [(l + m, l + m, (-1) ** m * s * phase), (l + m, l - m, 1j * (-1) ** m * s * phase)]
    return out


@functools.lru_cache(maxsize=None)
def wigner_3j(l1: int, l2: int, l3: int) -> np.ndarray:
    c = np.zeros((2 * l1 + 1, 2 * l2 + 1, 2 * l3 + 1), dtype=np.complex128)
    q1, q2, q3 = _q_entries(l1), _q_entries(l2), _q_entries(l3)
    for i, a, qa in q1:
        for k, b, qb in q2:
            for n, cc, qc in q3:
                su2 = _racah(l1, i - l1, l2, k - l2, l3, n - l3)
                if su2:
                    c[a, b, cc] += qa * qb * np.conj(qc) * su2
    c = c.real
    c /= np.linalg.norm(c)
    return c


# --------------------------------------------------------------------------- problems


def parse_irreps(text: str) -> List[Tuple[int, int, int]]:
    """'128x0e+1x1o' -> [(mul, l, parity)]"""
    out = []
    for term in text.replace(" ", "").split("+"):
        if not term:
            continue
        mul, ir = term.split("x") if "x" in term else ("1", term)
        l = int(ir[:-1])
        p = {"e": 1, "o": -1, "y": (-1) ** l}[ir[-1]]
        out.append((int(mul), l, p))
    return out


@dataclass
class Problem:
    irreps1: List[Tuple[int, int, int]]
    irreps2: List[Tuple[int, int, int]]
    irreps3: List[Tuple[int, int, int]]
    instructions: List[tuple]  # (i1, i2, i3, mode, has_weight[, path_weight])
    shared_weights: bool = False
    irrep_normalization: str = "component"
    path_normalization: str = "element"
    path_weights: List[float] = field(default_factory=list)
    weight_offsets: List[int] = field(default_factory=list)
    weight_numel: int = 0

    def __post_init__(self):
        self.instructions = [tuple(i) + ((1.0,) if len(i) == 5 else ()) for i in self.instructions]
        self._normalise()

    @staticmethod
    def dims(irreps):
        offs, o = [], 0
        for mul, l, _ in irreps:
            offs.append(o)
            o += mul * (2 * l + 1)
        return offs, o

    def shape(self, ins):
        i1, i2, i3, mode = ins[:4]
        m1, m2, m3 = self.irreps1[i1][0], self.irreps2[i2][0], self.irreps3[i3][0]
        return (m1, m2) if mode == "uvu" else (m1, m2, m3)

    def _normalise(self):
        def fan(ins):
            m1, m2 = self.irreps1[ins[0]][0], self.irreps2[ins[1]][0]
            return m2 if ins[3] == "uvu" else m1 * m2

        self.path_weights = []
        for ins in self.instructions:
            l1, l2, l3 = self.irreps1[ins[0]][1], self.irreps2[ins[1]][1], self.irreps3[ins[2]][1]
            alpha = {"component": 2 * l3 + 1, "norm": (2 * l1 + 1) * (2 * l2 + 1),
                     "none": 1}[self.irrep_normalization]
            same = [o for o in self.instructions if o[2] == ins[2]]
            if self.path_normalization == "element":
                x = sum(fan(o) for o in same)
            elif self.path_normalization == "path":
                x = fan(ins) * len(same)
            else:
                x = 1
            if x > 0:
                alpha /= x
            alpha *= ins[5]
            self.path_weights.append(math.sqrt(alpha))
        self.weight_offsets, o = [], 0
        for ins in self.instructions:
            self.weight_offsets.append(o)
            o += math.prod(self.shape(ins))
        self.weight_numel = o


def make_problem(in1: str, in2: str, out: str, instructions: Sequence[tuple],
                 shared_weights=False, **kw) -> Problem:
    return Problem(parse_irreps(in1), parse_irreps(in2), parse_irreps(out), list(instructions),
                   shared_weights=shared_weights, **kw)


# --------------------------------------------------------------------------- weight order


def oeq_permutation(p: Problem, chunk: int = 32) -> np.ndarray:
    """``perm`` with ``w_oeq = w_e3nn[..., perm]``: child instructions over 32-chunks of
    the multiplicities, each stored ``[v][u]`` (uvu) or ``[v][u][w]`` (uvw)."""
    perm = []
    for ins, off in zip(p.instructions, p.weight_offsets):
        shp = p.shape(ins)
        dense = np.arange(math.prod(shp)).reshape(shp) + off
        chunks = [[(s, min(s + chunk, m)) for s in range(0, m, chunk)] for m in shp]
        if ins[3] == "uvu":
            for us, ue in chunks[0]:
                for vs, ve in chunks[1]:
                    perm.append(dense[us:ue, vs:ve].T.ravel())
        else:
            for us, ue in chunks[0]:
                for vs, ve in chunks[1]:
                    for ws, we in chunks[2]:
                        perm.append(dense[us:ue, vs:ve, ws:we].transpose(1, 0, 2).ravel())
    return np.concatenate(perm).astype(np.int64) if perm else np.zeros(0, np.int64)


# --------------------------------------------------------------------------- contractions


def _blocks(arr, irreps, idx):
    offs, _ = Problem.dims(irreps)
    mul, l, _ = irreps[idx]
    return arr[:, offs[idx]:offs[idx] + mul * (2 * l + 1)].reshape(arr.shape[0], mul, 2 * l + 1)


def _wblock(p, W, k):
    shp = p.shape(p.instructions[k])
    o = p.weight_offsets[k]
    n = math.prod(shp)
    if p.shared_weights:
        return W[o:o + n].reshape(shp), True
    return W[:, o:o + n].reshape((W.shape[0],) + shp), False


def forward(p: Problem, X, Y, W):
    """Z = sum_instructions pw * contraction (e3nn weight order, mul_ir layout)."""
    B = X.shape[0]
    _, d3 = Problem.dims(p.irreps3)
    offs3, _ = Problem.dims(p.irreps3)
    Z = np.zeros((B, d3), dtype=np.float64)
    for k, ins in enumerate(p.instructions):
        x = _blocks(X, p.irreps1, ins[0])
        y = _blocks(Y, p.irreps2, ins[1])
        l1, l2, l3 = p.irreps1[ins[0]][1], p.irreps2[ins[1]][1], p.irreps3[ins[2]][1]
        C = wigner_3j(l1, l2, l3) * p.path_weights[k]
        w, shared = _wblock(p, W, k)
        if ins[3] == "uvu":
            eq = "ijk,bui,uv,bvj->buk" if shared else "ijk,bui,buv,bvj->buk"
        else:
            eq = "ijk,bui,uvw,bvj->bwk" if shared else "ijk,bui,buvw,bvj->bwk"
        z = np.einsum(eq, C, x, w, y, optimize=True)
        m3, _, _ = p.irreps3[ins[2]]
        Z[:, offs3[ins[2]]:offs3[ins[2]] + z.shape[1] * z.shape[2]] += z.reshape(B, -1)
    return Z


def backward(p: Problem, X, Y, W, G):
    """Adjoints (gX, gY, gW) of forward with output cotangent G."""
    B = X.shape[0]
    gX, gY, gW = np.zeros_like(X, dtype=np.float64), np.zeros_like(Y, dtype=np.float64), \
        np.zeros_like(W, dtype=np.float64)
    offs1, _ = Problem.dims(p.irreps1)
    offs2, _ = Problem.dims(p.irreps2)
    for k, ins in enumerate(p.instructions):
        x = _blocks(X, p.irreps1, ins[0])
        y = _blocks(Y, p.irreps2, ins[1])
        g = _blocks(G, p.irreps3, ins[2])
        l1, l2, l3 = p.irreps1[ins[0]][1], p.irreps2[ins[1]][1], p.irreps3[ins[2]][1]
        C = wigner_3j(l1, l2, l3) * p.path_weights[k]
        w, shared = _wblock(p, W, k)
        wb = "uv" if ins[3] == "uvu" else "uvw"
        gi = "buk" if ins[3] == "uvu" else "bwk"
        wbb = wb if shared else "b" + wb
        gx = np.einsum(f"ijk,{wbb},bvj,{gi}->bui", C, w, y, g, optimize=True)
        gy = np.einsum(f"ijk,bui,{wbb},{gi}->bvj", C, x, w, g, optimize=True)
        gw = np.einsum(f"ijk,bui,bvj,{gi}->{wbb}", C, x, y, g, optimize=True)
        m1, _, _ = p.irreps1[ins[0]]
        m2, _, _ = p.irreps2[ins[1]]
        gX[:, offs1[ins[0]]:offs1[ins[0]] + gx.shape[1] * gx.shape[2]] += gx.reshape(B, -1)
        gY[:, offs2[ins[1]]:offs2[ins[1]] + gy.shape[1] * gy.shape[2]] += gy.reshape(B, -1)
        o, n = p.weight_offsets[k], gw[0].size if not shared else gw.size
        if shared:
            gW[o:o + n] += gw.ravel()
        else:
            gW[:, o:o + n] += gw.reshape(B, -1)
    return gX, gY, gW


def double_backward(p: Problem, X, Y, W, G, a, b, c):
    """Gradients of <a,gX> + <b,gY> + <c,gW> w.r.t. (X, Y, W, G)."""
    gG = forward(p, a, Y, W) + forward(p, X, b, W) + forward(p, X, Y, c)
    gX1, _, gW1 = backward(p, X, b, W, G)       # bX(b,W,G), bW(X,b,G)
    _, gY2, gW2 = backward(p, a, Y, W, G)       # bY(a,W,G), bW(a,Y,G)
    gX3, gY3, _ = backward(p, X, Y, c, G)       # bX(Y,c,G), bY(X,c,G)
    return gX1 + gX3, gY2 + gY3, gW1 + gW2, gG


# --------------------------------------------------------------------------- convolution


def conv_forward(p: Problem, X, Y, W, rows, cols):
    Z = np.zeros((X.shape[0], Problem.dims(p.irreps3)[1]))
    np.add.at(Z, rows, forward(p, X[cols], Y, W))
    return Z


def conv_backward(p: Problem, X, Y, W, G, rows, cols):
    gXe, gY, gW = backward(p, X[cols], Y, W, G[rows])
    gX = np.zeros_like(X, dtype=np.float64)
    np.add.at(gX, cols, gXe)
    return gX, gY, gW


def conv_double_backward(p: Problem, X, Y, W, G, a, b, c, rows, cols):
    gX, gY, gW, gGe = double_backward(p, X[cols], Y, W, G[rows], a[cols], b, c)
    gXn = np.zeros_like(X, dtype=np.float64)
    np.add.at(gXn, cols, gX)
    gG = np.zeros((X.shape[0], Problem.dims(p.irreps3)[1]))
    np.add.at(gG, rows, gGe)
    return gXn, gY, gW, gG


def normalized_max_error(got, want) -> float:
    """max|got - want| / max(max|want|, 1e-30)."""
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    if want.size == 0:
        return 0.0
    return float(np.max(np.abs(got - want)) / max(np.max(np.abs(want)), 1e-30))
