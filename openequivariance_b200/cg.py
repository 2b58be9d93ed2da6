"""Real-basis Clebsch-Gordan (Wigner 3j) tables in e3nn's convention.

The reference builds these in ``core/e3nn_lite.py:656-864``: SU(2) Clebsch-Gordan
coefficients in exact rationals, a change of basis to real spherical harmonics
(with an extra ``(-i)^l`` phase so the result is real), and a normalisation to unit
Frobenius norm.  This module computes the same tensor from the textbook Racah
formula for the SU(2) coefficients, so the two implementations share only the
convention, not the code path.  Parity with the reference's ``wigner_3j`` is pinned
by ``tests/test_cg.py`` against fixtures generated from the reference.

The sparse lists produced here feed two consumers: the build-time generator of the
unrolled CUDA device code (``csrc/gen_cg.py``) and the run-time table used by the
kernels' generic path for degrees above the unrolled range.
"""

from __future__ import annotations

import functools
from fractions import Fraction
from math import factorial, sqrt
from typing import List, Tuple

import numpy as np

__all__ = ["su2_cg", "real_wigner_3j", "sparse_cg", "valid_triples"]


def _fact(n: int) -> int:
    return factorial(n)


def su2_cg(j1: int, m1: int, j2: int, m2: int, j3: int, m3: int) -> float:
    """<j1 m1; j2 m2 | j3 m3> for integer angular momenta (Condon-Shortley phase)."""
    if m1 + m2 != m3:
        return 0.0
    if not (abs(j1 - j2) <= j3 <= j1 + j2):
        return 0.0
    if abs(m1) > j1 or abs(m2) > j2 or abs(m3) > j3:
        return 0.0
    # Racah's closed form: sqrt(prefactor) * sum_k (-1)^k / (product of factorials).
    pref = Fraction(
        (2 * j3 + 1) * _fact(j3 + j1 - j2) * _fact(j3 - j1 + j2) * _fact(j1 + j2 - j3),
        _fact(j1 + j2 + j3 + 1),
    )
    pref *= (
        _fact(j3 + m3) * _fact(j3 - m3) * _fact(j1 - m1) * _fact(j1 + m1)
        * _fact(j2 - m2) * _fact(j2 + m2)
    )
    total = Fraction(0)
    k = 0
    while True:
        args = (k, j1 + j2 - j3 - k, j1 - m1 - k, j2 + m2 - k,
                j3 - j2 + m1 + k, j3 - j1 - m2 + k)
        if args[1] < 0 or args[2] < 0 or args[3] < 0:
            break
        if min(args) >= 0:
            den = 1
            for a in args:
                den *= _fact(a)
            total += Fraction((-1) ** k, den)
        k += 1
    # sqrt of the prefactor times the (exact) alternating sum.
    return float(np.sign(float(total))) * sqrt(float(pref * total * total)) if total != 0 else 0.0


def _real_to_complex(l: int) -> np.ndarray:  # noqa: E741
    """Columns: real basis m=-l..l; rows: complex basis m=-l..l (e3nn phase convention)."""
    q = np.zeros((2 * l + 1, 2 * l + 1), dtype=np.complex128)
    r = 1.0 / np.sqrt(2.0)
    for m in range(-l, l + 1):
        row = l + m
        if m < 0:
            q[row, l - m] = r
            q[row, l + m] = -1j * r
        elif m == 0:
            q[row, l] = 1.0
        else:
            s = (-1) ** m
            q[row, l + m] = s * r
            q[row, l - m] = 1j * s * r
    return ((-1j) ** l) * q


@functools.lru_cache(maxsize=None)
def _real_w3j_cached(l1: int, l2: int, l3: int) -> np.ndarray:
    su2 = np.zeros((2 * l1 + 1, 2 * l2 + 1, 2 * l3 + 1), dtype=np.float64)
    for a in range(2 * l1 + 1):
        for b in range(2 * l2 + 1):
            m3 = (a - l1) + (b - l2)
            if abs(m3) <= l3:
                su2[a, b, l3 + m3] = su2_cg(l1, a - l1, l2, b - l2, l3, m3)
    q1, q2, q3 = _real_to_complex(l1), _real_to_complex(l2), _real_to_complex(l3)
    c = np.einsum("ia,kb,nc,ikn->abc", q1, q2, np.conj(q3), su2.astype(np.complex128))
    if np.max(np.abs(c.imag)) > 1e-8:
        raise AssertionError("real Clebsch-Gordan tensor has an imaginary part")
    c = c.real
    return c / np.linalg.norm(c.ravel())


def real_wigner_3j(l1: int, l2: int, l3: int) -> np.ndarray:
    """Dense real CG tensor of shape ``[2l1+1, 2l2+1, 2l3+1]`` with unit Frobenius norm."""
    if not (abs(l2 - l3) <= l1 <= l2 + l3):
        raise ValueError(f"({l1},{l2},{l3}) violates the triangle rule")
    return _real_w3j_cached(int(l1), int(l2), int(l3)).copy()


# Entries smaller than this (relative to the unit-norm tensor) are numerical zeros of
# the basis change; the exact tensor has them at 0.
_ZERO_TOL = 1e-12


@functools.lru_cache(maxsize=None)
def sparse_cg(l1: int, l2: int, l3: int) -> Tuple[Tuple[int, int, int, float], ...]:
    """Non-zero entries ``(i, j, k, value)`` sorted by ``(i, j, k)``."""
    c = real_wigner_3j(l1, l2, l3)
    out: List[Tuple[int, int, int, float]] = []
    for i in range(c.shape[0]):
        for j in range(c.shape[1]):
            for k in range(c.shape[2]):
                v = float(c[i, j, k])
                if abs(v) > _ZERO_TOL:
                    out.append((i, j, k, v))
    return tuple(out)


def valid_triples(lmax: int) -> List[Tuple[int, int, int]]:
    """All ``(l1, l2, l3)`` with every degree <= lmax satisfying the triangle rule."""
    return [
        (a, b, c)
        for a in range(lmax + 1)
        for b in range(lmax + 1)
        for c in range(abs(a - b), min(a + b, lmax) + 1)
    ]
