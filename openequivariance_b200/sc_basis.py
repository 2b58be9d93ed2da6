"""Coupled product basis of the MACE symmetric contraction and its monomial form.

``u_matrix_real`` reproduces the reference's ``U_matrix_real``
(``_torch/symmetric_contraction/SymmetricContraction.py:17-121``): ``correlation`` copies
of the coupling irreps are coupled left to right with real Wigner 3j symbols (component
normalisation: each coupling scaled by ``sqrt(2 l_out + 1)``), every coupling path becomes
a basis tensor of shape ``[2 l_out + 1, K, ..., K]``, paths are ordered stably by output
irrep ``(l, p)``, and the U matrix of one output irrep stacks that irrep's paths on a new
last axis after dropping singleton axes.  For correlation 4 the intermediate irreps are
restricted to ``l < 12`` with parity ``(-1)^l`` as in the reference.

``monomial_map`` gives the symmetrisation used by the fused kernels: a contraction
``sum T[i1..inu] x_i1 .. x_inu`` equals ``sum_m S[m] phi_m(x)`` over the distinct monomials
``phi_m`` (sorted index tuples), with ``S = T_flat @ P`` for the 0/1 matrix ``P`` returned
here.  Monomials are ordered by degree, then lexicographically, as the kernels expect.
"""

from __future__ import annotations

import itertools
import math
from functools import lru_cache
from typing import List, Sequence, Tuple

import numpy as np

from .cg import real_wigner_3j


def _couple(paths, coupling: Sequence[Tuple[int, int]], dims: List[int], filt):
    """Adds one more copy of the coupling irreps to every path."""
    k = sum(2 * l + 1 for l, _ in coupling)
    new = []
    for (ll, pl), tensor in paths:
        start = 0
        for l, p in coupling:
            d = 2 * l + 1
            for lo in range(abs(ll - l), ll + l + 1):
                po = pl * p
                if filt is not None and (lo, po) not in filt:
                    continue
                w = real_wigner_3j(lo, ll, l) * math.sqrt(2 * lo + 1)
                # [out, left-path (flattened input axes), new irrep]
                c = np.tensordot(w, tensor.reshape(2 * ll + 1, -1), axes=([1], [0]))
                c = np.moveaxis(c, 1, 2).reshape(2 * lo + 1, *dims, d)
                t = np.zeros((2 * lo + 1, *dims, k))
                t[..., start:start + d] = c
                new.append(((lo, po), t))
            start += d
    return new


@lru_cache(maxsize=None)
def u_matrix_real(coupling: Tuple[Tuple[int, int], ...], ir_out: Tuple[int, int],
                  correlation: int) -> np.ndarray:
    """U of output irrep ``ir_out`` for ``coupling`` = ((l, p), ...), one copy of each."""
    k = sum(2 * l + 1 for l, _ in coupling)
    filt = None
    if correlation == 4:
        filt = {(i, 1 if i % 2 == 0 else -1) for i in range(12)}
    paths = []
    start = 0
    for l, p in coupling:
        t = np.zeros((2 * l + 1, k))
        t[:, start:start + 2 * l + 1] = np.eye(2 * l + 1)
        paths.append(((l, p), t))
        start += 2 * l + 1
    dims = [k]
    for _ in range(correlation - 1):
        paths = _couple(paths, coupling, dims, filt)
        paths.sort(key=lambda item: item[0])  # stable: equal irreps keep their order
        dims = dims + [k]
    cols = [np.squeeze(t)[..., None] for ir, t in paths if ir == tuple(ir_out)]
    if not cols:
        raise ValueError(f"output irrep {ir_out} is not reachable at correlation {correlation}")
    return np.concatenate(cols, axis=-1)


def monomials(k: int, degree: int) -> List[Tuple[int, ...]]:
    """Distinct monomials of degree ``degree`` in k variables (sorted index tuples)."""
    return list(itertools.combinations_with_replacement(range(k), degree))


def monomial_count(k: int, degree: int) -> int:
    return sum(len(monomials(k, d)) for d in range(1, degree + 1))


@lru_cache(maxsize=None)
def monomial_map(k: int, degree: int) -> np.ndarray:
    """0/1 matrix [k**degree, n_monomials(degree)] mapping index tuples to monomials."""
    mons = monomials(k, degree)
    pos = {m: i for i, m in enumerate(mons)}
    P = np.zeros((k ** degree, len(mons)))
    for flat, idx in enumerate(itertools.product(range(k), repeat=degree)):
        P[flat, pos[tuple(sorted(idx))]] = 1.0
    return P
