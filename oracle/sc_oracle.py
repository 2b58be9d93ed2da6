"""CPU oracle for the MACE symmetric contraction -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU legs use this module; it
is the checker, never the product.  It restates in torch-CPU float64 (autograd supplies the
gradients), independently of ``openequivariance_b200``:

* the coupled product basis ``_wigner_nj`` and ``U_matrix_real`` of the reference
  (``_torch/symmetric_contraction/SymmetricContraction.py:17-121``): recursive coupling of
  ``correlation`` copies of the input irreps with real Wigner 3j symbols (component
  normalisation, ``sqrt(2 l_out + 1)``), entries sorted by output irrep (stable), and the
  U matrix of an output irrep = its entries stacked on a new last axis after dropping
  singleton axes;
* ``Contraction.forward`` (``SymmetricContraction.py:220-253``): the top correlation
  ``out = sum_k (W_max U_max)[..., k] x_k`` followed by, for each lower correlation,
  ``out = sum_last ((W_nu U_nu) + out) x``;
* ``SymmetricContraction.forward`` (``SymmetricContraction.py:324-336``): the element of a
  node is the argmax of its one-hot row; per-node results are concatenated over output
  irreps (the reference's sort/unsort by element does not change any value).

Parity pin: ``tests/test_sc_oracle.py`` checks the U matrices, outputs and all gradients
against ``tests/golden/sc_*.npz``, generated from the reference module itself
(``tests/golden/make_golden_sc.py``).
"""

from __future__ import annotations

import math
import os
import sys
from typing import Dict, List, Sequence, Tuple

import numpy as np
import torch

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
from tp_oracle import parse_irreps, wigner_3j  # noqa: E402

Irrep = Tuple[int, int]  # (l, parity)


def _coupled_basis(irreps_list: Sequence[List[Tuple[int, int, int]]], filter_mid=None):
    """[(irrep_out, E)] with E of shape [2 l_out + 1, *input dims], sorted by irrep_out."""
    if len(irreps_list) == 1:
        irreps = irreps_list[0]
        dim = sum(m * (2 * l + 1) for m, l, _ in irreps)
        out, i = [], 0
        for mul, l, p in irreps:
            for _ in range(mul):
                E = np.zeros((2 * l + 1, dim))
                E[:, i:i + 2 * l + 1] = np.eye(2 * l + 1)
                out.append(((l, p), E))
                i += 2 * l + 1
        return out
    left, right = irreps_list[:-1], irreps_list[-1]
    dim_r = sum(m * (2 * l + 1) for m, l, _ in right)
    left_dims = [sum(m * (2 * l + 1) for m, l, _ in irr) for irr in left]
    out = []
    for (ll, pl), c_left in _coupled_basis(left, filter_mid):
        i = 0
        for mul, l, p in right:
            for lo in range(abs(ll - l), ll + l + 1):
                po = pl * p
                if filter_mid is not None and (lo, po) not in filter_mid:
                    continue
                w = wigner_3j(lo, ll, l) * math.sqrt(2 * lo + 1)
                c = np.einsum("jk,ijl->ikl", c_left.reshape(2 * ll + 1, -1), w)
                c = c.reshape(2 * lo + 1, *left_dims, 2 * l + 1)
                for u in range(mul):
                    E = np.zeros((2 * lo + 1, *left_dims, dim_r))
                    E[..., i + u * (2 * l + 1): i + (u + 1) * (2 * l + 1)] = c
                    out.append(((lo, po), E))
            i += mul * (2 * l + 1)
    return sorted(out, key=lambda t: t[0])


def u_matrix(coupling: List[Tuple[int, int, int]], ir_out: Irrep, correlation: int) -> np.ndarray:
    """U of one output irrep: [*(2l+1 if > 1), *input dims, n_paths] (singleton axes dropped)."""
    filt = None
    if correlation == 4:
        filt = [(i, 1 if i % 2 == 0 else -1) for i in range(12)]
    basis = _coupled_basis([coupling] * correlation, filt)
    cols = [np.squeeze(E)[..., None] for ir, E in basis if ir == tuple(ir_out)]
    return np.concatenate(cols, axis=-1)


class ScProblem:
    """A symmetric contraction: irreps_in = C x (coupling irreps), irreps_out = C x (outs)."""

    def __init__(self, irreps_in: str, irreps_out: str, correlation: int, num_elements: int):
        ins = parse_irreps(irreps_in)
        outs = parse_irreps(irreps_out)
        self.num_features = sum(m for m, l, p in ins if l == 0 and p == 1)
        self.coupling = [(1, l, p) for _, l, p in ins]
        self.k = sum(2 * l + 1 for _, l, _ in self.coupling)
        self.outs = [(l, p) for _, l, p in outs]
        self.correlation = correlation
        self.num_elements = num_elements
        self.U: List[Dict[int, np.ndarray]] = [
            {nu: u_matrix(self.coupling, ir, nu) for nu in range(1, correlation + 1)}
            for ir in self.outs]

    def weight_shapes(self) -> List[List[Tuple[int, int, int]]]:
        """Per output irrep: [weights_max shape, then weights[0..] shapes] as in the reference."""
        shapes = []
        for U in self.U:
            s = [(self.num_elements, U[self.correlation].shape[-1], self.num_features)]
            s += [(self.num_elements, U[nu].shape[-1], self.num_features)
                  for nu in range(self.correlation - 1, 0, -1)]
            shapes.append(s)
        return shapes


def _contract(U: Dict[int, np.ndarray], corr: int, w_max, ws, x, elem):
    """One output irrep's contraction for every node (torch float64)."""
    Ut = {nu: torch.as_tensor(U[nu]) for nu in U}
    # T_nu[e, c, ...] = sum_p W_nu[e, p, c] U_nu[..., p]
    t = torch.einsum("epc,...p->ec...", w_max, Ut[corr])[elem]        # [N, C, *U.shape[:-1]]
    out = (t * x.view(x.shape[0], x.shape[1], *([1] * (t.dim() - 3)), x.shape[2])).sum(-1)
    for i, w in enumerate(ws):
        nu = corr - i - 1
        t = torch.einsum("epc,...p->ec...", w, Ut[nu])[elem] + out
        out = (t * x.view(x.shape[0], x.shape[1], *([1] * (t.dim() - 3)), x.shape[2])).sum(-1)
    return out.reshape(out.shape[0], -1)


def forward(prob: ScProblem, weights: List[List[torch.Tensor]], x: torch.Tensor,
            elem: torch.Tensor) -> torch.Tensor:
    """Symmetric contraction of x [N, C, K] for nodes of elements elem [N] -> [N, sum(C d_out)]."""
    outs = [_contract(U, prob.correlation, w[0], w[1:], x, elem)
            for U, w in zip(prob.U, weights)]
    return torch.cat(outs, dim=-1)


def random_weights(prob: ScProblem, seed: int, dtype=torch.float64) -> List[List[torch.Tensor]]:
    g = torch.Generator().manual_seed(seed)
    return [[torch.randn(s, dtype=dtype, generator=g) / s[1] for s in shapes]
            for shapes in prob.weight_shapes()]
