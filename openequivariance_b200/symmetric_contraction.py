"""MACE symmetric contraction with the reference's module API.

Mirrors ``openequivariance._torch.symmetric_contraction`` (reference
``_torch/symmetric_contraction/SymmetricContraction.py:146-336``): the same constructor
arguments, the same parameters (``weights_max`` and the ``weights`` list per output irrep,
created in the same order with the same initialisation, so seeded modules and state dicts
interchange) and the same buffers (``U_matrix_{nu}``, ``U_permuted_{nu}``).

Execution differs.  The reference runs the top correlation as a per-element cuBLAS batched
GEMM (``group_gemm``) into an ``[N, C, d_out * K^(nu-1)]`` intermediate, then contracts the
lower correlations with torch element-wise ops, after a host synchronisation on the element
counts.  Here the whole contraction of every output irrep is one fused kernel pass
(``torch.ops.oeqb200.sc_forward``): the weights are folded into coefficients on the distinct
monomials of x (``sc_basis.monomial_map``) with small library GEMMs, and each (node, channel)
is a polynomial evaluation in registers; nothing is materialised and nothing synchronises
with the host.  First-order gradients (x and the coefficients, hence the weights) come from
``sc_backward``; when a backward pass itself records a graph (double backward, e.g. force
training), the gradient is recomputed with differentiable torch operations on the same
monomial form.  There is no CPU path: CPU tensors and shapes outside the kernels' range
(coupling dimension other than 4 or 9, correlation above 3, more than 16 output
components) raise.
"""

from __future__ import annotations

from typing import Dict, Optional, Union

import torch

from .irreps import Irreps
from .sc_basis import monomial_map, monomials, u_matrix_real

_KERNEL_K = (4, 9)
_KERNEL_DT = (4, 16)


def _coupling(irreps_in: Irreps):
    return tuple((mi.ir.l, mi.ir.p) for mi in irreps_in)


def _count_scalars(irreps: Irreps) -> int:
    return sum(mi.mul for mi in irreps if mi.ir.l == 0 and mi.ir.p == 1)


class Contraction(torch.nn.Module):
    """Contraction for one output irrep (reference ``SymmetricContraction.py:146-261``)."""

    def __init__(self, irreps_in: Irreps, irrep_out: Irreps, correlation: int,
                 internal_weights: bool = True, num_elements: Optional[int] = None,
                 weights: Optional[torch.Tensor] = None,
                 dtype: Optional[torch.dtype] = None) -> None:
        super().__init__()
        self.num_elements = num_elements
        self.num_features = _count_scalars(irreps_in)
        self.coupling = _coupling(irreps_in)
        self.k = sum(2 * l + 1 for l, _ in self.coupling)
        self.correlation = correlation
        self.ir_out = (irrep_out[0].ir.l, irrep_out[0].ir.p)
        self.d_out = 2 * self.ir_out[0] + 1
        if dtype is None:
            dtype = torch.get_default_dtype()
        for nu in range(1, correlation + 1):
            U = u_matrix_real(self.coupling, self.ir_out, nu)
            self.register_buffer(f"U_matrix_{nu}", torch.tensor(U, dtype=dtype))
        self.weights = torch.nn.ParameterList([])
        for i in range(correlation, 0, -1):
            num_params = self.U_tensors(i).size()[-1]
            w = torch.nn.Parameter(
                torch.randn((num_elements, num_params, self.num_features), dtype=dtype) / num_params)
            if i == correlation:
                self.weights_max = w
            else:
                self.weights.append(w)
        if not internal_weights:
            self.weights = weights[:-1]
            self.weights_max = weights[-1]
        for i in range(correlation, 0, -1):
            U = self.U_tensors(i)
            perm = [U.dim() - 1] + list(range(U.dim() - 1))
            self.register_buffer(f"U_permuted_{i}", U.permute(perm).reshape(U.shape[-1], -1))
        for nu in range(1, correlation + 1):
            self.register_buffer(f"_mono_{nu}",
                                 torch.tensor(monomial_map(self.k, nu), dtype=dtype),
                                 persistent=False)

    def U_tensors(self, nu: int) -> torch.Tensor:
        return dict(self.named_buffers())[f"U_matrix_{nu}"]

    def U_permuted(self, nu: int) -> torch.Tensor:
        return dict(self.named_buffers())[f"U_permuted_{nu}"]

    def weight_of(self, nu: int) -> torch.Tensor:
        if nu == self.correlation:
            return self.weights_max
        return self.weights[self.correlation - nu - 1]

    def coefficients(self, degree: int) -> torch.Tensor:
        """[E, C, d_out, monomials up to ``degree``] (zeros above this contraction's order)."""
        E, C = self.num_elements, self.num_features
        parts = []
        for nu in range(1, degree + 1):
            n_mono = len(monomials(self.k, nu))
            if nu > self.correlation:
                parts.append(self.weights_max.new_zeros(E, C, self.d_out, n_mono))
                continue
            w = self.weight_of(nu)
            t = w.transpose(1, 2).reshape(E * C, -1) @ self.U_permuted(nu)
            t = t.view(E * C * self.d_out, self.k ** nu) @ getattr(self, f"_mono_{nu}")
            parts.append(t.view(E, C, self.d_out, n_mono))
        return torch.cat(parts, dim=-1)


class SymmetricContraction(torch.nn.Module):
    """Reference ``SymmetricContraction`` (``SymmetricContraction.py:264-336``)."""

    def __init__(self, irreps_in, irreps_out, correlation: Union[int, Dict[str, int]],
                 irrep_normalization: str = "component", path_normalization: str = "element",
                 internal_weights: Optional[bool] = None, shared_weights: Optional[bool] = None,
                 num_elements: Optional[int] = None, dtype: Optional[torch.dtype] = None) -> None:
        super().__init__()
        self.num_elements = num_elements
        self.dtype = dtype if dtype is not None else torch.get_default_dtype()
        if irrep_normalization is None:
            irrep_normalization = "component"
        if path_normalization is None:
            path_normalization = "element"
        assert irrep_normalization in ["component", "norm", "none"]
        assert path_normalization in ["element", "path", "none"]
        self.irreps_in = Irreps(irreps_in)
        self.irreps_out = Irreps(irreps_out)
        if not isinstance(correlation, tuple):
            corr = correlation
            correlation = {}
            for irrep_out in self.irreps_out:
                correlation[irrep_out] = corr
        assert shared_weights or not internal_weights
        if internal_weights is None:
            internal_weights = True
        self.internal_weights = internal_weights
        self.shared_weights = shared_weights
        self.contractions = torch.nn.ModuleList()
        for irrep_out in self.irreps_out:
            self.contractions.append(Contraction(
                irreps_in=self.irreps_in, irrep_out=Irreps(str(irrep_out.ir)),
                correlation=correlation[irrep_out], internal_weights=self.internal_weights,
                num_elements=num_elements, weights=self.shared_weights, dtype=self.dtype))
        self.num_features = self.contractions[0].num_features
        self.k = self.contractions[0].k
        self.degree = max(c.correlation for c in self.contractions)
        # Output layout: contraction i occupies C * d_out columns, channel-major.
        cols, steps, off = [], [], 0
        for c in self.contractions:
            for o in range(c.d_out):
                cols.append(off + o)
                steps.append(c.d_out)
            off += self.num_features * c.d_out
        self.out_dim = off
        self._out_col, self._out_step = cols, steps
        self.nout = len(cols)
        self.dt = next((d for d in _KERNEL_DT if d >= self.nout), None)
        self.fused_ok = self.k in _KERNEL_K and self.degree <= 3 and self.dt is not None

    def coefficients(self) -> torch.Tensor:
        """[E, C, M, nout] monomial coefficients of all output irreps (differentiable)."""
        coef = torch.cat([c.coefficients(self.degree) for c in self.contractions], dim=2)
        return coef.permute(0, 1, 3, 2)

    def forward(self, x: torch.Tensor, y: torch.Tensor) -> torch.Tensor:
        if not x.is_cuda:
            raise RuntimeError("Tensor 'x' is not on the GPU.")
        if not self.fused_ok:
            raise NotImplementedError(
                f"SymmetricContraction: coupling dimension {self.k}, correlation {self.degree} "
                f"and {self.nout} output components are outside the fused kernels' range "
                f"(coupling dimension 4 or 9, correlation <= 3, at most 16 output components)")
        elem = torch.argmax(y, dim=1)
        coef = self.coefficients()
        from . import _ops

        _ops.ensure_registered()
        if self.dt > self.nout:
            coef = torch.nn.functional.pad(coef, (0, self.dt - self.nout))
        perm = torch.argsort(elem, stable=True)
        counts = torch.bincount(elem, minlength=self.num_elements)
        eoff = torch.cat([counts.new_zeros(1), torch.cumsum(counts, 0)])
        return _FusedSC.apply(x, coef.contiguous(), perm, eoff, elem, self)


def _monomial_features(sc: SymmetricContraction, x: torch.Tensor) -> torch.Tensor:
    """phi [N, C, M] in the kernels' monomial order."""
    feats = []
    for d in range(1, sc.degree + 1):
        idx = torch.tensor(monomials(sc.k, d), device=x.device)
        f = x[..., idx[:, 0]]
        for j in range(1, d):
            f = f * x[..., idx[:, j]]
        feats.append(f)
    return torch.cat(feats, dim=-1)


def _torch_contraction(sc: SymmetricContraction, x, coef, elem) -> torch.Tensor:
    """Differentiable torch evaluation of the same polynomial.  Used only to record the
    double backward (on the device, inside ``_FusedSC.backward``); the forward and first
    backward always run the fused kernels."""
    phi = _monomial_features(sc, x)                                   # [N, C, M]
    nout = sc.nout
    vals = torch.einsum("ncm,ncmo->nco", phi, coef[elem][..., :nout])  # [N, C, nout]
    cols = torch.tensor(sc._out_col, device=x.device)
    steps = torch.tensor(sc._out_step, device=x.device)
    c = torch.arange(sc.num_features, device=x.device)
    index = cols[None, :] + c[:, None] * steps[None, :]               # [C, nout]
    out = vals.new_zeros(x.shape[0], sc.out_dim)
    return out.index_put((torch.arange(x.shape[0], device=x.device)[:, None, None],
                          index[None].expand(x.shape[0], -1, -1)), vals)


class _FusedSC(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, coef, perm, eoff, elem, sc):
        ctx.sc = sc
        ctx.save_for_backward(x, coef, perm, eoff, elem)
        return torch.ops.oeqb200.sc_forward(x, perm, eoff, coef, sc._out_col, sc._out_step,
                                            sc.out_dim, sc.degree)

    @staticmethod
    def backward(ctx, gout):
        x, coef, perm, eoff, elem = ctx.saved_tensors
        sc = ctx.sc
        if torch.is_grad_enabled():
            # The backward is being recorded (double backward): differentiate the torch form.
            out = _torch_contraction(sc, x, coef, elem)
            gx, gc = torch.autograd.grad(out, (x, coef), gout, create_graph=True, allow_unused=True)
            return gx, gc, None, None, None, None
        gx, gc = torch.ops.oeqb200.sc_backward(x, perm, eoff, coef, gout.contiguous(),
                                               sc._out_col, sc._out_step, sc.degree)
        return gx, gc, None, None, None, None


__all__ = ["SymmetricContraction", "Contraction"]
