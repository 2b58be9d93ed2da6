"""Irreducible-representation bookkeeping and the tensor-product problem spec.

This module is the drop-in contract of the package: ``Irrep``, ``Irreps`` and
``TPProblem`` behave like the reference's ``openequivariance.core.e3nn_lite``
classes (``core/e3nn_lite.py:57-351`` for the irreps, ``core/e3nn_lite.py:363-654``
for ``TPProblem``), which in turn follow e3nn 0.5's ``o3.Irreps`` and
``o3.TensorProduct`` argument conventions.  The normalisation rule that turns
user instructions into per-path weights (``core/e3nn_lite.py:502-578``) is the
one piece of arithmetic here; it is restated in ``TPProblem._normalise``.

Nothing in this module touches torch or the GPU.
"""

from __future__ import annotations

import collections
import copy
import itertools
from math import prod, sqrt
from typing import Any, List, NamedTuple, Optional, Tuple

import numpy as np

__all__ = ["Irrep", "Irreps", "_MulIr", "Instruction", "TPProblem"]

_PARITY_CHAR = {1: "e", -1: "o"}


class Irrep(tuple):
    """An O(3) irrep ``(l, p)``; parses strings such as ``"2e"``, ``"1o"`` or ``"3y"``."""

    def __new__(cls, l, p=None):
        if p is None:
            if isinstance(l, Irrep):
                return l
            if isinstance(l, str):
                text = l.strip()
                try:
                    deg = int(text[:-1])
                    if deg < 0:
                        raise ValueError
                    par = {"e": 1, "o": -1, "y": (-1) ** deg}[text[-1]]
                except Exception:
                    raise ValueError(f'unable to convert string "{text}" into an Irrep')
                l, p = deg, par
            elif isinstance(l, tuple):
                l, p = l
        if not isinstance(l, (int, np.integer)) or l < 0:
            raise ValueError(f"l must be positive integer, got {l}")
        if p not in (-1, 1):
            raise ValueError(f"parity must be on of (-1, 1), got {p}")
        return super().__new__(cls, (int(l), int(p)))

    @property
    def l(self) -> int:  # noqa: E743
        return self[0]

    @property
    def p(self) -> int:
        return self[1]

    @property
    def dim(self) -> int:
        return 2 * self[0] + 1

    def is_scalar(self) -> bool:
        return self[0] == 0 and self[1] == 1

    def __repr__(self) -> str:
        return f"{self[0]}{_PARITY_CHAR[self[1]]}"

    @classmethod
    def iterator(cls, lmax=None):
        for deg in itertools.count():
            yield Irrep(deg, (-1) ** deg)
            yield Irrep(deg, -((-1) ** deg))
            if deg == lmax:
                break

    def __mul__(self, other):
        """All irreps in the decomposition of ``self (x) other``."""
        other = Irrep(other)
        par = self.p * other.p
        for deg in range(abs(self.l - other.l), self.l + other.l + 1):
            yield Irrep(deg, par)

    def __rmul__(self, other):
        if not isinstance(other, int):
            raise TypeError("can only multiply an Irrep by an int")
        return Irreps([(other, self)])

    def __add__(self, other):
        return Irreps(self) + Irreps(other)

    def count(self, _value):
        raise NotImplementedError

    def index(self, _value):
        raise NotImplementedError

    def __contains__(self, _object):
        raise NotImplementedError

    def __len__(self):
        raise NotImplementedError


class _MulIr(tuple):
    """``mul`` copies of one irrep."""

    def __new__(cls, mul, ir=None):
        if ir is None:
            mul, ir = mul
        if not isinstance(mul, (int, np.integer)):
            raise TypeError("multiplicity must be an int")
        if not isinstance(ir, Irrep):
            raise TypeError("ir must be an Irrep")
        return super().__new__(cls, (int(mul), ir))

    @property
    def mul(self) -> int:
        return self[0]

    @property
    def ir(self) -> Irrep:
        return self[1]

    @property
    def dim(self) -> int:
        return self[0] * self[1].dim

    def __repr__(self) -> str:
        return f"{self[0]}x{self[1]!r}"

    def __getitem__(self, item):
        return super().__getitem__(item)

    def count(self, _value):
        raise NotImplementedError

    def index(self, _value):
        raise NotImplementedError


def _as_mul_ir(entry) -> _MulIr:
    if isinstance(entry, _MulIr):
        return entry
    if isinstance(entry, str):
        return _MulIr(1, Irrep(entry))
    if isinstance(entry, Irrep):
        return _MulIr(1, entry)
    try:
        mul, ir = entry
    except Exception:
        raise ValueError(f'Unable to interpret "{entry}" as an irrep.')
    if not isinstance(mul, (int, np.integer)) or mul < 0:
        raise ValueError(f'Unable to interpret "{entry}" as an irrep.')
    return _MulIr(int(mul), Irrep(ir))


class Irreps(tuple):
    """A direct sum of irreps with multiplicities, e.g. ``Irreps("128x0e+128x1o")``."""

    def __new__(cls, irreps=None):
        if isinstance(irreps, Irreps):
            return super().__new__(cls, irreps)
        items: List[_MulIr] = []
        if irreps is None:
            pass
        elif isinstance(irreps, Irrep):
            items.append(_MulIr(1, irreps))
        elif isinstance(irreps, str):
            text = irreps.strip()
            if text:
                try:
                    for term in text.split("+"):
                        term = term.strip()
                        if "x" in term:
                            mul_s, ir_s = term.split("x")
                            mul = int(mul_s)
                            if mul < 0:
                                raise ValueError
                            items.append(_MulIr(mul, Irrep(ir_s)))
                        else:
                            items.append(_MulIr(1, Irrep(term)))
                except Exception:
                    raise ValueError(f'Unable to convert string "{irreps}" into an Irreps')
        else:
            items = [_as_mul_ir(entry) for entry in irreps]
        return super().__new__(cls, items)

    @staticmethod
    def spherical_harmonics(lmax: int, p: int = -1) -> "Irreps":
        return Irreps([(1, (deg, p**deg)) for deg in range(lmax + 1)])

    def slices(self):
        out, start = [], 0
        for mul_ir in self:
            out.append(slice(start, start + mul_ir.dim))
            start += mul_ir.dim
        return out

    def __getitem__(self, i):
        item = super().__getitem__(i)
        if isinstance(i, slice):
            return Irreps(item)
        return item

    def __contains__(self, ir) -> bool:
        ir = Irrep(ir)
        return any(entry.ir == ir for entry in self)

    def count(self, ir) -> int:
        ir = Irrep(ir)
        return sum(entry.mul for entry in self if entry.ir == ir)

    def index(self, _object):
        raise NotImplementedError

    def __add__(self, other) -> "Irreps":
        return Irreps(tuple.__add__(self, Irreps(other)))

    def __mul__(self, other) -> "Irreps":
        if isinstance(other, Irreps):
            raise NotImplementedError("Use a tensor product for Irreps x Irreps")
        return Irreps(tuple.__mul__(self, other))

    def __rmul__(self, other) -> "Irreps":
        return Irreps(tuple.__rmul__(self, other))

    def simplify(self) -> "Irreps":
        merged: List[Tuple[int, Irrep]] = []
        for mul, ir in self:
            if merged and merged[-1][1] == ir:
                merged[-1] = (merged[-1][0] + mul, ir)
            elif mul > 0:
                merged.append((mul, ir))
        return Irreps(merged)

    def remove_zero_multiplicities(self) -> "Irreps":
        return Irreps([(mul, ir) for mul, ir in self if mul > 0])

    def sort(self):
        """Sort by irrep; returns ``(irreps, p, inv)`` with ``p`` the forward permutation."""
        SortResult = collections.namedtuple("sort", ["irreps", "p", "inv"])
        keyed = sorted((ir, i, mul) for i, (mul, ir) in enumerate(self))
        inv = tuple(i for _, i, _ in keyed)
        p = tuple(inv.index(i) for i in range(len(inv)))
        return SortResult(Irreps([(mul, ir) for ir, _, mul in keyed]), p, inv)

    def regroup(self) -> "Irreps":
        return self.sort().irreps.simplify()

    @property
    def dim(self) -> int:
        return sum(entry.dim for entry in self)

    @property
    def num_irreps(self) -> int:
        return sum(entry.mul for entry in self)

    @property
    def ls(self) -> List[int]:
        return [ir.l for mul, ir in self for _ in range(mul)]

    @property
    def lmax(self) -> int:
        if len(self) == 0:
            raise ValueError("Cannot get lmax of empty Irreps")
        return max(self.ls)

    def __repr__(self) -> str:
        return "+".join(repr(entry) for entry in self)


class Instruction(NamedTuple):
    i_in1: int
    i_in2: int
    i_out: int
    connection_mode: str
    has_weight: bool
    path_weight: float
    path_shape: tuple


_MODES = ("uvw", "uvu", "uvv", "uuw", "uuu", "uvuv", "uvu<v", "u<vw")


class TPProblem:
    """Specification of a Clebsch-Gordan tensor product (e3nn ``o3.TensorProduct`` args).

    Mirrors ``TPProblem`` of the reference (``core/e3nn_lite.py:363-654``): same
    constructor arguments, same ``instructions`` (with normalised ``path_weight``),
    ``weight_numel`` and ``weight_range_and_shape_for_instruction``.  The kernels
    of this package support the subset that the reference supports (see
    ``openequivariance_b200.plan.analyze_problem``).
    """

    def __init__(
        self,
        irreps_in1,
        irreps_in2,
        irreps_out,
        instructions: List[tuple],
        in1_var: Optional[List[float]] = None,
        in2_var: Optional[List[float]] = None,
        out_var: Optional[List[float]] = None,
        irrep_normalization: str = "component",
        path_normalization: str = "element",
        internal_weights: Optional[bool] = False,
        shared_weights: Optional[bool] = None,
        label: Optional[str] = None,
        irrep_dtype=np.float32,
        weight_dtype=np.float32,
        layout: str = "mul_ir",
    ) -> None:
        assert irrep_normalization in ("component", "norm", "none")
        assert path_normalization in ("element", "path", "none")
        assert layout in ("mul_ir", "ir_mul")
        assert issubclass(irrep_dtype, np.generic)
        assert issubclass(weight_dtype, np.generic)

        self.irreps_in1 = Irreps(irreps_in1)
        self.irreps_in2 = Irreps(irreps_in2)
        self.irreps_out = Irreps(irreps_out)
        self.instructions_raw = instructions
        self.in1_var = in1_var
        self.in2_var = in2_var
        self.out_var = out_var
        self.irrep_normalization = irrep_normalization
        self.path_normalization = path_normalization
        self.label = label if label is not None else ""
        self.layout = layout

        parsed = []
        for raw in instructions:
            raw = tuple(raw)
            if len(raw) == 5:
                raw = raw + (1.0,)
            i1, i2, io, mode, has_w, pw = raw
            parsed.append(
                Instruction(i1, i2, io, mode, has_w, pw, self._path_shape(i1, i2, io, mode))
            )

        v1 = self._variances(in1_var, self.irreps_in1, "ir1_var", "irreps_in1")
        v2 = self._variances(in2_var, self.irreps_in2, "ir2_var", "irreps_in2")
        vo = self._variances(out_var, self.irreps_out, "out_var", "irreps_out")
        coeffs = self._normalise(parsed, v1, v2, vo)
        self.instructions = [
            Instruction(ins.i_in1, ins.i_in2, ins.i_out, ins.connection_mode,
                        ins.has_weight, c, ins.path_shape)
            for ins, c in zip(parsed, coeffs)
        ]

        self._in1_dim = self.irreps_in1.dim
        self._in2_dim = self.irreps_in2.dim
        if shared_weights is False and internal_weights is None:
            internal_weights = False
        if shared_weights is None:
            shared_weights = True
        assert shared_weights or not internal_weights
        self.internal_weights = internal_weights
        self.shared_weights = shared_weights
        self.weight_numel = sum(
            prod(ins.path_shape) for ins in self.instructions if ins.has_weight
        )
        self.output_mask = None
        self.irrep_dtype = irrep_dtype
        self.weight_dtype = weight_dtype

    # -- construction helpers -------------------------------------------------
    def _path_shape(self, i1, i2, io, mode):
        m1 = self.irreps_in1[i1].mul
        m2 = self.irreps_in2[i2].mul
        mo = self.irreps_out[io].mul
        shapes = {
            "uvw": (m1, m2, mo),
            "uvu": (m1, m2),
            "uvv": (m1, m2),
            "uuw": (m1, mo),
            "uuu": (m1,),
            "uvuv": (m1, m2),
            "uvu<v": (m1 * (m2 - 1) // 2,),
            "u<vw": (m1 * (m2 - 1) // 2, mo),
        }
        if mode not in shapes:
            raise KeyError(mode)
        return shapes[mode]

    @staticmethod
    def _variances(given, irreps, name, irreps_name):
        if given is None:
            return [1.0] * len(irreps)
        out = [float(v) for v in given]
        assert len(out) == len(irreps), f"Len of {name} must be equal to len({irreps_name})"
        return out

    def _fan_in(self, ins) -> int:
        """Number of summed elements feeding one output component (e3nn path counting)."""
        m1 = self.irreps_in1[ins.i_in1].mul
        m2 = self.irreps_in2[ins.i_in2].mul
        return {
            "uvw": m1 * m2,
            "uvu": m2,
            "uvv": m1,
            "uuw": m1,
            "uuu": 1,
            "uvuv": 1,
            "uvu<v": 1,
            "u<vw": m1 * (m2 - 1) // 2,
        }[ins.connection_mode]

    def _normalise(self, parsed, v1, v2, vo) -> List[float]:
        """Per-path weights ``sqrt(alpha)``; restates ``core/e3nn_lite.py:531-565``."""
        coeffs = []
        for ins in parsed:
            a = self.irreps_in1[ins.i_in1]
            b = self.irreps_in2[ins.i_in2]
            o = self.irreps_out[ins.i_out]
            assert a.ir.p * b.ir.p == o.ir.p
            assert abs(a.ir.l - b.ir.l) <= o.ir.l <= a.ir.l + b.ir.l
            assert ins.connection_mode in _MODES

            if self.irrep_normalization == "component":
                alpha = o.ir.dim
            elif self.irrep_normalization == "norm":
                alpha = a.ir.dim * b.ir.dim
            else:
                alpha = 1

            if self.path_normalization == "element":
                x = sum(
                    v1[other.i_in1] * v2[other.i_in2] * self._fan_in(other)
                    for other in parsed
                    if other.i_out == ins.i_out
                )
            elif self.path_normalization == "path":
                x = v1[ins.i_in1] * v2[ins.i_in2] * self._fan_in(ins)
                x *= len([other for other in parsed if other.i_out == ins.i_out])
            else:
                x = 1
            if x > 0.0:
                alpha /= x
            alpha *= vo[ins.i_out]
            alpha *= ins.path_weight
            coeffs.append(sqrt(alpha))
        return coeffs

    # -- queries ----------------------------------------------------------------
    def weight_range_and_shape_for_instruction(self, instruction: int) -> Tuple[int, int, tuple]:
        if not self.instructions[instruction].has_weight:
            raise ValueError(f"Instruction {instruction} has no weights.")
        offset = sum(prod(ins.path_shape) for ins in self.instructions[:instruction])
        ins = self.instructions[instruction]
        return offset, offset + prod(ins.path_shape), ins.path_shape

    def clone(self):
        return copy.deepcopy(self)

    def __str__(self) -> str:
        return (
            f"{self.__class__.__name__}"
            f"({self.irreps_in1.simplify()} x {self.irreps_in2.simplify()}) -> "
            f"{self.irreps_out.simplify()}"
        )

    def __repr__(self) -> str:
        lines = [str(self)]
        for field in ("irrep_normalization", "path_normalization", "internal_weights",
                      "shared_weights", "in1_var", "in2_var", "out_var"):
            lines.append(f"{field} = {getattr(self, field)!r}")
        lines.append(f"num weights {self.weight_numel} ")
        for ins in self.instructions:
            lines.append(
                f"| {ins.i_in1:3} | {ins.i_in2:3} | {ins.i_out:3} | {ins.connection_mode:<5} "
                f"| {str(ins.has_weight):<5} | {ins.path_weight:<4.2f} |"
            )
        return "\n".join(lines) + "\n"

    # A problem is plain data; equality/hash are by value so plan caches can key on it.
    def _key(self) -> Any:
        return (
            repr(self.irreps_in1), repr(self.irreps_in2), repr(self.irreps_out),
            tuple(self.instructions), self.shared_weights, self.layout,
            np.dtype(self.irrep_dtype).str, np.dtype(self.weight_dtype).str,
        )
