"""``TensorProductConv``: drop-in for ``oeq.TensorProductConv``
(reference ``_torch/TensorProductConv.py:33-659``).

Computes ``z_i = sum_{(i, j, e)} W_e (x_j (x)_CG y_e)`` for edges ``e`` with receiver
``rows[e] = i`` and sender ``cols[e] = j``.  Two summation modes, as in the reference:

* atomic (``deterministic=False``): any edge order, scatter with atomics;
* deterministic (``deterministic=True``): ``rows`` sorted receiver-major and a
  ``sender_perm`` giving the sender-sorted edge order; every output row is reduced by one
  warp in a fixed order, so results are bitwise reproducible.  ``kahan=True`` adds
  compensated summation (float32 only).
"""

from __future__ import annotations

from typing import Optional

import numpy as np
import torch

from . import _ops
from .irreps import TPProblem
from .plan import analyze_problem, descriptor_hash, pack_descriptor, reorder_weights
from .tensor_product import TensorProduct, _descriptor_tensor
from .utils import oeq_to_torch_dtype, torch_to_oeq_dtype


class TensorProductConv(torch.nn.Module):
    r"""Fused CG tensor product + graph convolution.

    :param problem: tensor product specification.
    :param deterministic: ``False`` = atomic scatter; ``True`` = sorted, fixup-free
           segmented reduction (needs ``sender_perm``).
    :param kahan: compensated summation (requires ``deterministic=True`` and float32).
    :param torch_op: kept for API compatibility.
    :param use_opaque: deprecated, ignored.
    """

    def __init__(self, problem: TPProblem, *, deterministic: bool = False, kahan: bool = False,
                 torch_op: bool = True, use_opaque: bool = False):
        torch.nn.Module.__init__(self)
        self.input_args = {"problem": problem, "deterministic": deterministic, "kahan": kahan,
                           "torch_op": torch_op, "use_opaque": use_opaque}
        self._init_class()

    def _init_class(self):
        problem = self.input_args["problem"]
        self.deterministic = self.input_args["deterministic"]
        self.kahan = self.input_args["kahan"]
        self.torch_op = self.input_args["torch_op"]
        if self.kahan:
            assert self.deterministic
        analyze_problem(problem)
        if problem.shared_weights:
            assert not self.deterministic, (
                "Deterministic convolution does not support shared weights"
            )
        if self.kahan:
            assert problem.irrep_dtype == problem.weight_dtype == np.float32
        self.config = problem.clone()
        self.L1, self.L2, self.L3 = (self.config.irreps_in1, self.config.irreps_in2,
                                     self.config.irreps_out)
        self.idx_dtype = np.int64
        desc = pack_descriptor(self.config, deterministic=self.deterministic, kahan=self.kahan)
        self.kernel = _descriptor_tensor(desc)
        self.hash = descriptor_hash(desc)
        self.L3_dim = self.config.irreps_out.dim
        self.weight_numel = self.config.weight_numel
        _ops.ensure_registered()
        # The kernels need no workspace; a 1-byte buffer keeps the operator signature.
        self.allocate_workspace(1)
        self.dummy_transpose_perm = torch.zeros(1, dtype=torch.int64, device="cuda")

    def allocate_workspace(self, size_bytes: int) -> None:
        self.workspace_size = size_bytes
        self.workspace_buffer = torch.zeros(size_bytes, dtype=torch.uint8, device="cuda")
        self.workspace_ptr = self.workspace_buffer.data_ptr()

    def to(self, *args, **kwargs):
        device, dtype, non_blocking, convert_to_format = torch._C._nn._parse_to(*args, **kwargs)
        if dtype is not None:
            updated = self.input_args["problem"].clone()
            updated.irrep_dtype = torch_to_oeq_dtype(dtype)
            updated.weight_dtype = torch_to_oeq_dtype(dtype)
            self.input_args["problem"] = updated
            self._init_class()
        torch.nn.Module.to(self, *args, **kwargs)
        return self

    def _apply(self, fn, recurse=True):
        if getattr(self, "_applying", False):
            return super()._apply(fn, recurse)
        current = oeq_to_torch_dtype(np.dtype(self.input_args["problem"].irrep_dtype).type)
        result = fn(torch.tensor(0.0, dtype=current))
        if result.dtype != current and result.dtype in (torch.float32, torch.float64):
            self._applying = True
            try:
                self.to(result.dtype)
            finally:
                self._applying = False
        return super()._apply(fn, recurse)

    def __getstate__(self):
        return self.input_args

    def __setstate__(self, state):
        torch.nn.Module.__init__(self)
        self.input_args = state
        self._init_class()

    def reorder_weights_from_e3nn(self, weights, has_batch_dim: bool = True):
        return reorder_weights(self.config, weights, "forward", has_batch_dim)

    def reorder_weights_to_e3nn(self, weights, has_batch_dim: bool = True):
        return reorder_weights(self.config, weights, "backward", has_batch_dim)

    @staticmethod
    def name():
        return "LoopUnrollConv"

    def forward(self, X: torch.Tensor, Y: torch.Tensor, W: torch.Tensor, rows: torch.Tensor,
                cols: torch.Tensor, sender_perm: Optional[torch.Tensor] = None) -> torch.Tensor:
        r"""``X [|V|, in1.dim]``, ``Y [|E|, in2.dim]``, ``W [|E|, weight_numel]`` (or
        ``[weight_numel]`` shared), int64 ``rows``/``cols`` ``[|E|]``; ``sender_perm``
        ``[|E|]`` is required in deterministic mode.  Returns ``[|V|, out.dim]``."""
        if sender_perm is None:
            sender_perm = self.dummy_transpose_perm
        return torch.ops.libtorch_tp_jit.jit_conv_forward(
            self.kernel, self.hash, X, Y, W, self.L3_dim, rows, cols, self.workspace_buffer,
            sender_perm)


class TensorProductConvKahan(TensorProductConv):
    def __init__(self, config, *, torch_op=True):
        super().__init__(config, torch_op=torch_op, deterministic=True, kahan=True)

    @staticmethod
    def name():
        return "LoopUnrollConvKahan"


class TensorProductConvDeterministic(TensorProductConv):
    def __init__(self, config, *, torch_op=True):
        super().__init__(config, torch_op=torch_op, deterministic=True)

    @staticmethod
    def name():
        return "LoopUnrollConvDeterministic"


class TensorProductConvAtomic(TensorProductConv):
    def __init__(self, config, *, torch_op=True):
        super().__init__(config, torch_op=torch_op, deterministic=False)

    @staticmethod
    def name():
        return "LoopUnrollConvAtomic"


def scatter_add_rows(messages: torch.Tensor, rows: torch.Tensor, target_dim: int) -> torch.Tensor:
    out = messages.new_zeros((target_dim, messages.size(1)))
    return out.index_add_(0, rows, messages)


class TensorProductConvScatterSum(torch.nn.Module):
    """Unfused baseline: batch tensor product on gathered senders, then ``index_add``."""

    def __init__(self, config, *, torch_op=True):
        super().__init__()
        self.config = config.clone()
        self.reference_tp = TensorProduct(config, torch_op=torch_op)
        self.reorder_weights_from_e3nn = self.reference_tp.reorder_weights_from_e3nn
        self.reorder_weights_to_e3nn = self.reference_tp.reorder_weights_to_e3nn

    def forward(self, L1_in, L2_in, weights, rows, cols, sender_perm=None):
        messages = self.reference_tp(L1_in[cols], L2_in, weights)
        return scatter_add_rows(messages, rows, L1_in.size(0))

    @staticmethod
    def name():
        return "LoopUnrollConvScatterSum"
