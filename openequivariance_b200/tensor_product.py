"""``TensorProduct``: drop-in for ``oeq.TensorProduct`` (reference ``_torch/TensorProduct.py``).

Same constructor (``problem, torch_op=True, use_opaque=False``), same ``forward(x, y, W)``,
same ``reorder_weights_from_e3nn / reorder_weights_to_e3nn``, ``.to(dtype)`` regeneration
and pickling of ``input_args``.  The module holds a binary problem descriptor (in place of
the reference's generated CUDA source) and calls ``torch.ops.libtorch_tp_jit.*``, whose
implementation is the sm_100a library behind ``include/oeqb200.h``.
"""

from __future__ import annotations

import numpy as np
import torch

from . import _ops
from .irreps import TPProblem
from .plan import analyze_problem, descriptor_hash, pack_descriptor, reorder_weights
from .utils import oeq_to_torch_dtype, torch_to_oeq_dtype


def _descriptor_tensor(desc: bytes) -> torch.Tensor:
    t = torch.tensor(np.frombuffer(desc, dtype=np.uint8), device="cpu")
    t.requires_grad = False
    return t


class TensorProduct(torch.nn.Module):
    r"""Computes :math:`W (x \otimes_{\textrm{CG}} y)` like ``e3nn.o3.TensorProduct``.

    :param problem: the tensor product specification (:class:`TPProblem`).
    :param torch_op: kept for API compatibility; the operator path is always used.
    :param use_opaque: deprecated, ignored (as in the reference).
    """

    def __init__(self, problem: TPProblem, torch_op: bool = True, use_opaque: bool = False):
        torch.nn.Module.__init__(self)
        self.input_args = {"problem": problem, "torch_op": torch_op, "use_opaque": use_opaque}
        self._init_class()

    def _init_class(self):
        problem = self.input_args["problem"]
        analyze_problem(problem)
        self.config = problem.clone()
        self.torch_op = self.input_args["torch_op"]
        self.L1, self.L2, self.L3 = (self.config.irreps_in1, self.config.irreps_in2,
                                     self.config.irreps_out)
        self.irrep_dtype, self.weight_dtype = self.config.irrep_dtype, self.config.weight_dtype
        desc = pack_descriptor(self.config)
        self.kernel = _descriptor_tensor(desc)
        self.hash = descriptor_hash(desc)
        self.L3_dim = self.config.irreps_out.dim
        self.weight_numel = self.config.weight_numel
        self.kernel_prop = {
            "L1_dim": self.L1.dim, "L2_dim": self.L2.dim, "L3_dim": self.L3.dim,
            "weight_numel": self.weight_numel, "shared_weights": int(self.config.shared_weights),
        }
        _ops.ensure_registered()

    # -- module plumbing (reference _torch/TensorProduct.py:55-100) ---------------------
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
        """e3nn weight order -> the order ``forward`` expects (same type returned)."""
        return reorder_weights(self.config, weights, "forward", has_batch_dim)

    def reorder_weights_to_e3nn(self, weights, has_batch_dim: bool = True):
        """Inverse of :meth:`reorder_weights_from_e3nn`."""
        return reorder_weights(self.config, weights, "backward", has_batch_dim)

    @staticmethod
    def name():
        return "LoopUnrollTP"

    def forward(self, x: torch.Tensor, y: torch.Tensor, W: torch.Tensor) -> torch.Tensor:
        r"""``x [B, irreps_in1.dim]``, ``y [B, irreps_in2.dim]``, ``W [B, weight_numel]``
        (or ``[weight_numel]`` with shared weights) -> ``[B, irreps_out.dim]``."""
        return torch.ops.libtorch_tp_jit.jit_tp_forward(self.kernel, self.hash, x, y, W,
                                                       self.L3_dim)

    # -- numpy conveniences used by the reference's harness (TensorProduct.py:138-181) --
    def forward_cpu(self, L1_in, L2_in, L3_out, weights) -> None:
        w = self.reorder_weights_from_e3nn(weights, not self.config.shared_weights)
        out = self.forward(torch.tensor(L1_in, device="cuda"), torch.tensor(L2_in, device="cuda"),
                           torch.tensor(w, device="cuda"))
        L3_out[:] = out.cpu().numpy()

    def backward_cpu(self, L1_in, L1_grad, L2_in, L2_grad, L3_grad, weights, weights_grad) -> None:
        w = self.reorder_weights_from_e3nn(weights, not self.config.shared_weights)
        x = torch.tensor(L1_in, device="cuda", requires_grad=True)
        y = torch.tensor(L2_in, device="cuda", requires_grad=True)
        wt = torch.tensor(w, device="cuda", requires_grad=True)
        out = self.forward(x, y, wt)
        out.backward(gradient=torch.tensor(L3_grad, device="cuda"))
        L1_grad[:] = x.grad.cpu().numpy()
        L2_grad[:] = y.grad.cpu().numpy()
        weights_grad[:] = self.reorder_weights_to_e3nn(wt.grad.cpu().numpy(),
                                                       not self.config.shared_weights)
