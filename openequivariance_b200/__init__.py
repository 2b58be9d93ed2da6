"""B200-native (sm_100a) Clebsch-Gordan tensor products with the OpenEquivariance API.

Public names mirror the reference package ``openequivariance`` (its ``__init__.py:106-116``):
``TPProblem``, ``Irreps``, ``TensorProduct``, ``TensorProductConv``, ``transpose_irreps``,
``torch_to_oeq_dtype`` and ``torch_ext_so_path``, plus the MACE ``SymmetricContraction``.
Set ``OEQ_NOTORCH=1`` to import only the torch-free problem specification.
"""

import os

import numpy as np

from .irreps import Instruction, Irrep, Irreps, TPProblem, _MulIr

__version__ = "0.1.0"

if os.environ.get("OEQ_NOTORCH", "0") != "1":
    import torch

    from .symmetric_contraction import SymmetricContraction
    from .tensor_product import TensorProduct
    from .tensor_product_conv import TensorProductConv
    from .utils import torch_to_oeq_dtype, transpose_irreps

    torch.serialization.add_safe_globals(
        [TensorProduct, TensorProductConv, TPProblem, Irrep, Irreps, _MulIr, Instruction,
         np.float32, np.float64]
    )


def set_device_checks(enabled: bool) -> bool:
    """Turns the synchronous device checks on or off; returns the previous setting.

    The kernels never fault on bad graph indices: they skip them and raise a status flag.
    With checks on, every convolution call validates rows / cols / transpose_perm on the
    device before launching (range, receiver order in deterministic mode, permutation and
    sender order of ``transpose_perm``) and every call reads its plan's status flag
    afterwards; a problem raises ``RuntimeError`` naming it.  Each check synchronises the
    stream (checks are skipped during CUDA-graph capture).  ``OEQB_DEVICE_CHECKS=1`` in the
    environment turns them on at load time.
    """
    import torch

    from ._ext import load_torch_ops

    load_torch_ops()
    return bool(torch.ops.oeqb200.set_device_checks(bool(enabled)))


def check_device_status() -> None:
    """Reads and clears the status flag of every plan on the current device and raises
    ``RuntimeError`` if a kernel flagged a bad index or an expired pipeline wait since the
    last check (synchronises the current stream)."""
    import torch

    from ._ext import load_torch_ops

    load_torch_ops()
    torch.ops.oeqb200.check_device_status()


def torch_ext_so_path():
    """Path of the ``.so`` to link when using the operators from the PyTorch C++ API."""
    from ._ext import TORCH_LIB_PATH

    return str(TORCH_LIB_PATH)


class _JaxUnavailable:
    """JAX is outside this package's scope; mirrors the reference's error stub."""

    def TensorProduct(self, *args, **kwargs):
        raise ImportError("openequivariance_b200 has no JAX frontend")

    def TensorProductConv(self, *args, **kwargs):
        raise ImportError("openequivariance_b200 has no JAX frontend")


jax = _JaxUnavailable()

__all__ = [
    "TPProblem",
    "Irreps",
    "TensorProduct",
    "TensorProductConv",
    "SymmetricContraction",
    "torch_to_oeq_dtype",
    "torch_ext_so_path",
    "jax",
    "transpose_irreps",
    "set_device_checks",
    "check_device_status",
]
