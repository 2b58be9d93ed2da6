"""Small helpers of the public API: dtype conversion and irrep layout transposes.

``transpose_irreps`` mirrors the reference's ``_torch/utils.py:81-147`` and
``transpose_irrep_layout`` its numpy twin (``core/utils.py:216-264``): each irrep block
of the trailing feature axis is viewed as ``[mul, dim]`` (``mul_ir``) or ``[dim, mul]``
(``ir_mul``) and transposed.
"""

from __future__ import annotations

import numpy as np

from .irreps import Irreps

__all__ = ["torch_to_oeq_dtype", "oeq_to_torch_dtype", "transpose_irreps",
           "transpose_irrep_layout"]


def torch_to_oeq_dtype(torch_dtype):
    """``torch.float32``/``torch.float64`` -> ``np.float32``/``np.float64``."""
    import torch

    if torch_dtype == torch.float32:
        return np.float32
    if torch_dtype == torch.float64:
        return np.float64
    raise ValueError("Unsupported torch dtype!")


def oeq_to_torch_dtype(oeq_dtype):
    import torch

    if oeq_dtype == np.float32:
        return torch.float32
    if oeq_dtype == np.float64:
        return torch.float64
    raise ValueError("Unsupported numpy dtype!")


def _check_layouts(src_layout: str, dst_layout: str) -> None:
    if src_layout not in ("mul_ir", "ir_mul"):
        raise ValueError(f"Unsupported src_layout: {src_layout}")
    if dst_layout not in ("mul_ir", "ir_mul"):
        raise ValueError(f"Unsupported dst_layout: {dst_layout}")


def transpose_irreps(array, irreps: Irreps, src_layout: str, dst_layout: str):
    """Transposes a ``[..., irreps.dim]`` torch tensor between ``mul_ir`` and ``ir_mul``.

    Differentiable (plain torch ops).  Returns a new tensor, a copy when the layouts match.
    """
    import torch

    _check_layouts(src_layout, dst_layout)
    if not isinstance(array, torch.Tensor):
        raise TypeError(f"Expected torch.Tensor, got {type(array)}")
    irreps = Irreps(irreps)
    if src_layout == dst_layout:
        return array.clone()
    lead = array.shape[:-1]
    pieces = []
    for mul_ir, sl in zip(irreps, irreps.slices()):
        block = array[..., sl]
        if src_layout == "mul_ir":
            block = block.reshape(*lead, mul_ir.mul, mul_ir.ir.dim)
        else:
            block = block.reshape(*lead, mul_ir.ir.dim, mul_ir.mul)
        pieces.append(block.transpose(-1, -2).reshape(*lead, mul_ir.dim))
    if not pieces:
        return array.clone()
    return torch.cat(pieces, dim=-1)


def transpose_irrep_layout(array: np.ndarray, irreps: Irreps, src_layout: str,
                           dst_layout: str) -> np.ndarray:
    """numpy version of :func:`transpose_irreps`."""
    _check_layouts(src_layout, dst_layout)
    x = np.asarray(array)
    irreps = Irreps(irreps)
    if src_layout == dst_layout:
        return x.copy()
    out = np.empty_like(x)
    lead = x.shape[:-1]
    for mul_ir, sl in zip(irreps, irreps.slices()):
        block = x[..., sl]
        if src_layout == "mul_ir":
            block = block.reshape(*lead, mul_ir.mul, mul_ir.ir.dim)
        else:
            block = block.reshape(*lead, mul_ir.ir.dim, mul_ir.mul)
        out[..., sl] = np.swapaxes(block, -1, -2).reshape(*lead, mul_ir.dim)
    return out
