"""Problem analysis, weight ordering and the binary problem descriptor.

* ``analyze_problem`` is the support gate of the reference
  (``core/utils.py:81-117``): one connection mode for all instructions, ``uvu`` or
  ``uvw``, every instruction weighted, ``ir_mul`` only for ``uvu``, equal irrep and
  weight dtypes, no internal weights.  The assertion messages are the reference's.
* ``oeq_weight_permutation`` restates the reference's weight reordering
  (``ComputationSchedule.weight_reordering_info``, ``ComputationSchedule.py:653-714``,
  applied by ``_torch/utils.py:8-46``): multiplicities are split into chunks of 32
  and every chunk triple stores its block as ``[v][u]`` (uvu) or ``[v][u][w]`` (uvw).
  Users pass weights in this "oeq" order, so the kernels read it directly.
* ``pack_descriptor`` produces the bytes the C ABI parses (layout documented in
  ``include/oeqb200.h``); ``descriptor_hash`` keys the native plan cache.
"""

from __future__ import annotations

import hashlib
import struct
from math import prod
from typing import Dict, List, Tuple

import numpy as np

from .cg import sparse_cg
from .irreps import TPProblem

__all__ = [
    "analyze_problem",
    "oeq_weight_permutation",
    "reorder_weights",
    "pack_descriptor",
    "descriptor_hash",
    "CHUNK",
]

CHUNK = 32  # multiplicity chunk of the reference's weight layout (its warp size)
MAGIC = 0x4251454F
VERSION = 1


def analyze_problem(problem: TPProblem) -> Dict[str, bool]:
    """Rejects problems the kernels do not support, exactly like the reference."""
    for i, inst in enumerate(problem.instructions):
        assert inst.connection_mode == problem.instructions[0].connection_mode, (
            f"All instructions must have the same connection mode, got "
            f"{inst.connection_mode} and {problem.instructions[0].connection_mode}"
        )
        assert inst.has_weight, (
            f"All instructions must have trainable weights, got {inst.has_weight} at index {i}"
        )
    assert problem.instructions[0].connection_mode in ["uvu", "uvw"], (
        f"Connection mode must be 'uvu' or 'uvw', got {problem.instructions[0].connection_mode}"
    )
    if problem.layout == "ir_mul":
        assert problem.instructions[0].connection_mode == "uvu", (
            "layout='ir_mul' is only supported for pure 'uvu' problems"
        )
    assert problem.irrep_dtype == problem.weight_dtype, (
        f"irrep_dtype and weight_dtype must be the same, got {problem.irrep_dtype} "
        f"and {problem.weight_dtype}"
    )
    assert not problem.internal_weights, (
        f"Openequivariance does not support internal weights, got {problem.internal_weights}"
    )
    assert len(problem.instructions) > 0, "Tensor product has no valid instructions!"
    for ins in problem.instructions:
        for irreps, idx in ((problem.irreps_in1, ins.i_in1), (problem.irreps_in2, ins.i_in2),
                            (problem.irreps_out, ins.i_out)):
            assert irreps[idx].ir.l <= 7, "irreps with l > 7 are not supported"
    assert np.dtype(problem.irrep_dtype) in (np.dtype(np.float32), np.dtype(np.float64)), (
        "irrep_dtype must be float32 or float64"
    )
    return {"is_uvw": problem.instructions[0].connection_mode == "uvw"}


def _chunk(idx: int, mul: int) -> Tuple[int, int]:
    start = (idx // CHUNK) * CHUNK
    return start, min(CHUNK, mul - start)


def _oeq_index_uvu(m1: int, m2: int, u: int, v: int) -> int:
    u0, ul = _chunk(u, m1)
    return u0 * m2 + v * ul + (u - u0)


def _oeq_index_uvw(m1: int, m2: int, m3: int, u: int, v: int, w: int) -> int:
    u0, ul = _chunk(u, m1)
    v0, vl = _chunk(v, m2)
    w0, wl = _chunk(w, m3)
    return (u0 * m2 * m3 + ul * v0 * m3 + ul * vl * w0
            + (v - v0) * ul * wl + (u - u0) * wl + (w - w0))


def oeq_weight_permutation(problem: TPProblem) -> np.ndarray:
    """``perm`` with ``w_oeq = w_e3nn[..., perm]`` (e3nn order is ``[u,v]`` / ``[u,v,w]``)."""
    perm = np.arange(problem.weight_numel, dtype=np.int64)
    offset = 0
    for ins in problem.instructions:
        size = prod(ins.path_shape)
        if not ins.has_weight:
            offset += size
            continue
        if ins.connection_mode == "uvu":
            m1, m2 = ins.path_shape
            for u in range(m1):
                for v in range(m2):
                    perm[offset + _oeq_index_uvu(m1, m2, u, v)] = offset + u * m2 + v
        elif ins.connection_mode == "uvw":
            m1, m2, m3 = ins.path_shape
            u = np.arange(m1)[:, None, None]
            v = np.arange(m2)[None, :, None]
            w = np.arange(m3)[None, None, :]
            u0 = (u // CHUNK) * CHUNK
            ul = np.minimum(CHUNK, m1 - u0)
            v0 = (v // CHUNK) * CHUNK
            vl = np.minimum(CHUNK, m2 - v0)
            w0 = (w // CHUNK) * CHUNK
            wl = np.minimum(CHUNK, m3 - w0)
            oeq = (u0 * m2 * m3 + ul * v0 * m3 + ul * vl * w0
                   + (v - v0) * ul * wl + (u - u0) * wl + (w - w0))
            e3nn = u * m2 * m3 + v * m3 + w
            perm[offset + oeq.ravel()] = offset + np.broadcast_to(e3nn, oeq.shape).ravel()
        offset += size
    return perm


def reorder_weights(problem: TPProblem, weights, direction: str, has_batch_dim: bool = True):
    """e3nn <-> oeq weight order for numpy arrays or torch tensors (same type returned)."""
    assert direction in ("forward", "backward")
    perm = oeq_weight_permutation(problem)
    if direction == "backward":
        inv = np.empty_like(perm)
        inv[perm] = np.arange(perm.size)
        perm = inv
    if isinstance(weights, np.ndarray):
        return np.ascontiguousarray(weights[..., perm])
    import torch

    idx = torch.as_tensor(perm, device=weights.device)
    return torch.index_select(weights, weights.dim() - 1, idx)


def pack_descriptor(problem: TPProblem, deterministic: bool = False, kahan: bool = False) -> bytes:
    """Serialises a (supported) problem for ``oeqb_plan_create``."""
    info = analyze_problem(problem)
    dt = np.dtype(problem.irrep_dtype)
    dtype_code = 1 if dt == np.dtype(np.float32) else 2
    irreps = [problem.irreps_in1, problem.irreps_in2, problem.irreps_out]

    cg_entries: List[Tuple[int, int, int, float]] = []
    cg_index: Dict[Tuple[int, int, int], Tuple[int, int]] = {}
    ins_rows = []
    woff = 0
    for ins in problem.instructions:
        l1 = problem.irreps_in1[ins.i_in1].ir.l
        l2 = problem.irreps_in2[ins.i_in2].ir.l
        l3 = problem.irreps_out[ins.i_out].ir.l
        key = (l1, l2, l3)
        if key not in cg_index:
            nz = sparse_cg(*key)
            cg_index[key] = (len(cg_entries), len(nz))
            cg_entries.extend(nz)
        off, nnz = cg_index[key]
        ins_rows.append((ins.i_in1, ins.i_in2, ins.i_out, woff, off, nnz, float(ins.path_weight)))
        woff += prod(ins.path_shape)

    flags = (1 if deterministic else 0) | (2 if kahan else 0)
    header = [
        MAGIC, VERSION, dtype_code, 1 if problem.layout == "ir_mul" else 0,
        1 if info["is_uvw"] else 0, 1 if problem.shared_weights else 0,
        len(irreps[0]), len(irreps[1]), len(irreps[2]), len(problem.instructions),
        irreps[0].dim, irreps[1].dim, irreps[2].dim, problem.weight_numel,
        len(cg_entries), flags,
    ]
    out = bytearray(struct.pack("<16q", *header))
    for rep in irreps:
        for mul_ir, sl in zip(rep, rep.slices()):
            out += struct.pack("<3q", mul_ir.mul, mul_ir.ir.l, sl.start)
    for row in ins_rows:
        out += struct.pack("<6qd", *row)
    for i, j, k, c in cg_entries:
        out += struct.pack("<3qd", i, j, k, c)
    return bytes(out)


def descriptor_hash(desc: bytes) -> int:
    """56-bit key of a descriptor (fits a torch ``int`` argument)."""
    return int.from_bytes(hashlib.sha256(desc).digest()[:7], "big")
