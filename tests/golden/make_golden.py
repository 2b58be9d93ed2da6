"""Generates the golden fixtures in this directory from the reference implementation.

Run where a checkout of the reference is available, naming it in ``OEQ_REFERENCE_ROOT``:
``OEQ_REFERENCE_ROOT=<checkout> python tests/golden/make_golden.py``.  The tests never read
the reference; the committed ``*.npz`` files are what they read.

What is taken from the reference (imported with ``OEQ_NOTORCH=1``):

* ``core/e3nn_lite.py``: ``wigner_3j`` tables and ``TPProblem`` path weights;
* ``_torch/utils.py:8-46`` ``reorder_helper`` (with ``ComputationSchedule``): the
  e3nn -> oeq weight permutation;
* ``core/ComputationSchedule.py``: the per-segment child instructions, their
  ``CGTensor`` coefficient literals (path weight folded in, exactly the constants the
  reference's generated kernels embed) and weight offsets.  ``_interp_forward`` /
  ``_interp_backward`` walk those objects with the loop structure of
  ``templates/loop_unroll_tp.cuh:19-313`` to produce reference outputs;
* ``benchmark/test_buffers.py``: the seeded input buffers;
* ``core/ConvolutionBase.py:57-82`` ``CoordGraph``: receiver sort + transpose permutation.
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np

OUT = Path(__file__).resolve().parent
if "OEQ_REFERENCE_ROOT" not in os.environ:
    sys.exit("set OEQ_REFERENCE_ROOT to a checkout of the reference (the directory that holds "
             "openequivariance/openequivariance)")
REF = Path(os.environ["OEQ_REFERENCE_ROOT"]) / "openequivariance"


def _import_reference():
    os.environ["OEQ_NOTORCH"] = "1"
    sys.path.insert(0, str(REF))
    import openequivariance.core.e3nn_lite as el
    from openequivariance.core.ComputationSchedule import ComputationSchedule, SMEMCapacityException
    from openequivariance.benchmark import test_buffers as tb
    from openequivariance.benchmark import problems as pr
    from openequivariance.core.ConvolutionBase import CoordGraph
    from openequivariance._torch.utils import reorder_helper
    return el, ComputationSchedule, SMEMCapacityException, tb, pr, CoordGraph, reorder_helper


el, ComputationSchedule, SMEMCapacityException, tb, pr, CoordGraph, reorder_helper = \
    _import_reference()


def _schedule(problem, direction):
    is_uvw = problem.instructions[0].connection_mode == "uvw"
    for warps in (4, 2, 1):
        try:
            return ComputationSchedule(
                problem, smem_limit=200000, warps_per_block=warps, warp_size=32, block_count=1,
                direction=direction, irrep_dtype=np.float64, weight_dtype=np.float64,
                include_scratch=is_uvw, stream_weights=is_uvw)
        except SMEMCapacityException:
            continue
    raise RuntimeError("schedule failed")


def _tuples(tensor):
    return [(int(a), int(b), int(c), float.fromhex(v.rstrip("f"))) for a, b, c, v in tensor.tuples]


def _child_block(arr, child_irreps, idx):
    sl = child_irreps.slices()[idx]
    mul, ir = child_irreps[idx]
    return arr[:, sl].reshape(arr.shape[0], mul, ir.dim)


def _interp_forward(sched, X, Y, W):
    B = X.shape[0]
    Z = np.zeros((B, sched.L3.dim))
    shared = sched.updated_config.shared_weights
    for seg in sched.segments:
        for k, (u, v, w, tensor) in enumerate(seg.interactions):
            inst = seg.problem.instructions[k]
            cu, cv, cw = seg.L1Map.idxs[u], seg.L2Map.idxs[v], seg.L3Map.idxs[w]
            x = _child_block(X, sched.L1, cu)
            y = _child_block(Y, sched.L2, cv)
            z = _child_block(Z, sched.L3, cw)  # view into Z
            m1, m2, m3 = sched.L1[cu].mul, sched.L2[cv].mul, sched.L3[cw].mul
            off = seg.weight_offset + seg.problem.weight_range_and_shape_for_instruction(k)[0]
            Wr = W[None, :] if shared else W
            for kk in range(m2):
                if inst.connection_mode == "uvu":
                    wt = Wr[:, off + kk * m1: off + (kk + 1) * m1]          # [B, u]
                    for i, j, kz, c in _tuples(tensor):
                        z[:, :, kz] += c * x[:, :, i] * (y[:, kk, j][:, None] * wt)
                else:
                    blk = Wr[:, off + kk * m1 * m3: off + (kk + 1) * m1 * m3].reshape(-1, m1, m3)
                    t = np.zeros((B, m1, z.shape[2]))
                    for i, j, kz, c in _tuples(tensor):
                        t[:, :, kz] += c * x[:, :, i] * y[:, kk, j][:, None]
                    z += np.einsum("buw,buk->bwk", np.broadcast_to(blk, (B, m1, m3)), t)
    return Z


def _interp_backward(sched, X, Y, W, G):
    B = X.shape[0]
    shared = sched.updated_config.shared_weights
    gX, gY = np.zeros_like(X), np.zeros_like(Y)
    gW = np.zeros((B, W.shape[-1])) if not shared else np.zeros(W.shape[-1])
    for seg in sched.segments:
        for k, (u, v, w, tensor) in enumerate(seg.interactions):
            inst = seg.problem.instructions[k]
            cu, cv, cw = seg.L1Map.idxs[u], seg.L2Map.idxs[v], seg.L3Map.idxs[w]
            x = _child_block(X, sched.L1, cu)
            y = _child_block(Y, sched.L2, cv)
            g = _child_block(G, sched.L3, cw)
            gx = _child_block(gX, sched.L1, cu)
            gy = _child_block(gY, sched.L2, cv)
            m1, m2, m3 = sched.L1[cu].mul, sched.L2[cv].mul, sched.L3[cw].mul
            off = seg.weight_offset + seg.problem.weight_range_and_shape_for_instruction(k)[0]
            Wr = W[None, :] if shared else W
            tup = _tuples(tensor)
            for kk in range(m2):
                if inst.connection_mode == "uvu":
                    wt = np.broadcast_to(Wr[:, off + kk * m1: off + (kk + 1) * m1], (B, m1))
                    wg = np.zeros((B, m1))
                    for i, j, kz, c in tup:
                        s1 = g[:, :, kz] * c
                        wg += s1 * y[:, kk, j][:, None] * x[:, :, i]
                        gy[:, kk, j] += np.sum(s1 * wt * x[:, :, i], axis=1)
                        gx[:, :, i] += s1 * wt * y[:, kk, j][:, None]
                    if shared:
                        gW[off + kk * m1: off + (kk + 1) * m1] += wg.sum(0)
                    else:
                        gW[:, off + kk * m1: off + (kk + 1) * m1] = wg
                else:
                    blk = np.broadcast_to(
                        Wr[:, off + kk * m1 * m3: off + (kk + 1) * m1 * m3].reshape(-1, m1, m3),
                        (B, m1, m3))
                    dt = np.einsum("buw,bwk->buk", blk, g)
                    t = np.zeros((B, m1, g.shape[2]))
                    for i, j, kz, c in tup:
                        s1 = dt[:, :, kz] * c
                        gy[:, kk, j] += np.sum(s1 * x[:, :, i], axis=1)
                        gx[:, :, i] += s1 * y[:, kk, j][:, None]
                        t[:, :, kz] += c * x[:, :, i] * y[:, kk, j][:, None]
                    wgrad = np.einsum("bwk,buk->buw", g, t).reshape(B, -1)
                    if shared:
                        gW[off + kk * m1 * m3: off + (kk + 1) * m1 * m3] += wgrad.sum(0)
                    else:
                        gW[:, off + kk * m1 * m3: off + (kk + 1) * m1 * m3] = wgrad
    return gX, gY, gW


def _problems():
    CTPP, FCTPP = pr.ChannelwiseTPP, pr.FullyConnectedTPProblem
    out = {
        "c1": el.TPProblem("1x2e", "1x3e", "1x2e", [(0, 0, 0, "uvu", True)],
                           shared_weights=False, internal_weights=False),
        "mace_large": pr.mace_problems()[0],
        "c2_literal": CTPP("128x0e+128x1o+128x2e", "1x0e+1x1o+1x2e+1x3o",
                           "128x0e+128x0o+128x1e+128x1o+128x2e+128x2o+128x3e+128x3o",
                           "c2-literal"),
        "c4_nequip_uvw": FCTPP("32x0e+32x0o+32x1e+32x1o+32x2e+32x2o", "1x0e+1x1o+1x2e",
                               "32x0e+32x0o+32x1e+32x1o+32x2e+32x2o"),
        "diffdock_l1": pr.diffdock_problems()[0],
        "uvu_33_l222": el.TPProblem("33x2e", "1x2e", "33x2e", [(0, 0, 0, "uvu", True)],
                                    shared_weights=False, internal_weights=False),
        "uvu_16x40_l111": el.TPProblem("16x1e", "40x1e", "16x1e", [(0, 0, 0, "uvu", True)],
                                       shared_weights=False, internal_weights=False),
        "uvw_49_l101": el.TPProblem("49x1e", "1x0e", "49x1e", [(0, 0, 0, "uvw", True)],
                                    shared_weights=False, internal_weights=False),
        "uvw_24x24_l111": el.TPProblem("24x1e", "24x1e", "24x1e", [(0, 0, 0, "uvw", True)],
                                       shared_weights=False, internal_weights=False),
        "uvu_l725": el.TPProblem("3x7e", "1x2e", "3x5e", [(0, 0, 0, "uvu", True)],
                                 shared_weights=False, internal_weights=False),
        "uvw_l535": el.TPProblem("5x5e", "2x3e", "4x5e", [(0, 0, 0, "uvw", True)],
                                 shared_weights=False, internal_weights=False),
        "mace_medium_shared": pr.mace_problems()[1],
        "nequip_lips": pr.nequip_problems()[0],
    }
    out["mace_medium_shared"].shared_weights = True
    for p in out.values():
        p.irrep_dtype = p.weight_dtype = np.float64
    return out


def _spec(problem):
    return dict(
        irreps_in1=str(problem.irreps_in1), irreps_in2=str(problem.irreps_in2),
        irreps_out=str(problem.irreps_out),
        instructions=np.array([[i.i_in1, i.i_in2, i.i_out] for i in problem.instructions],
                              dtype=np.int64),
        modes=np.array([i.connection_mode for i in problem.instructions]),
        path_weights=np.array([i.path_weight for i in problem.instructions]),
        weight_numel=np.int64(problem.weight_numel),
        shared_weights=np.bool_(problem.shared_weights),
    )


def _perm(problem):
    import torch

    sched = _schedule(problem, "forward")
    idx = torch.arange(problem.weight_numel, dtype=torch.float64)
    return reorder_helper(sched, idx, "forward", False).numpy().astype(np.int64)


def make_tp(seed=12345):
    for name, problem in _problems().items():
        row_doubles = (problem.irreps_in1.dim + problem.irreps_in2.dim + problem.irreps_out.dim
                       + (0 if problem.shared_weights else problem.weight_numel))
        batch = 6 if row_doubles <= 2000 else 2
        fs, bs = _schedule(problem, "forward"), _schedule(problem, "backward")
        perm = _perm(problem)
        X, Y, We3, _ = tb.get_random_buffers_forward(problem, batch, seed)
        X2, Y2, G, We3b, _, _, _ = tb.get_random_buffers_backward(problem, batch, seed + 1)
        W = We3[..., perm]
        Wb = We3b[..., perm]
        Z = _interp_forward(fs, X, Y, W)
        gX, gY, gW = _interp_backward(bs, X2, Y2, Wb, G)
        np.savez_compressed(
            OUT / f"tp_{name}.npz", **_spec(problem), perm=perm,
            X=X, Y=Y, W_e3nn=We3, Z=Z,
            bX=X2, bY=Y2, bW_e3nn=We3b, G=G, gX=gX, gY=gY, gW_oeq=gW)
        print("wrote", name, problem.weight_numel)


def make_conv(seed=7):
    rng = np.random.default_rng(seed)
    n = 8
    pairs = set()
    while len(pairs) < 20:
        a, b = rng.integers(0, n, 2)
        if a != b:
            pairs.add((int(a), int(b)))
            pairs.add((int(b), int(a)))
    pairs = sorted(pairs)
    rows = np.array([p[0] for p in pairs], dtype=np.int64)
    cols = np.array([p[1] for p in pairs], dtype=np.int64)
    shuffle = rng.permutation(len(rows))
    g = CoordGraph(np.zeros((n, 3)), rows[shuffle], cols[shuffle], "golden")
    for name in ("c1", "nequip_lips", "uvw_l535", "uvu_l725"):
        problem = _problems()[name]
        fs, bs = _schedule(problem, "forward"), _schedule(problem, "backward")
        perm = _perm(problem)
        X, Y, We3, _ = tb.get_random_buffers_forward_conv(problem, n, g.nnz, seed)
        _, _, G, _, _, _, _ = tb.get_random_buffers_backward_conv(problem, n, g.nnz, seed + 1)
        W = We3[..., perm]
        msg = _interp_forward(fs, X[g.cols], Y, W)
        Z = np.zeros((n, problem.irreps_out.dim))
        np.add.at(Z, g.rows, msg)
        gXe, gY, gW = _interp_backward(bs, X[g.cols], Y, W, G[g.rows])
        gX = np.zeros_like(X)
        np.add.at(gX, g.cols, gXe)
        np.savez_compressed(
            OUT / f"conv_{name}.npz", **_spec(problem), perm=perm, rows=g.rows, cols=g.cols,
            transpose_perm=g.transpose_perm, node_count=np.int64(n), X=X, Y=Y, W_e3nn=We3,
            Z=Z, G=G, gX=gX, gY=gY, gW_oeq=gW)
        print("wrote conv", name, g.nnz)


def make_cg(lmax=4):
    tables = {}
    triples = [(a, b, c) for a in range(lmax + 1) for b in range(lmax + 1)
               for c in range(abs(a - b), min(a + b, lmax) + 1)]
    triples += [(7, 2, 5), (5, 3, 5), (6, 6, 6), (7, 7, 7)]
    for t in triples:
        tables[f"{t[0]}_{t[1]}_{t[2]}"] = el.wigner_3j(*t)
    np.savez_compressed(OUT / "cg_wigner3j.npz", **tables)
    print("wrote", len(tables), "cg tables")


if __name__ == "__main__":
    make_cg()
    make_tp()
    make_conv()
