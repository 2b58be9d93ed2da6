"""Timed CPU baseline -- TEST/BENCH INFRASTRUCTURE ONLY (used by ``bench.py``'s
reference arm and ``cpu_baseline`` leg, never by the product).

The reference has no CPU implementation of this path: its ``forward_cpu``/``backward_cpu``
take numpy arrays but run e3nn on the GPU (``_torch/E3NNTensorProduct.py:52,66-70``), and
e3nn is not installed.  This module is the CPU port that stands in for it: the oracle's
e3nn-semantics contractions (``oracle/tp_oracle.py``) expressed as multithreaded torch-CPU
einsums (one per instruction, Clebsch-Gordan tables dense), plus ``index_add`` scatters
for the convolution.
"""

from __future__ import annotations

import os
import time

import numpy as np
import torch

import tp_oracle as O


class CpuTP:
    def __init__(self, p: O.Problem, dtype=torch.float32):
        self.p = p
        self.dtype = dtype
        self.o1, self.d1 = O.Problem.dims(p.irreps1)
        self.o2, self.d2 = O.Problem.dims(p.irreps2)
        self.o3, self.d3 = O.Problem.dims(p.irreps3)
        self.C = []
        for k, ins in enumerate(p.instructions):
            l1, l2, l3 = p.irreps1[ins[0]][1], p.irreps2[ins[1]][1], p.irreps3[ins[2]][1]
            c = O.wigner_3j(l1, l2, l3) * p.path_weights[k]
            self.C.append(torch.tensor(c, dtype=dtype))

    def _blk(self, a, irreps, offs, i):
        mul, l, _ = irreps[i]
        return a[:, offs[i]:offs[i] + mul * (2 * l + 1)].reshape(a.shape[0], mul, 2 * l + 1)

    def _w(self, W, k):
        shp = self.p.shape(self.p.instructions[k])
        o = self.p.weight_offsets[k]
        n = int(np.prod(shp))
        if self.p.shared_weights:
            return W[o:o + n].reshape(shp)
        return W[:, o:o + n].reshape((W.shape[0],) + shp)

    def forward(self, X, Y, W):
        p = self.p
        Z = torch.zeros(X.shape[0], self.d3, dtype=self.dtype)
        for k, ins in enumerate(p.instructions):
            x = self._blk(X, p.irreps1, self.o1, ins[0])
            y = self._blk(Y, p.irreps2, self.o2, ins[1])
            w = self._w(W, k)
            s = "" if p.shared_weights else "b"
            if ins[3] == "uvu":
                z = torch.einsum(f"ijk,bui,{s}uv,bvj->buk", self.C[k], x, w, y)
            else:
                z = torch.einsum(f"ijk,bui,{s}uvw,bvj->bwk", self.C[k], x, w, y)
            o = self.o3[ins[2]]
            Z[:, o:o + z.shape[1] * z.shape[2]] += z.reshape(X.shape[0], -1)
        return Z

    def backward(self, X, Y, W, G):
        p = self.p
        gX, gY, gW = torch.zeros_like(X), torch.zeros_like(Y), torch.zeros_like(W)
        for k, ins in enumerate(p.instructions):
            x = self._blk(X, p.irreps1, self.o1, ins[0])
            y = self._blk(Y, p.irreps2, self.o2, ins[1])
            g = self._blk(G, p.irreps3, self.o3, ins[2])
            w = self._w(W, k)
            s = "" if p.shared_weights else "b"
            wi = "uv" if ins[3] == "uvu" else "uvw"
            gi = "buk" if ins[3] == "uvu" else "bwk"
            gx = torch.einsum(f"ijk,{s}{wi},bvj,{gi}->bui", self.C[k], w, y, g)
            gy = torch.einsum(f"ijk,bui,{s}{wi},{gi}->bvj", self.C[k], x, w, g)
            gw = torch.einsum(f"ijk,bui,bvj,{gi}->{s}{wi}", self.C[k], x, y, g)
            o1, o2 = self.o1[ins[0]], self.o2[ins[1]]
            gX[:, o1:o1 + gx.shape[1] * gx.shape[2]] += gx.reshape(X.shape[0], -1)
            gY[:, o2:o2 + gy.shape[1] * gy.shape[2]] += gy.reshape(X.shape[0], -1)
            o = p.weight_offsets[k]
            if p.shared_weights:
                gW[o:o + gw.numel()] += gw.reshape(-1)
            else:
                gW[:, o:o + gw[0].numel()] += gw.reshape(X.shape[0], -1)
        return gX, gY, gW


def time_tp_fwd_bwd(p: O.Problem, rows: int, reps: int = 1, seed: int = 0, threads=None):
    """Seconds per forward+backward over ``rows`` rows, and the thread count used."""
    threads = threads or os.cpu_count() or 1
    torch.set_num_threads(threads)
    rng = np.random.default_rng(seed)
    tp = CpuTP(p)
    d1, d2, d3 = tp.d1, tp.d2, tp.d3
    X = torch.tensor(rng.normal(size=(rows, d1)), dtype=torch.float32)
    Y = torch.tensor(rng.normal(size=(rows, d2)), dtype=torch.float32)
    wshape = (p.weight_numel,) if p.shared_weights else (rows, p.weight_numel)
    W = torch.tensor(rng.normal(size=wshape), dtype=torch.float32)
    G = torch.tensor(rng.normal(size=(rows, d3)), dtype=torch.float32)
    tp.forward(X[:2], Y[:2], W if p.shared_weights else W[:2])  # warm the einsum planner
    t0 = time.perf_counter()
    for _ in range(reps):
        tp.forward(X, Y, W)
        tp.backward(X, Y, W, G)
    return (time.perf_counter() - t0) / reps, threads


def time_conv_fwd_bwd(p: O.Problem, X, Y, W, G, rows, cols, reps=1, threads=None):
    threads = threads or os.cpu_count() or 1
    torch.set_num_threads(threads)
    tp = CpuTP(p)
    r = torch.as_tensor(rows)
    c = torch.as_tensor(cols)
    t0 = time.perf_counter()
    for _ in range(reps):
        msg = tp.forward(X[c], Y, W)
        Z = torch.zeros(X.shape[0], tp.d3).index_add_(0, r, msg)
        gXe, gY, gW = tp.backward(X[c], Y, W, G[r])
        gX = torch.zeros_like(X).index_add_(0, c, gXe)
    del Z, gX, gY, gW
    return (time.perf_counter() - t0) / reps, threads
