"""Graph preprocessing on the device: periodic radius graphs and the receiver-sorted layout.

The reference prepares convolution graphs on the host: ``CoordGraph``
(``core/ConvolutionBase.py:57-82``) sorts edges by (receiver, sender) and derives the
transpose permutation (the edge order sorted by (sender, receiver)) that the deterministic
backward pass needs; its benchmarks build radius graphs with scipy.  Here both steps run as
torch operations on whatever device the positions live on, so graphs that change every MD
step never leave the GPU:

* ``radius_graph``: all ordered pairs (receiver i, sender j), i != j, with minimum-image
  distance below the cutoff in a periodic cubic box, found through a cell list (cells of
  side >= cutoff, the 27 neighbouring cells of each node's cell);
* ``coord_graph``: receiver-sorted rows/cols plus the transpose permutation, as
  ``CoordGraph``;
* ``morton_order``: a spatial node numbering (Z-order curve of the positions), so that
  contiguous node ranges, which the multi-GPU convolution assigns to ranks, are compact
  regions with small halos.  The reference has no counterpart (its graphs are partitioned
  by nobody).
"""

from __future__ import annotations

from typing import Tuple

import torch


def _spread_bits(v: torch.Tensor) -> torch.Tensor:
    """Inserts two zero bits after each of the 21 low bits of v (int64)."""
    v = v & 0x1FFFFF
    v = (v | (v << 32)) & 0x1F00000000FFFF
    v = (v | (v << 16)) & 0x1F0000FF0000FF
    v = (v | (v << 8)) & 0x100F00F00F00F00F
    v = (v | (v << 4)) & 0x10C30C30C30C30C3
    v = (v | (v << 2)) & 0x1249249249249249
    return v


def morton_order(pos: torch.Tensor, box: float, bits: int = 16) -> torch.Tensor:
    """Permutation listing the nodes along a Z-order (Morton) curve of their positions.

    Positions are wrapped into the periodic box and quantised to ``2**bits`` cells per axis;
    node ``order[k]`` gets the new id ``k``.  Renumber with ``pos = pos[order]`` (and every
    per-node array alike) before building the graph.
    """
    assert 1 <= bits <= 21
    scale = float(1 << bits) / box
    q = torch.clamp((torch.remainder(pos, box) * scale).to(torch.int64), 0, (1 << bits) - 1)
    code = _spread_bits(q[:, 0]) | (_spread_bits(q[:, 1]) << 1) | (_spread_bits(q[:, 2]) << 2)
    return torch.argsort(code, stable=True)


def coord_graph(rows: torch.Tensor, cols: torch.Tensor, num_nodes: int
                ) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    """(rows, cols, transpose_perm, order): edges sorted by (receiver, sender).

    ``order`` maps sorted positions to the input edge order; ``transpose_perm[p]`` is the
    position (in the sorted list) of the p-th edge in (sender, receiver) order.
    """
    key = rows.to(torch.int64) * num_nodes + cols.to(torch.int64)
    key, order = torch.sort(key)
    rows_s, cols_s = key // num_nodes, key % num_nodes
    tkey = cols_s * num_nodes + rows_s
    tperm = torch.argsort(tkey, stable=True)
    return rows_s, cols_s, tperm, order


def radius_graph(pos: torch.Tensor, box: float, cutoff: float, chunk_pairs: int = 1 << 26
                 ) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    """Directed periodic radius graph: (rows, cols, transpose_perm, edge_vec), receiver-sorted.

    ``edge_vec[e]`` is the minimum-image vector from receiver ``rows[e]`` to sender
    ``cols[e]``.  ``chunk_pairs`` bounds the candidate pairs materialised at once.
    """
    n = pos.shape[0]
    dev = pos.device
    ncell = int(box // cutoff)
    if ncell < 3:
        # Too few cells for a 27-cell stencil without repeats: test every pair.
        i, j = torch.meshgrid(torch.arange(n, device=dev), torch.arange(n, device=dev),
                              indexing="ij")
        i, j = i.reshape(-1), j.reshape(-1)
        d = pos[j] - pos[i]
        d = d - box * torch.round(d / box)
        keep = (i != j) & ((d * d).sum(1) < cutoff * cutoff)
        rows, cols, tperm, _ = coord_graph(i[keep], j[keep], n)
        vec = pos[cols] - pos[rows]
        return rows, cols, tperm, vec - box * torch.round(vec / box)
    side = box / ncell
    cell3 = torch.clamp((torch.remainder(pos, box) / side).to(torch.int64), 0, ncell - 1)
    cell = (cell3[:, 0] * ncell + cell3[:, 1]) * ncell + cell3[:, 2]
    cell_sorted, node_of = torch.sort(cell)
    counts = torch.bincount(cell_sorted, minlength=ncell ** 3)
    start = torch.cumsum(counts, 0) - counts
    rows_all, cols_all = [], []
    offsets = [(a, b, c) for a in (-1, 0, 1) for b in (-1, 0, 1) for c in (-1, 0, 1)]
    for da, db, dc in offsets:
        nb = ((cell3 + torch.tensor([da, db, dc], device=dev)) % ncell)
        nbc = (nb[:, 0] * ncell + nb[:, 1]) * ncell + nb[:, 2]
        cnt = counts[nbc]                       # candidates per receiver
        total = int(cnt.sum())
        if total == 0:
            continue
        recv_all = torch.arange(n, device=dev)
        # Process receivers in chunks so that at most ~chunk_pairs candidates exist at once.
        csum = torch.cumsum(cnt, 0)
        lo = 0
        while lo < n:
            base = int(csum[lo - 1]) if lo > 0 else 0
            hi = int(torch.searchsorted(csum, torch.tensor(base + chunk_pairs, device=dev)))
            hi = max(hi, lo + 1)
            hi = min(hi, n)
            c = cnt[lo:hi]
            recv = torch.repeat_interleave(recv_all[lo:hi], c)
            first = torch.repeat_interleave(start[nbc[lo:hi]], c)
            rank = torch.arange(recv.numel(), device=dev) - torch.repeat_interleave(
                torch.cumsum(c, 0) - c, c)
            send = node_of[first + rank]
            d = pos[send] - pos[recv]
            d = d - box * torch.round(d / box)
            keep = (send != recv) & ((d * d).sum(1) < cutoff * cutoff)
            rows_all.append(recv[keep])
            cols_all.append(send[keep])
            lo = hi
    rows = torch.cat(rows_all)
    cols = torch.cat(cols_all)
    rows, cols, tperm, _ = coord_graph(rows, cols, n)
    vec = pos[cols] - pos[rows]
    vec = vec - box * torch.round(vec / box)
    return rows, cols, tperm, vec
