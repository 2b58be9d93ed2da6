"""Multi-GPU fused convolution: receiver-range node partitions with halo exchange.

Each rank owns a contiguous range of receiver nodes (ranges balanced by edge count) and every
edge whose receiver it owns.  With nodes numbered in a spatial order (``graph.morton_order``)
a contiguous range is a compact region of space, so only the senders near its surface (the
*halo*) belong to other ranks.  A rank's edges fall into two blocks, each receiver-sorted:

* interior edges, whose sender the rank owns;
* boundary edges, whose sender is a halo node (plus up to three edges with an owned sender,
  so that the boundary block starts at a multiple of 4 edges).

Per pass, node data crosses NVLink once each way, overlapped with the interior edges:

* forward: the rank sends the X rows its neighbours need (``all_to_all_single``, NCCL,
  started asynchronously) and meanwhile runs the fused convolution of its interior edges;
  once the halo rows have arrived it runs the boundary edges and adds their messages;
* backward: the boundary edges go first (their dX contributions belong to halo nodes), the
  contributions travel back to their owners while the interior edges run, and each owner
  adds what it received in rank order (deterministic: one writer per row and call).

dY and dW stay local per edge.  Node ids are local: ``[0, n_own)`` the owned nodes,
``[n_own, n_own + n_halo)`` the halo nodes grouped by owning rank (ascending global id), so the
single-GPU kernels run unchanged on a node space of ``n_own + n_halo`` rows.  Every rank issues
the same collectives in the same order.  The reference has no multi-GPU path (its
``tests/multidevice_test.py:14-30`` runs independent replicas); this partitions its fused
convolution (``TensorProductConv.forward``, ``_torch/TensorProductConv.py:145-200``).
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Callable, List, Optional

import torch
import torch.distributed as dist


@dataclass
class ReceiverPartition:
    """This rank's share of a receiver-sorted graph (see the module docstring)."""

    rank: int
    world: int
    num_nodes: int
    node_lo: int                   # owned nodes [node_lo, node_hi) (global ids)
    node_hi: int
    halo_nodes: torch.Tensor       # [n_halo] global ids of the halo, grouped by owner rank
    recv_counts: List[int]         # halo rows arriving from each rank
    send_idx: torch.Tensor         # owned local ids sent to the other ranks, by destination
    send_counts: List[int]         # rows sent to each rank
    edge_index: torch.Tensor       # [E_local] global edge ids in local order (interior first)
    n_interior: int
    rows_int: torch.Tensor         # interior edges: local receiver / sender ids
    cols_int: torch.Tensor
    rows_bnd: torch.Tensor         # boundary edges: local receiver / sender (halo) ids
    cols_bnd: torch.Tensor
    tperm_int: torch.Tensor        # each block's edges in (sender, receiver) order
    tperm_bnd: torch.Tensor
    send_splits: List[torch.Tensor] = field(default_factory=list)  # send_idx per destination
    n_boundary_local: int = 0      # boundary-block edges whose sender is owned (0..3)
    # Fixed-order sums of the dX rows that come back from the other ranks: the positions of
    # send_idx sorted by (node, rank), the distinct nodes, and each node's count.
    back_order: Optional[torch.Tensor] = None
    back_nodes: Optional[torch.Tensor] = None
    back_counts: Optional[torch.Tensor] = None

    @property
    def n_own(self) -> int:
        return self.node_hi - self.node_lo

    @property
    def n_halo(self) -> int:
        return int(self.halo_nodes.numel())

    @property
    def n_local_nodes(self) -> int:
        return self.n_own + self.n_halo

    @property
    def n_edges(self) -> int:
        return int(self.edge_index.numel())

    @property
    def n_boundary(self) -> int:
        return self.n_edges - self.n_interior

    @staticmethod
    def build(rows: torch.Tensor, cols: torch.Tensor, num_nodes: int, world: int, rank: int
              ) -> "ReceiverPartition":
        """Partition of the receiver-sorted global graph (rows, cols), on their device.

        Every rank calls this with the whole graph and computes the same node ranges; no
        communication is needed.  Node ranges balance the edge counts.
        """
        rows = rows.to(torch.int64)
        cols = cols.to(torch.int64)
        dev = rows.device
        E = rows.numel()
        deg_cum = torch.searchsorted(rows, torch.arange(num_nodes + 1, device=dev))
        targets = torch.tensor([E * r // world for r in range(world + 1)], device=dev)
        bounds = torch.searchsorted(deg_cum, targets).clamp(max=num_nodes)
        bounds[0], bounds[-1] = 0, num_nodes
        bounds = torch.cummax(bounds, 0).values
        b = bounds.tolist()
        ecut = deg_cum[bounds].tolist()
        owner = torch.searchsorted(bounds[1:], torch.arange(num_nodes, device=dev), right=True)
        lo, hi = b[rank], b[rank + 1]
        e_lo, e_hi = ecut[rank], ecut[rank + 1]
        n_own = hi - lo
        r_g, c_g = rows[e_lo:e_hi], cols[e_lo:e_hi]
        local_src = owner[c_g] == rank
        halo = torch.unique(c_g[~local_src])  # sorted global ids, hence grouped by owner
        # The boundary block starts at a multiple of 4 edges, so that its Y / dY rows are
        # 16-byte aligned whenever the caller's arrays are (the vectorised edge kernels need
        # that): the last (count % 4) edges with a local sender join the boundary block.
        inner = local_src.clone()
        extra = int(inner.sum()) % 4 if halo.numel() else 0
        if extra:
            inner[torch.nonzero(inner).flatten()[-extra:]] = False
        idx = torch.arange(e_lo, e_hi, device=dev)
        recv_counts = torch.bincount(owner[halo], minlength=world).tolist() if halo.numel() \
            else [0] * world
        rows_int, cols_int = r_g[inner] - lo, c_g[inner] - lo
        rows_bnd = r_g[~inner] - lo
        cb = c_g[~inner]
        in_halo = n_own + torch.searchsorted(halo, cb).clamp(max=max(halo.numel() - 1, 0))
        cols_bnd = torch.where(owner[cb] == rank, cb - lo, in_halo)
        # What every other rank needs from this one: the senders of its edges that this rank
        # owns, in ascending global id (the order that rank expects them in its halo).
        send_splits, send_counts = [], []
        for r in range(world):
            if r == rank:
                send_splits.append(torch.empty(0, dtype=torch.int64, device=dev))
            else:
                cr = cols[ecut[r]:ecut[r + 1]]
                send_splits.append(torch.unique(cr[owner[cr] == rank]) - lo)
            send_counts.append(int(send_splits[-1].numel()))
        n_loc = n_own + int(halo.numel())

        def tperm(rr, cc):
            return torch.argsort(cc * max(n_loc, 1) + rr, stable=True)

        send_idx = torch.cat(send_splits)
        # send_idx is grouped by destination rank, so a stable sort by node keeps rank order.
        back_order = torch.argsort(send_idx, stable=True)
        back_nodes, back_counts = torch.unique_consecutive(send_idx[back_order],
                                                           return_counts=True)
        return ReceiverPartition(
            rank, world, num_nodes, lo, hi, halo, recv_counts, send_idx,
            send_counts, torch.cat([idx[inner], idx[~inner]]), int(inner.sum()),
            rows_int, cols_int, rows_bnd, cols_bnd, tperm(rows_int, cols_int),
            tperm(rows_bnd, cols_bnd), send_splits, extra, back_order, back_nodes, back_counts)


def _local_conv_ops(conv):
    """(forward, backward-into) of the fused convolution module on a local node space.

    ``fwd(X, Y, W, rows, cols, tperm) -> Z`` with Z of X's row count;
    ``bwd(X, Y, W, G, rows, cols, tperm, gX, gY, gW)`` writes the gradients into the given
    tensors (contiguous row slices of the callers' buffers).
    """
    ops = torch.ops.libtorch_tp_jit

    def fwd(X, Y, W, rows, cols, tperm):
        perm = tperm if conv.deterministic else conv.dummy_transpose_perm
        return ops.jit_conv_forward(conv.kernel, conv.hash, X, Y, W, conv.L3_dim, rows, cols,
                                    conv.workspace_buffer, perm)

    def bwd(X, Y, W, G, rows, cols, tperm, gX, gY, gW):
        perm = tperm if conv.deterministic else conv.dummy_transpose_perm
        torch.ops.oeqb200.conv_backward_into(conv.kernel, conv.hash, X, Y, W, G, rows, cols,
                                             conv.workspace_buffer, perm, gX, gY, gW)

    return fwd, bwd


class _HaloConvFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, X_own, Y, W, pc):
        part = pc.part
        n_own, n_loc, ni = part.n_own, part.n_local_nodes, part.n_interior
        shared = pc.shared_weights
        exchange = part.world > 1
        if part.n_halo == 0:
            X_loc = X_own.contiguous()
        else:
            X_loc = X_own.new_empty(n_loc, X_own.shape[1])
            X_loc[:n_own].copy_(X_own)
        work = None
        if exchange:
            send = X_own.index_select(0, part.send_idx)
            work = dist.all_to_all_single(X_loc[n_own:], send, part.recv_counts,
                                          part.send_counts, group=pc.group, async_op=True)
        Wi = W if shared else W[:ni]
        Z = pc.fwd(X_loc, Y[:ni], Wi, part.rows_int, part.cols_int, part.tperm_int)
        if work is not None:
            work.wait()
        if part.n_boundary:
            Wb = W if shared else W[ni:]
            Z.add_(pc.fwd(X_loc, Y[ni:], Wb, part.rows_bnd, part.cols_bnd, part.tperm_bnd))
        ctx.save_for_backward(X_loc, Y, W)
        ctx.pc = pc
        return Z[:n_own]

    @staticmethod
    def backward(ctx, gZ):
        if torch.is_grad_enabled():
            raise RuntimeError("double backward through PartitionedConv is not supported")
        X_loc, Y, W = ctx.saved_tensors
        pc = ctx.pc
        part = pc.part
        n_own, n_loc, ni = part.n_own, part.n_local_nodes, part.n_interior
        shared = pc.shared_weights
        if part.n_halo == 0:
            gZ_loc = gZ.contiguous()
        else:
            gZ_loc = gZ.new_zeros(n_loc, gZ.shape[1])
            gZ_loc[:n_own].copy_(gZ)
        gY = torch.empty_like(Y)
        gW = torch.empty_like(W)
        d1 = X_loc.shape[1]
        work, back = None, None
        if part.n_boundary or part.world > 1:
            gX_b = X_loc.new_empty(n_loc, d1)
            gW_b = torch.empty_like(W) if shared else gW[ni:]
            if part.n_boundary:
                pc.bwd(X_loc, Y[ni:], W if shared else W[ni:], gZ_loc, part.rows_bnd,
                       part.cols_bnd, part.tperm_bnd, gX_b, gY[ni:], gW_b)
            else:
                gX_b.zero_()
                if shared:
                    gW_b.zero_()
            if part.world > 1:
                back = X_loc.new_empty(int(part.send_idx.numel()), d1)
                work = dist.all_to_all_single(back, gX_b[n_own:], part.send_counts,
                                              part.recv_counts, group=pc.group, async_op=True)
        gX_i = X_loc.new_empty(n_loc, d1)
        gW_i = torch.empty_like(W) if shared else gW[:ni]
        pc.bwd(X_loc, Y[:ni], W if shared else W[:ni], gZ_loc, part.rows_int, part.cols_int,
               part.tperm_int, gX_i, gY[:ni], gW_i)
        gX = gX_i[:n_own]
        if part.n_boundary_local:
            gX.add_(gX_b[:n_own])  # the boundary block's edges with an owned sender
        if work is not None:
            work.wait()
            if back.shape[0]:
                if pc.deterministic:
                    # Each node's contributions summed in rank order, then one add per node.
                    sums = torch.segment_reduce(back[part.back_order], "sum",
                                                lengths=part.back_counts)
                    gX.index_add_(0, part.back_nodes, sums)
                else:
                    gX.index_add_(0, part.send_idx, back)
        if shared:
            gW = gW_i + gW_b if (part.n_boundary or part.world > 1) else gW_i
            if part.world > 1:
                dist.all_reduce(gW, group=pc.group)
        return gX, gY, gW, None


class _HaloConvRows8Fn(torch.autograd.Function):
    """The atomic pass on node arrays in the kernels' padded-row layout (``[nodes, 8]``,
    ``oeqb_conv_forward_rows8`` / ``oeqb_conv_backward_rows8``).

    Halo rows arrive from the other ranks straight into the padded X buffer, and the boundary
    backward's dX rows leave straight from the padded accumulator.  With more than one rank
    the boundary block runs on a side stream, on the ``reserve_sms`` SMs the interior kernel
    leaves free, in order with the exchange: forward = exchange, then boundary edges (adding
    into Z) beside the interior edges; backward = boundary edges, then exchange, beside the
    interior edges.  Both blocks add into Z / the dX accumulator with vector reductions, so
    running them at the same time is fine in this (atomic) mode."""

    @staticmethod
    def forward(ctx, X_own, Y, W, pc):
        part = pc.part
        n_own, n_loc, ni = part.n_own, part.n_local_nodes, part.n_interior
        conv = pc.conv
        ops = torch.ops.oeqb200
        d1 = X_own.shape[1]
        cur = torch.cuda.current_stream(X_own.device)
        xp = X_own.new_empty(n_loc, 8)
        xp[:n_own, :d1].copy_(X_own)
        Z = X_own.new_zeros(n_loc, conv.L3_dim)
        if part.world == 1:
            ops.conv_forward_rows8(conv.kernel, conv.hash, xp, Y[:ni], W[:ni], Z, part.rows_int,
                                   part.cols_int, True, 0)
        else:
            R = pc.reserve_sms
            send = xp.index_select(0, part.send_idx)
            side = pc.side_stream(X_own.device)
            side.wait_stream(cur)
            with torch.cuda.stream(side):
                work = dist.all_to_all_single(xp[n_own:], send, part.recv_counts,
                                              part.send_counts, group=pc.group, async_op=True)
                work.wait()
                if part.n_boundary:
                    ops.conv_forward_rows8(conv.kernel, conv.hash, xp, Y[ni:], W[ni:], Z,
                                           part.rows_bnd, part.cols_bnd, True, R)
            ops.conv_forward_rows8(conv.kernel, conv.hash, xp, Y[:ni], W[:ni], Z, part.rows_int,
                                   part.cols_int, True, -R)
            cur.wait_stream(side)
            for t in (xp, send, Z, Y, W):
                t.record_stream(side)
        ctx.save_for_backward(xp, Y, W)
        ctx.pc = pc
        ctx.d1 = d1
        return Z[:n_own]

    @staticmethod
    def backward(ctx, gZ):
        if torch.is_grad_enabled():
            raise RuntimeError("double backward through PartitionedConv is not supported")
        xp, Y, W = ctx.saved_tensors
        pc = ctx.pc
        part = pc.part
        conv = pc.conv
        ops = torch.ops.oeqb200
        n_own, n_loc, ni = part.n_own, part.n_local_nodes, part.n_interior
        cur = torch.cuda.current_stream(xp.device)
        gp = xp.new_empty(n_loc, 8)  # only the receivers' (owned) rows are read
        gp[:n_own, :gZ.shape[1]].copy_(gZ)
        dxp = xp.new_zeros(n_loc, 8)
        gY = torch.empty_like(Y)
        gW = torch.empty_like(W)
        if part.world == 1:
            ops.conv_backward_rows8(conv.kernel, conv.hash, xp, gp, Y[:ni], W[:ni], gY[:ni],
                                    gW[:ni], dxp, part.rows_int, part.cols_int, 0)
        else:
            R = pc.reserve_sms
            back = xp.new_empty(int(part.send_idx.numel()), 8)
            side = pc.side_stream(xp.device)
            side.wait_stream(cur)
            with torch.cuda.stream(side):
                if part.n_boundary:
                    ops.conv_backward_rows8(conv.kernel, conv.hash, xp, gp, Y[ni:], W[ni:],
                                            gY[ni:], gW[ni:], dxp, part.rows_bnd, part.cols_bnd, R)
                work = dist.all_to_all_single(back, dxp[n_own:], part.send_counts,
                                              part.recv_counts, group=pc.group, async_op=True)
                work.wait()
            ops.conv_backward_rows8(conv.kernel, conv.hash, xp, gp, Y[:ni], W[:ni], gY[:ni],
                                    gW[:ni], dxp, part.rows_int, part.cols_int, -R)
            cur.wait_stream(side)
            for t in (xp, gp, dxp, back, gY, gW, Y, W):
                t.record_stream(side)
            if back.shape[0]:
                dxp.index_add_(0, part.send_idx, back)
        return dxp[:n_own, :ctx.d1].contiguous(), gY, gW, None


class PartitionedConv(torch.nn.Module):
    """Fused convolution of a receiver-partitioned graph (one rank per GPU).

    ``forward(X_own, Y_local, W_local)`` takes this rank's node rows of X
    (``X[part.node_lo:part.node_hi]``) and its edges' Y and W in the partition's local edge
    order (``Y[part.edge_index]``: interior edges first) and returns this rank's rows of Z.
    ``conv`` is a ``TensorProductConv`` (atomic or deterministic).  ``local_ops`` replaces its
    kernels with another (forward, backward-into) pair of the same signature (e.g. a CPU
    implementation for host-side tests); ``shared_weights`` and ``deterministic`` must then
    be given.

    Nothing in a pass synchronises with the host, so a whole training or MD step that uses the
    module (forward, autograd backward, the NCCL exchanges) can be captured in one CUDA graph
    and replayed, which removes the per-step launch cost of its ~20 small operations.
    """

    def __init__(self, conv, part: ReceiverPartition, group=None,
                 local_ops: Optional[tuple[Callable, Callable]] = None,
                 shared_weights: Optional[bool] = None, deterministic: Optional[bool] = None,
                 reserve_sms: int = 16):
        super().__init__()
        self.conv = conv
        self.part = part
        self.group = group
        self._default_ops = local_ops is None
        self.fwd, self.bwd = local_ops if local_ops is not None else _local_conv_ops(conv)
        self.shared_weights = (bool(conv.config.shared_weights) if shared_weights is None
                               else shared_weights)
        self.deterministic = (bool(conv.deterministic) if deterministic is None
                              else deterministic)
        # SMs the interior kernels leave free for the exchange and the boundary block, which
        # run beside them on a side stream (padded-row path, more than one rank).
        self.reserve_sms = reserve_sms
        self._rows8 = None
        self._side = {}

    def side_stream(self, device):
        """This module's second stream on `device` (the boundary block and the exchange), of
        high priority: when its kernels and the interior kernel become ready together, the
        block scheduler places its CTAs first.  (Give NCCL high-priority streams too,
        ``ProcessGroupNCCL.Options(is_high_priority_stream=True)``, for the same reason.)"""
        key = device.index
        if key not in self._side:
            self._side[key] = torch.cuda.Stream(device, priority=-1)
        return self._side[key]

    def _use_rows8(self, X_own):
        """The padded-row path: atomic plans of the single-path class, on the GPU."""
        if self._rows8 is None:
            ok = (local_ops_default(self) and not self.deterministic and X_own.is_cuda
                  and X_own.dtype == torch.float32)
            if ok:
                ok = bool(torch.ops.oeqb200.conv_rows8_ok(self.conv.kernel, self.conv.hash,
                                                          X_own.device.index))
            self._rows8 = ok
        return self._rows8

    def forward(self, X_own, Y_local, W_local):
        if self._use_rows8(X_own) and Y_local.is_contiguous() and W_local.is_contiguous():
            return _HaloConvRows8Fn.apply(X_own, Y_local, W_local, self)
        return _HaloConvFn.apply(X_own, Y_local, W_local, self)


def local_ops_default(pc) -> bool:
    """True when ``pc`` runs this package's kernels (no ``local_ops`` replacement)."""
    return pc._default_ops
