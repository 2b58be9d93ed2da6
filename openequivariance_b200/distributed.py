"""Multi-GPU fused convolution: receiver-range node partitions over ``torch.distributed``.

Each rank owns a contiguous range of receiver nodes (ranges balanced by edge count) and every
edge whose receiver it owns; with receiver-sorted edges (``graph.coord_graph``) that is a
contiguous slice of the edge list.  Edge data (Y, W) and the rank's node data (X, Z rows) stay
local.  One pass exchanges node data only:

* forward: ``all_gather`` of X (each rank's senders may live anywhere), then the fused
  convolution of the local edges into the rank's Z rows;
* backward: dY and dW are local per edge; each rank's dX contributions to every sender are
  summed onto the owners with ``reduce_scatter``.

Node ranges are padded to a common size so the collectives are the fixed-size
``all_gather_into_tensor`` / ``reduce_scatter_tensor``; the local edges index that padded
global space (rank r's node v sits at row ``r * n_max + (v - lo_r)``), so the single-GPU
kernels run unchanged.  Every rank issues the same collectives in the same order.  Sums
over ranks use the backend's fixed reduction order, so deterministic mode stays reproducible
run to run.  The reference has no multi-GPU path; this follows the receiver-range plan for
its convolution (``TensorProductConv.forward``, ``_torch/TensorProductConv.py:145-200``).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Optional

import torch
import torch.distributed as dist


@dataclass
class ReceiverPartition:
    """This rank's share of a receiver-sorted graph."""

    rank: int
    world: int
    num_nodes: int
    node_lo: int                 # owned receiver nodes [node_lo, node_hi)
    node_hi: int
    n_max: int                   # padded node-range size (all ranks)
    edge_lo: int                 # owned edges [edge_lo, edge_hi) of the global edge list
    edge_hi: int
    rows: torch.Tensor           # local edges, receivers in padded global index space
    cols: torch.Tensor           # local edges, senders in padded global index space
    transpose_perm: torch.Tensor  # local edges in (sender, receiver) order

    @property
    def n_local(self) -> int:
        return self.node_hi - self.node_lo

    @staticmethod
    def build(rows: torch.Tensor, cols: torch.Tensor, num_nodes: int, world: int, rank: int
              ) -> "ReceiverPartition":
        """Partition of receiver-sorted (rows, cols); node ranges balance the edge counts."""
        rows = rows.to(torch.int64)
        cols = cols.to(torch.int64)
        E = rows.numel()
        # Node boundaries at equal edge quantiles, snapped to receiver boundaries.
        deg_cum = torch.searchsorted(rows, torch.arange(num_nodes + 1, device=rows.device))
        targets = torch.tensor([E * r // world for r in range(world + 1)], device=rows.device)
        bounds = torch.searchsorted(deg_cum, targets).clamp(max=num_nodes)
        bounds[0], bounds[-1] = 0, num_nodes
        bounds = torch.cummax(bounds, 0).values
        b = bounds.tolist()
        n_max = max(1, max(b[r + 1] - b[r] for r in range(world)))
        lo, hi = b[rank], b[rank + 1]
        e_lo, e_hi = int(deg_cum[lo]), int(deg_cum[hi])
        owner = torch.searchsorted(bounds[1:], torch.arange(num_nodes, device=rows.device),
                                   right=True)
        padded = owner * n_max + (torch.arange(num_nodes, device=rows.device) - bounds[owner])
        r_loc = padded[rows[e_lo:e_hi]]
        c_loc = padded[cols[e_lo:e_hi]]
        # Local transpose permutation: local edges in (sender, receiver) order.
        tperm = torch.argsort(c_loc * (world * n_max) + r_loc, stable=True)
        return ReceiverPartition(rank, world, num_nodes, lo, hi, n_max, e_lo, e_hi,
                                 r_loc, c_loc, tperm)


def _local_conv_ops(conv):
    """Forward / backward of the fused convolution module on padded global node arrays."""
    ops = torch.ops.libtorch_tp_jit

    def fwd(X, Y, W, part):
        perm = part.transpose_perm if conv.deterministic else conv.dummy_transpose_perm
        return ops.jit_conv_forward(conv.kernel, conv.hash, X, Y, W, conv.L3_dim, part.rows,
                                    part.cols, conv.workspace_buffer, perm)

    def bwd(X, Y, W, G, part):
        perm = part.transpose_perm if conv.deterministic else conv.dummy_transpose_perm
        return ops.jit_conv_backward(conv.kernel, conv.hash, X, Y, W, G, part.rows, part.cols,
                                     conv.workspace_buffer, perm)

    return fwd, bwd


class _PartitionedConvFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, X_local, Y, W, part, fwd, bwd, group):
        n_max, world, rank = part.n_max, part.world, part.rank
        X_pad = X_local.new_zeros(n_max, X_local.shape[1])
        X_pad[: part.n_local] = X_local
        if world == 1:
            X_full = X_pad
        else:
            X_full = X_local.new_empty(world * n_max, X_local.shape[1])
            dist.all_gather_into_tensor(X_full, X_pad, group=group)
        Z_full = fwd(X_full, Y, W, part)
        ctx.save_for_backward(X_full, Y, W)
        ctx.part, ctx.bwd, ctx.group = part, bwd, group
        return Z_full[rank * n_max: rank * n_max + part.n_local].clone()

    @staticmethod
    def backward(ctx, gZ_local):
        if torch.is_grad_enabled():
            raise RuntimeError("double backward through PartitionedConv is not supported")
        X_full, Y, W = ctx.saved_tensors
        part = ctx.part
        n_max, rank = part.n_max, part.rank
        gZ_full = gZ_local.new_zeros(part.world * n_max, gZ_local.shape[1])
        gZ_full[rank * n_max: rank * n_max + part.n_local] = gZ_local
        gX_full, gY, gW = ctx.bwd(X_full, Y, W, gZ_full, part)
        if part.world == 1:
            gX_pad = gX_full
        else:
            gX_pad = gX_full.new_empty(n_max, gX_full.shape[1])
            dist.reduce_scatter_tensor(gX_pad, gX_full.contiguous(), op=dist.ReduceOp.SUM,
                                       group=ctx.group)
        return gX_pad[: part.n_local], gY, gW, None, None, None, None


class PartitionedConv(torch.nn.Module):
    """Fused convolution of a receiver-partitioned graph (one rank per GPU).

    ``forward(X_local, Y_local, W_local)`` takes this rank's node rows of X and its edges' Y
    and W (rows ``part.edge_lo:part.edge_hi`` of the receiver-sorted edge arrays) and returns
    this rank's rows of Z.  ``conv`` is a ``TensorProductConv`` (atomic or deterministic);
    ``local_ops`` replaces its kernels with another (forward, backward) pair of the same
    signature, e.g. a CPU implementation for host-side tests.
    """

    def __init__(self, conv, part: ReceiverPartition, group=None,
                 local_ops: Optional[tuple[Callable, Callable]] = None):
        super().__init__()
        self.conv = conv
        self.part = part
        self.group = group
        self.fwd, self.bwd = local_ops if local_ops is not None else _local_conv_ops(conv)

    def forward(self, X_local, Y_local, W_local):
        return _PartitionedConvFn.apply(X_local, Y_local, W_local, self.part, self.fwd, self.bwd,
                                        self.group)
