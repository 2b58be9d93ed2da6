"""Receiver-partitioned convolution with halo exchange on world_size 2 and 3 gloo ranks (CPU).

The host logic of ``openequivariance_b200.distributed`` (node ranges, halo lists, local node
space, interior / boundary edge blocks, the two ``all_to_all_single`` exchanges and the
rank-ordered halo sums) runs as in the multi-GPU path; the per-rank convolution is the CPU
oracle instead of the CUDA kernels.  Every rank checks its rows of Z, dX and its edges' dY, dW
against the single-process oracle.

A second test injects a failure on the host: one rank never enters the exchange, and the
others must leave it with an error once the process group's timeout expires, not hang.
"""

import datetime
import os
import sys
import time

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
sys.path.insert(0, os.path.join(os.path.dirname(HERE), "oracle"))

PROBLEM = ("2x0e+2x1o", "1x0e+1x1o", "2x0e+2x1o",
           [(0, 0, 0, "uvu", True), (1, 1, 0, "uvu", True), (0, 1, 1, "uvu", True),
            (1, 0, 1, "uvu", True)])


def _oracle_ops(p):
    import tp_oracle as O

    def fwd(X, Y, W, rows, cols, tperm):
        return torch.tensor(O.conv_forward(p, X.numpy(), Y.numpy(), W.numpy(), rows.numpy(),
                                           cols.numpy()))

    def bwd(X, Y, W, G, rows, cols, tperm, gX, gY, gW):
        a, b, c = O.conv_backward(p, X.numpy(), Y.numpy(), W.numpy(), G.numpy(), rows.numpy(),
                                  cols.numpy())
        gX.copy_(torch.tensor(a))
        gY.copy_(torch.tensor(b))
        gW.copy_(torch.tensor(c))

    return fwd, bwd


def _graph(n=300, box=10.0, cutoff=2.5, spatial=True):
    from openequivariance_b200.graph import morton_order, radius_graph

    rng = np.random.default_rng(0)
    pos = torch.tensor(rng.uniform(0, box, size=(n, 3)))
    if spatial:
        pos = pos[morton_order(pos, box)]
    rows, cols, tperm, _ = radius_graph(pos, box, cutoff)
    return rows, cols


def _worker(rank, world, port, results, spatial, det):
    import tp_oracle as O

    from openequivariance_b200.distributed import PartitionedConv, ReceiverPartition

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        n = 300
        rows, cols = _graph(n, spatial=spatial)
        p = O.make_problem(*PROBLEM)
        rng = np.random.default_rng(0)
        E = rows.numel()
        X = rng.normal(size=(n, 8))
        Y = rng.normal(size=(E, 4))
        W = rng.normal(size=(E, p.weight_numel))
        G = rng.normal(size=(n, 8))
        part = ReceiverPartition.build(rows, cols, n, world, rank)
        conv = PartitionedConv(None, part, local_ops=_oracle_ops(p), shared_weights=False,
                               deterministic=det)
        lo, hi = part.node_lo, part.node_hi
        ei = part.edge_index.numpy()
        x = torch.tensor(X[lo:hi], requires_grad=True)
        y = torch.tensor(Y[ei], requires_grad=True)
        w = torch.tensor(W[ei], requires_grad=True)
        z = conv(x, y, w)
        z.backward(torch.tensor(G[lo:hi]))
        Zr = O.conv_forward(p, X, Y, W, rows.numpy(), cols.numpy())
        gX, gY, gW = O.conv_backward(p, X, Y, W, G, rows.numpy(), cols.numpy())
        np.testing.assert_allclose(z.detach().numpy(), Zr[lo:hi], atol=1e-10)
        np.testing.assert_allclose(x.grad.numpy(), gX[lo:hi], atol=1e-10)
        np.testing.assert_allclose(y.grad.numpy(), gY[ei], atol=1e-10)
        np.testing.assert_allclose(w.grad.numpy(), gW[ei], atol=1e-10)
        # Ownership covers every node and edge exactly once.
        counts = torch.tensor([hi - lo, part.n_edges], dtype=torch.int64)
        dist.all_reduce(counts)
        assert counts.tolist() == [n, E]
        # Blocks: receiver-sorted, the boundary block starts at a multiple of 4 edges, its
        # senders are the halo (plus at most 3 local ones), and each transpose permutation
        # orders its block by (sender, receiver).
        assert part.n_interior % 4 == 0
        for r_, c_, t_ in ((part.rows_int, part.cols_int, part.tperm_int),
                           (part.rows_bnd, part.cols_bnd, part.tperm_bnd)):
            assert bool((r_[1:] >= r_[:-1]).all())
            key = c_[t_] * part.n_local_nodes + r_[t_]
            assert bool((key[1:] >= key[:-1]).all())
        assert int((part.cols_bnd < part.n_own).sum()) <= 3
        assert bool((part.cols_int < part.n_own).all())
        results[rank] = (part.n_halo, part.n_own)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("det", [False, True], ids=["atomic", "deterministic"])
@pytest.mark.parametrize("world", [2, 3])
def test_partitioned_conv_gloo(world, det):
    port = 29600 + 2 * world + det
    ctx = mp.get_context("spawn")
    results = ctx.Manager().dict()
    mp.start_processes(_worker, args=(world, port, results, True, det), nprocs=world,
                       start_method="spawn")
    assert sorted(results.keys()) == list(range(world))


def test_spatial_order_shrinks_halos():
    """Morton numbering makes receiver ranges compact: far fewer halo nodes than with the
    random numbering of the same graph (the exchange volume of every pass)."""
    from openequivariance_b200.distributed import ReceiverPartition

    n, world = 2000, 4
    halos = {}
    for spatial in (False, True):
        rows, cols = _graph(n, box=20.0, cutoff=2.5, spatial=spatial)
        halos[spatial] = sum(ReceiverPartition.build(rows, cols, n, world, r).n_halo
                             for r in range(world))
    assert halos[True] < 0.5 * halos[False], halos


def _stalled_worker(rank, world, port, results):
    """Rank 1 never joins the exchange; rank 0 must get an error within the group timeout."""
    import tp_oracle as O

    from openequivariance_b200.distributed import PartitionedConv, ReceiverPartition

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=3))
    try:
        rows, cols = _graph(200)
        p = O.make_problem(*PROBLEM)
        part = ReceiverPartition.build(rows, cols, 200, world, rank)
        if rank == 1:
            # Stays alive without entering the collective until rank 0 has reported.
            deadline = time.time() + 60
            while 0 not in results and time.time() < deadline:
                time.sleep(0.1)
            results[1] = "idle"
            return
        conv = PartitionedConv(None, part, local_ops=_oracle_ops(p), shared_weights=False,
                               deterministic=False)
        rng = np.random.default_rng(0)
        x = torch.tensor(rng.normal(size=(part.n_own, 8)))
        y = torch.tensor(rng.normal(size=(part.n_edges, 4)))
        w = torch.tensor(rng.normal(size=(part.n_edges, p.weight_numel)))
        t0 = time.time()
        try:
            conv(x, y, w)
            results[0] = "no error"
        except RuntimeError as e:
            results[0] = ("error", time.time() - t0, str(e)[:200])
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def test_missing_rank_times_out_instead_of_hanging():
    port = 29650
    ctx = mp.get_context("spawn")
    results = ctx.Manager().dict()
    mp.start_processes(_stalled_worker, args=(2, port, results), nprocs=2, start_method="spawn")
    got = results.get(0)
    assert isinstance(got, tuple) and got[0] == "error", got
    assert got[1] < 30, got
    assert results.get(1) == "idle"
