"""Receiver-partitioned convolution on world_size 2 and 3 gloo ranks (CPU).

The host logic of ``openequivariance_b200.distributed`` (node partition, padded global
index space, all-gather of X, reduce-scatter of dX, local transpose permutation) runs as in
the multi-GPU path; the per-rank convolution is the CPU oracle instead of the CUDA kernels.
Every rank checks its rows of Z, dX and its edges' dY, dW against the single-process oracle.
"""

import os
import sys

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
sys.path.insert(0, os.path.join(os.path.dirname(HERE), "oracle"))


def _worker(rank, world, port, results):
    import tp_oracle as O

    from openequivariance_b200.distributed import PartitionedConv, ReceiverPartition
    from openequivariance_b200.graph import radius_graph

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(0)
        n = 300
        pos = torch.tensor(rng.uniform(0, 10.0, size=(n, 3)))
        rows, cols, tperm, _ = radius_graph(pos, 10.0, 2.5)
        p = O.make_problem("2x0e+2x1o", "1x0e+1x1o", "2x0e+2x1o",
                           [(0, 0, 0, "uvu", True), (1, 1, 0, "uvu", True),
                            (0, 1, 1, "uvu", True), (1, 0, 1, "uvu", True)])
        E = rows.numel()
        X = rng.normal(size=(n, 8))
        Y = rng.normal(size=(E, 4))
        W = rng.normal(size=(E, p.weight_numel))
        G = rng.normal(size=(n, 8))
        part = ReceiverPartition.build(rows, cols, n, world, rank)

        def fwd(Xf, Yl, Wl, pt):
            return torch.tensor(O.conv_forward(p, Xf.numpy(), Yl.numpy(), Wl.numpy(),
                                               pt.rows.numpy(), pt.cols.numpy()))

        def bwd(Xf, Yl, Wl, Gf, pt):
            gX, gY, gW = O.conv_backward(p, Xf.numpy(), Yl.numpy(), Wl.numpy(), Gf.numpy(),
                                         pt.rows.numpy(), pt.cols.numpy())
            return torch.tensor(gX), torch.tensor(gY), torch.tensor(gW)

        conv = PartitionedConv(None, part, local_ops=(fwd, bwd))
        lo, hi, elo, ehi = part.node_lo, part.node_hi, part.edge_lo, part.edge_hi
        x = torch.tensor(X[lo:hi], requires_grad=True)
        y = torch.tensor(Y[elo:ehi], requires_grad=True)
        w = torch.tensor(W[elo:ehi], requires_grad=True)
        z = conv(x, y, w)
        z.backward(torch.tensor(G[lo:hi]))
        Zr = O.conv_forward(p, X, Y, W, rows.numpy(), cols.numpy())
        gX, gY, gW = O.conv_backward(p, X, Y, W, G, rows.numpy(), cols.numpy())
        np.testing.assert_allclose(z.detach().numpy(), Zr[lo:hi], atol=1e-10)
        np.testing.assert_allclose(x.grad.numpy(), gX[lo:hi], atol=1e-10)
        np.testing.assert_allclose(y.grad.numpy(), gY[elo:ehi], atol=1e-10)
        np.testing.assert_allclose(w.grad.numpy(), gW[elo:ehi], atol=1e-10)
        # Ownership covers every node and edge exactly once.
        counts = torch.tensor([hi - lo, ehi - elo], dtype=torch.int64)
        dist.all_reduce(counts)
        assert counts.tolist() == [n, E]
        # The local transpose permutation orders local edges by (sender, receiver).
        key = part.cols[part.transpose_perm] * (world * part.n_max) + part.rows[part.transpose_perm]
        assert bool((key[1:] >= key[:-1]).all())
        results[rank] = 1
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_partitioned_conv_gloo(world):
    port = 29600 + world
    ctx = mp.get_context("spawn")
    results = ctx.Manager().dict()
    mp.start_processes(_worker, args=(world, port, results), nprocs=world, start_method="spawn")
    assert sorted(results.keys()) == list(range(world))
