"""Receiver-partitioned convolution with NCCL halo exchange on 2, 4 and 8 GPUs.

Skipped when fewer GPUs are visible.  Each rank runs the partitioned forward and backward of a
Morton-numbered radius graph and compares its rows with a single-GPU TensorProductConv run of
the whole graph (same seeded inputs), at the normalised 1e-5 bound.  Deterministic mode is also
checked for bitwise run-to-run reproducibility.  NVLS is off (``NCCL_NVLS_ENABLE=0``): the
exchange is point-to-point.
"""

import os
import sys

import pytest
import torch
import torch.multiprocessing as mp

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))


def _worker(rank, world, port, mode, results):
    import datetime

    import torch.distributed as dist

    import openequivariance_b200 as oeq
    from openequivariance_b200.distributed import PartitionedConv, ReceiverPartition
    from openequivariance_b200.graph import morton_order, radius_graph
    from openequivariance_b200.problems import real_spherical_harmonics

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        dev = torch.device("cuda", rank)
        g = torch.Generator().manual_seed(0)
        n, box = 3000, 20.0
        pos = (torch.rand(n, 3, generator=g, dtype=torch.float64) * box).to(dev)
        pos = pos[morton_order(pos, box)]
        rows, cols, tperm, vec = radius_graph(pos, box, 4.0)
        E = rows.numel()
        prob = oeq.TPProblem("4x0e+4x1o", "1x0e+1x1o", "4x0e+4x1o",
                             [(0, 0, 0, "uvu", True), (1, 1, 0, "uvu", True),
                              (0, 1, 1, "uvu", True), (1, 0, 1, "uvu", True)],
                             shared_weights=False, internal_weights=False)
        det = mode == "deterministic"
        conv = oeq.TensorProductConv(prob, deterministic=det)
        X = torch.randn(n, 16, generator=g).to(dev)
        Y = real_spherical_harmonics(vec, 1).float()
        W = torch.randn(E, prob.weight_numel, generator=g).to(dev)
        G = torch.randn(n, 16, generator=g).to(dev)
        # Single-GPU reference on the whole graph.
        xr, yr, wr = (t.clone().requires_grad_() for t in (X, Y, W))
        zr = conv(xr, yr, wr, rows, cols, tperm if det else None)
        zr.backward(G)
        part = ReceiverPartition.build(rows, cols, n, world, rank)
        pc = PartitionedConv(conv, part)
        lo, hi, ei = part.node_lo, part.node_hi, part.edge_index
        assert world == 1 or part.n_halo < 0.9 * n
        outs = []
        for _ in range(2):
            x = X[lo:hi].clone().requires_grad_()
            y = Y[ei].clone().requires_grad_()
            w = W[ei].clone().requires_grad_()
            z = pc(x, y, w)
            gx, gy, gw = torch.autograd.grad(z, (x, y, w), G[lo:hi])
            outs.append((z, gx, gy, gw))
        z, gx, gy, gw = outs[0]
        def nerr(a, b):
            return float((a - b).abs().max() / b.abs().max().clamp_min(1e-30))

        for what, a, b in (("Z", z, zr[lo:hi]), ("dX", gx, xr.grad[lo:hi]),
                           ("dY", gy, yr.grad[ei]), ("dW", gw, wr.grad[ei])):
            e = nerr(a, b)
            assert e <= 1e-5, f"rank {rank} {what}: normalised max error {e:.3e}"
        if det:
            for a, b in zip(outs[0], outs[1]):
                assert torch.equal(a, b)
        results[rank] = 1
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("mode", ["atomic", "deterministic"])
def test_partitioned_conv_nccl(mode, world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    results = ctx.Manager().dict()
    port = 29700 + 2 * world + (mode == "deterministic")
    mp.start_processes(_worker, args=(world, port, mode, results), nprocs=world,
                       start_method="spawn")
    assert sorted(results.keys()) == list(range(world))
