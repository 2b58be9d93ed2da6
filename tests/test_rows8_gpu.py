"""The padded-row convolution entry points (``oeqb_conv_forward_rows8`` /
``oeqb_conv_backward_rows8``) that the multi-GPU partition runs on, checked on one GPU.

The edge list is split into two receiver-sorted blocks as the partition splits interior and
boundary edges (the second block starting at a multiple of 4 edges); the forward of the second
block accumulates into the first block's output, and both backward blocks add into one padded
dX accumulator.  The results must equal the single-call module and the fp64 oracle.  The
partitioned module itself is also run with one rank (no exchange).
"""

import numpy as np
import pytest
import torch

import tp_oracle as O

pytestmark = pytest.mark.gpu


def _setup(seed=0, n=400, box=12.0, cutoff=3.0):
    import openequivariance_b200 as oeq
    from openequivariance_b200.graph import morton_order, radius_graph

    g = torch.Generator().manual_seed(seed)
    pos = (torch.rand(n, 3, generator=g, dtype=torch.float64) * box).cuda()
    pos = pos[morton_order(pos, box)]
    rows, cols, tperm, _ = radius_graph(pos, box, cutoff)
    prob = oeq.TPProblem("1x2e", "1x3e", "1x2e", [(0, 0, 0, "uvu", True)],
                         shared_weights=False, internal_weights=False)
    conv = oeq.TensorProductConv(prob)
    E = rows.numel()
    gen = torch.Generator(device="cuda").manual_seed(seed + 1)
    X = torch.randn(n, 5, device="cuda", generator=gen)
    Y = torch.randn(E, 7, device="cuda", generator=gen)
    W = torch.randn(E, 1, device="cuda", generator=gen)
    G = torch.randn(n, 5, device="cuda", generator=gen)
    return conv, prob, rows, cols, X, Y, W, G


def _nerr(a, b):
    return float((a.double() - b.double()).abs().max() / b.double().abs().max().clamp_min(1e-30))


def test_rows8_blocks_match_module(cuda_device):
    conv, prob, rows, cols, X, Y, W, G = _setup()
    ops = torch.ops.oeqb200
    assert ops.conv_rows8_ok(conv.kernel, conv.hash, 0)
    n, E = X.shape[0], rows.numel()
    cut = (E // 2) & ~3
    xp = torch.zeros(n, 8, device="cuda")
    xp[:, :5] = X
    gp = torch.zeros(n, 8, device="cuda")
    gp[:, :5] = G
    Z = torch.empty(n, 5, device="cuda")
    # sm_budget: -16 = all SMs but 16, 8 = at most 8 SMs, 0 = all.
    ops.conv_forward_rows8(conv.kernel, conv.hash, xp, Y[:cut], W[:cut], Z, rows[:cut].contiguous(),
                           cols[:cut].contiguous(), False, -16)
    ops.conv_forward_rows8(conv.kernel, conv.hash, xp, Y[cut:], W[cut:], Z, rows[cut:].contiguous(),
                           cols[cut:].contiguous(), True, 8)
    x, y, w = (t.clone().requires_grad_() for t in (X, Y, W))
    z = conv(x, y, w, rows, cols)
    z.backward(G)
    assert _nerr(Z, z.detach()) <= 1e-5
    dY, dW = torch.empty_like(Y), torch.empty_like(W)
    dxp = torch.zeros(n, 8, device="cuda")
    ops.conv_backward_rows8(conv.kernel, conv.hash, xp, gp, Y[cut:], W[cut:], dY[cut:], dW[cut:],
                            dxp, rows[cut:].contiguous(), cols[cut:].contiguous(), 8)
    ops.conv_backward_rows8(conv.kernel, conv.hash, xp, gp, Y[:cut], W[:cut], dY[:cut], dW[:cut],
                            dxp, rows[:cut].contiguous(), cols[:cut].contiguous(), -16)
    assert _nerr(dxp[:, :5], x.grad) <= 1e-5
    assert _nerr(dY, y.grad) <= 1e-5
    assert _nerr(dW, w.grad) <= 1e-5
    # And the oracle (fp64).
    p = O.make_problem("1x2e", "1x3e", "1x2e", [(0, 0, 0, "uvu", True)])
    r, c = rows.cpu().numpy(), cols.cpu().numpy()
    A = [t.double().cpu().numpy() for t in (X, Y, W, G)]
    assert O.normalized_max_error(Z.double().cpu().numpy(), O.conv_forward(p, *A[:3], r, c)) <= 1e-5
    gx, gy, gw = O.conv_backward(p, *A, r, c)
    assert O.normalized_max_error(dxp[:, :5].double().cpu().numpy(), gx) <= 1e-5


def test_rows8_refuses_other_plans(cuda_device):
    import openequivariance_b200 as oeq

    prob = oeq.TPProblem("2x0e+2x1o", "1x0e+1x1o", "2x0e+2x1o",
                         [(0, 0, 0, "uvu", True), (1, 1, 0, "uvu", True)],
                         shared_weights=False, internal_weights=False)
    det = oeq.TensorProductConv(_setup()[1], deterministic=True)
    multi = oeq.TensorProductConv(prob)
    assert not torch.ops.oeqb200.conv_rows8_ok(det.kernel, det.hash, 0)
    assert not torch.ops.oeqb200.conv_rows8_ok(multi.kernel, multi.hash, 0)


def test_partitioned_conv_one_rank_padded_path(cuda_device):
    from openequivariance_b200.distributed import PartitionedConv, ReceiverPartition

    conv, prob, rows, cols, X, Y, W, G = _setup(seed=3)
    n = X.shape[0]
    part = ReceiverPartition.build(rows, cols, n, 1, 0)
    pc = PartitionedConv(conv, part)
    ei = part.edge_index
    x, y, w = X.clone().requires_grad_(), Y[ei].clone().requires_grad_(), W[ei].clone().requires_grad_()
    z = pc(x, y, w)
    assert pc._rows8
    z.backward(G)
    xr, yr, wr = (t.clone().requires_grad_() for t in (X, Y, W))
    zr = conv(xr, yr, wr, rows, cols)
    zr.backward(G)
    assert _nerr(z.detach(), zr.detach()) <= 1e-5
    assert _nerr(x.grad, xr.grad) <= 1e-5
    assert _nerr(y.grad, yr.grad[ei]) <= 1e-5
    assert _nerr(w.grad, wr.grad[ei]) <= 1e-5
