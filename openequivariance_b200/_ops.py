"""torch.library metadata for the ``libtorch_tp_jit`` operators: fake kernels (for
``torch.compile``/``export``), autograd formulas and autocast-to-fp32.

The operator schemas are the reference's (``extension/torch_core.hpp:710-722``) so its
registration pattern (``_torch/TensorProduct.py:184-376``,
``_torch/TensorProductConv.py:285-581``) carries over.  Gradients rely on the ops being
trilinear in ``(X, Y, W)``:

* ``forward(X,Y,W) = f(X,Y,W)``;
* ``backward(X,Y,W,G) = (bX(Y,W,G), bY(X,W,G), bW(X,Y,G))`` are the adjoints of ``f``
  in each argument;
* ``double_backward(X,Y,W,G,a,b,c)`` returns
  ``(bX(b,W,G)+bX(Y,c,G), bY(a,W,G)+bY(X,c,G), bW(a,Y,G)+bW(X,b,G),
  f(a,Y,W)+f(X,b,W)+f(X,Y,c))``.

The triple backward below is derived from those identities (7 operator calls); it is
not the reference's composition but yields the same gradients.
"""

from __future__ import annotations

import torch

_registered = False


def _zeros_if_none(t, like):
    return torch.zeros_like(like) if t is None else t


def _tp_ops():
    ops = torch.ops.libtorch_tp_jit
    return ops.jit_tp_forward, ops.jit_tp_backward, ops.jit_tp_double_backward


def _register_tp():
    lib = "libtorch_tp_jit"
    _, bwd_op, dbl_op = _tp_ops()

    @torch.library.register_fake(f"{lib}::jit_tp_forward")
    def _fake_fwd(kernel, hash, L1_in, L2_in, W, L3_dim):
        return L1_in.new_empty(L1_in.shape[0], L3_dim)

    @torch.library.register_fake(f"{lib}::jit_tp_backward")
    def _fake_bwd(kernel, hash, L1_in, L2_in, W, L3_grad):
        return torch.empty_like(L1_in), torch.empty_like(L2_in), torch.empty_like(W)

    @torch.library.register_fake(f"{lib}::jit_tp_double_backward")
    def _fake_dbl(kernel, hash, L1_in, L2_in, W, L3_grad, E, F, G):
        return (torch.empty_like(L1_in), torch.empty_like(L2_in), torch.empty_like(W),
                torch.empty_like(L3_grad))

    def setup_fwd(ctx, inputs, output):
        ctx.kernel, ctx.hash, ctx.X, ctx.Y, ctx.W, _ = inputs

    def grad_fwd(ctx, gZ):
        gX, gY, gW = bwd_op(ctx.kernel, ctx.hash, ctx.X, ctx.Y, ctx.W, gZ)
        return None, None, gX, gY, gW, None

    torch.library.register_autograd(f"{lib}::jit_tp_forward", grad_fwd, setup_context=setup_fwd)

    def setup_bwd(ctx, inputs, output):
        ctx.kernel, ctx.hash, ctx.X, ctx.Y, ctx.W, ctx.G = inputs

    def grad_bwd(ctx, a, b, c):
        a = _zeros_if_none(a, ctx.X)
        b = _zeros_if_none(b, ctx.Y)
        c = _zeros_if_none(c, ctx.W)
        gX, gY, gW, gG = dbl_op(ctx.kernel, ctx.hash, ctx.X, ctx.Y, ctx.W, ctx.G, a, b, c)
        return None, None, gX, gY, gW, gG

    torch.library.register_autograd(f"{lib}::jit_tp_backward", grad_bwd, setup_context=setup_bwd)

    def setup_dbl(ctx, inputs, output):
        (ctx.kernel, ctx.hash, ctx.X, ctx.Y, ctx.W, ctx.G, ctx.a, ctx.b, ctx.c) = inputs

    def grad_dbl(ctx, tX, tY, tW, tG):
        k, h = ctx.kernel, ctx.hash
        X, Y, W, G, a, b, c = ctx.X, ctx.Y, ctx.W, ctx.G, ctx.a, ctx.b, ctx.c
        return (None, None) + _triple(
            lambda *args: bwd_op(k, h, *args), lambda *args: dbl_op(k, h, *args),
            X, Y, W, G, a, b, c, tX, tY, tW, tG, ())

    torch.library.register_autograd(f"{lib}::jit_tp_double_backward", grad_dbl,
                                    setup_context=setup_dbl)


def _triple(bwd, dbl, X, Y, W, G, a, b, c, tX, tY, tW, tG, extra):
    """Gradients of double_backward w.r.t. (X, Y, W, G, a, b, c) for cotangents t*."""
    tX = _zeros_if_none(tX, X)
    tY = _zeros_if_none(tY, Y)
    tW = _zeros_if_none(tW, W)
    tG = _zeros_if_none(tG, G)
    zc = torch.zeros_like(c)
    # d/d(a,b,c): adjoints with cotangent tG, plus the G-terms carrying tX, tY, tW.
    ga1, gb1, gc1 = bwd(X, Y, W, tG, *extra)
    ga2, gb2, gc2, _ = dbl(X, Y, W, G, tX, tY, tW, *extra)
    # d/d(X,Y,W): the double-backward terms with cotangent tG, plus the cross terms.
    gX1, gY1, gW1, _ = dbl(X, Y, W, tG, a, b, c, *extra)
    gX2, gY2, gW2, _ = dbl(tX, tY, tW, G, a, b, c, *extra)
    # d/dG: f(tX,b,W)+f(a,tY,W) + f(tX,Y,c)+f(X,tY,c) + f(a,Y,tW)+f(X,b,tW).
    _, _, _, gG1 = dbl(a, b, W, G, tX, tY, zc, *extra)
    _, _, _, gG2 = dbl(X, Y, c, G, tX, tY, zc, *extra)
    _, _, _, gG3 = dbl(X, Y, tW, G, a, b, zc, *extra)
    return (gX1 + gX2, gY1 + gY2, gW1 + gW2, gG1 + gG2 + gG3, ga1 + ga2, gb1 + gb2, gc1 + gc2)


def _register_conv():
    lib = "libtorch_tp_jit"
    ops = torch.ops.libtorch_tp_jit
    bwd_op, dbl_op = ops.jit_conv_backward, ops.jit_conv_double_backward

    @torch.library.register_fake(f"{lib}::jit_conv_forward")
    def _fake_fwd(kernel, hash, L1_in, L2_in, W, L3_dim, rows, cols, workspace, perm):
        return L1_in.new_empty(L1_in.shape[0], L3_dim)

    @torch.library.register_fake(f"{lib}::jit_conv_backward")
    def _fake_bwd(kernel, hash, L1_in, L2_in, W, L3_grad, rows, cols, workspace, perm):
        return torch.empty_like(L1_in), torch.empty_like(L2_in), torch.empty_like(W)

    @torch.library.register_fake(f"{lib}::jit_conv_double_backward")
    def _fake_dbl(kernel, hash, L1_in, L2_in, W, L3_grad, E, F, G, rows, cols, workspace,
                  perm):
        return (torch.empty_like(L1_in), torch.empty_like(L2_in), torch.empty_like(W),
                torch.empty_like(L3_grad))

    def setup_fwd(ctx, inputs, output):
        (ctx.kernel, ctx.hash, ctx.X, ctx.Y, ctx.W, _, ctx.rows, ctx.cols, ctx.ws,
         ctx.perm) = inputs

    def grad_fwd(ctx, gZ):
        gX, gY, gW = bwd_op(ctx.kernel, ctx.hash, ctx.X, ctx.Y, ctx.W, gZ, ctx.rows, ctx.cols,
                            ctx.ws, ctx.perm)
        return None, None, gX, gY, gW, None, None, None, None, None

    torch.library.register_autograd(f"{lib}::jit_conv_forward", grad_fwd,
                                    setup_context=setup_fwd)

    def setup_bwd(ctx, inputs, output):
        (ctx.kernel, ctx.hash, ctx.X, ctx.Y, ctx.W, ctx.G, ctx.rows, ctx.cols, ctx.ws,
         ctx.perm) = inputs

    def grad_bwd(ctx, a, b, c):
        a = _zeros_if_none(a, ctx.X)
        b = _zeros_if_none(b, ctx.Y)
        c = _zeros_if_none(c, ctx.W)
        gX, gY, gW, gG = dbl_op(ctx.kernel, ctx.hash, ctx.X, ctx.Y, ctx.W, ctx.G, a, b, c,
                                ctx.rows, ctx.cols, ctx.ws, ctx.perm)
        return None, None, gX, gY, gW, gG, None, None, None, None

    torch.library.register_autograd(f"{lib}::jit_conv_backward", grad_bwd,
                                    setup_context=setup_bwd)

    def setup_dbl(ctx, inputs, output):
        (ctx.kernel, ctx.hash, ctx.X, ctx.Y, ctx.W, ctx.G, ctx.a, ctx.b, ctx.c, ctx.rows,
         ctx.cols, ctx.ws, ctx.perm) = inputs

    def grad_dbl(ctx, tX, tY, tW, tG):
        k, h = ctx.kernel, ctx.hash
        extra = (ctx.rows, ctx.cols, ctx.ws, ctx.perm)
        grads = _triple(lambda *args: bwd_op(k, h, *args), lambda *args: dbl_op(k, h, *args),
                        ctx.X, ctx.Y, ctx.W, ctx.G, ctx.a, ctx.b, ctx.c, tX, tY, tW, tG, extra)
        return (None, None) + grads + (None, None, None, None)

    torch.library.register_autograd(f"{lib}::jit_conv_double_backward", grad_dbl,
                                    setup_context=setup_dbl)


def _register_sc():
    """group_gemm (reference schema, ``SymmetricContraction.py:339-414`` formulas) and the
    fused contraction ops' fake kernels."""
    lib = "libtorch_tp_jit"
    op = torch.ops.libtorch_tp_jit.group_gemm

    @torch.library.register_fake(f"{lib}::group_gemm")
    def _fake_gg(A, B, ragged_counts, num_W, batch_size, m, k, ragged_inner):
        if ragged_inner == 0:
            return A.new_empty(B.shape[0], batch_size, m)
        return A.new_empty(num_W, batch_size, m, k)

    def setup_gg(ctx, inputs, output):
        ctx.A, ctx.B, ctx.counts, ctx.num_W, ctx.batch, ctx.m, ctx.k, ctx.inner = inputs

    def grad_gg(ctx, g):
        # ragged_inner == 0: C = A B  -> dA = sum_r g (x) B (inner form), dB = A^T g.
        # ragged_inner == 1: C = sum_r A (x) B -> dA = C-shaped g applied to B, dB = g^T A.
        if ctx.inner == 0:
            gA = op(g, ctx.B, ctx.counts, ctx.num_W, ctx.batch, ctx.m, ctx.k, 1)
            gB = op(ctx.A.transpose(2, 3), g, ctx.counts, ctx.num_W, ctx.batch, ctx.k, ctx.m, 0)
        else:
            gA = op(g, ctx.B, ctx.counts, ctx.num_W, ctx.batch, ctx.m, ctx.k, 0)
            gB = op(g.transpose(2, 3), ctx.A, ctx.counts, ctx.num_W, ctx.batch, ctx.k, ctx.m, 0)
        return gA, gB, None, None, None, None, None, None

    torch.library.register_autograd(f"{lib}::group_gemm", grad_gg, setup_context=setup_gg)

    @torch.library.register_fake("oeqb200::sc_forward")
    def _fake_scf(x, perm, elem_offsets, coef, out_col, out_step, out_dim, degree):
        return x.new_empty(x.shape[0], out_dim)

    @torch.library.register_fake("oeqb200::sc_backward")
    def _fake_scb(x, perm, elem_offsets, coef, grad_out, out_col, out_step, degree):
        return torch.empty_like(x), torch.empty_like(coef)

    @torch.library.register_fake("oeqb200::conv_backward_into")
    def _fake_cbi(kernel, hash, L1_in, L2_in, W, L3_grad, rows, cols, workspace, perm,
                  L1_grad, L2_grad, W_grad):
        return None


def _register_autocast():
    for name in ("jit_tp_forward", "jit_tp_backward", "jit_tp_double_backward",
                 "jit_conv_forward", "jit_conv_backward", "jit_conv_double_backward"):
        torch.library.register_autocast(f"libtorch_tp_jit::{name}", "cuda", torch.float32)


def ensure_registered() -> None:
    """Loads the native operators and attaches fakes/autograd/autocast (idempotent)."""
    global _registered
    if _registered:
        return
    from . import _ext

    _ext.load_torch_ops()
    _register_tp()
    _register_conv()
    _register_sc()
    _register_autocast()
    _registered = True
