"""The symmetric-contraction oracle against fixtures generated from the reference module."""

import glob
import os
import sys

import numpy as np
import pytest
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(os.path.dirname(HERE), "oracle"))
import sc_oracle as SO  # noqa: E402

FIXTURES = sorted(glob.glob(os.path.join(HERE, "golden", "sc_*.npz")))


def _load(path):
    d = np.load(path)
    corr, ne = (int(v) for v in d["meta"])
    prob = SO.ScProblem(str(d["irreps_in"]), str(d["irreps_out"]), corr, ne)
    weights = []
    for ci in range(len(prob.outs)):
        w = [torch.tensor(d[f"c{ci}_weights_max"])]
        w += [torch.tensor(d[f"c{ci}_weights_{i}"]) for i in range(corr - 1)]
        weights.append(w)
    return d, prob, weights


@pytest.mark.parametrize("path", FIXTURES, ids=[os.path.basename(p)[3:-4] for p in FIXTURES])
def test_u_matrices(path):
    d, prob, _ = _load(path)
    for ci, U in enumerate(prob.U):
        for nu, u in U.items():
            ref = d[f"c{ci}_U{nu}"]
            assert u.shape == ref.shape, (ci, nu)
            np.testing.assert_allclose(u, ref, atol=1e-12, rtol=0)


@pytest.mark.parametrize("path", FIXTURES, ids=[os.path.basename(p)[3:-4] for p in FIXTURES])
def test_forward_and_gradients(path):
    d, prob, weights = _load(path)
    x = torch.tensor(d["x"], requires_grad=True)
    for w in weights:
        for t in w:
            t.requires_grad_(True)
    elem = torch.tensor(d["labels"])
    out = SO.forward(prob, weights, x, elem)
    np.testing.assert_allclose(out.detach().numpy(), d["out"], atol=1e-12, rtol=1e-12)
    flat = [t for w in weights for t in w]
    grads = torch.autograd.grad((out * torch.tensor(d["grad_out"])).sum(), [x] + flat)
    np.testing.assert_allclose(grads[0].numpy(), d["grad_x"], atol=1e-11, rtol=1e-11)
    gi = 1
    for ci in range(len(prob.outs)):
        np.testing.assert_allclose(grads[gi].numpy(), d[f"c{ci}_grad_weights_max"], atol=1e-11)
        gi += 1
        for i in range(prob.correlation - 1):
            np.testing.assert_allclose(grads[gi].numpy(), d[f"c{ci}_grad_weights_{i}"], atol=1e-11)
            gi += 1
