"""Problem builders used by benchmarks and tests.

``channelwise_tpp`` / ``fully_connected_tpp`` construct the same instruction lists as the
reference's ``ChannelwiseTPP`` and ``FullyConnectedTPProblem``
(``benchmark/problems.py:14-33,122-170``), which follow MACE's and e3nn's conventions:

* channelwise (uvu): one ``mul x ir_out`` output block per parity-allowed
  ``(ir_in1, ir_in2, ir_out)``, outputs sorted by irrep;
* fully connected (uvw): one instruction per parity-allowed triple into the given outputs.

``baseline_problem`` returns the BASELINE configurations C1, C2 (literal reading),
C2-ml (the reference's ``mace-large``) and C4.
"""

from __future__ import annotations

import numpy as np

from .irreps import Irrep, Irreps, TPProblem


def channelwise_tpp(irreps_in1, irreps_in2, irreps_out, label=None, irrep_dtype=np.float32,
                    weight_dtype=np.float32, shared_weights=False) -> TPProblem:
    in1, in2, want = Irreps(irreps_in1), Irreps(irreps_in2), Irreps(irreps_out)
    outs, instr = [], []
    for i, (mul, ir1) in enumerate(in1):
        for j, (_, ir2) in enumerate(in2):
            for ir3 in ir1 * ir2:
                if ir3 in want:
                    instr.append((i, j, len(outs), "uvu", True))
                    outs.append((mul, ir3))
    sorted_out, perm, _ = Irreps(outs).sort()
    instr = sorted(((a, b, perm[k], m, t) for a, b, k, m, t in instr), key=lambda x: x[2])
    return TPProblem(in1, in2, sorted_out, instr, internal_weights=False,
                     shared_weights=shared_weights, label=label, irrep_dtype=irrep_dtype,
                     weight_dtype=weight_dtype)


def fully_connected_tpp(irreps_in1, irreps_in2, irreps_out, **kwargs) -> TPProblem:
    in1, in2, out = Irreps(irreps_in1), Irreps(irreps_in2), Irreps(irreps_out)
    instr = [(i, j, k, "uvw", True, 1.0)
             for i, (_, ir1) in enumerate(in1)
             for j, (_, ir2) in enumerate(in2)
             for k, (_, ir3) in enumerate(out)
             if ir3 in ir1 * ir2]
    return TPProblem(in1, in2, out, instr, **kwargs)


def baseline_problem(name: str, dtype=np.float32) -> TPProblem:
    """'c1', 'c2' (literal, 24 paths), 'c2ml' (mace-large), 'c4'."""
    if name == "c1":
        return TPProblem("1x2e", "1x3e", "1x2e", [(0, 0, 0, "uvu", True)],
                         shared_weights=False, internal_weights=False, irrep_dtype=dtype,
                         weight_dtype=dtype, label="C1")
    if name == "c2":
        return channelwise_tpp("128x0e+128x1o+128x2e", "1x0e+1x1o+1x2e+1x3o",
                               "128x0e+128x0o+128x1e+128x1o+128x2e+128x2o+128x3e+128x3o",
                               label="C2", irrep_dtype=dtype, weight_dtype=dtype)
    if name == "c2ml":
        return channelwise_tpp("128x0e+128x1o+128x2e", "1x0e+1x1o+1x2e+1x3o",
                               "128x0e+128x1o+128x2e+128x3o", label="mace-large",
                               irrep_dtype=dtype, weight_dtype=dtype)
    if name == "c4":
        ir = "32x0e+32x0o+32x1e+32x1o+32x2e+32x2o"
        return fully_connected_tpp(ir, "1x0e+1x1o+1x2e", ir, label="C4", irrep_dtype=dtype,
                                   weight_dtype=dtype)
    raise KeyError(name)


def real_spherical_harmonics(vec: np.ndarray, lmax: int) -> np.ndarray:
    """Component-normalised real spherical harmonics (e3nn ordering m=-l..l) of unit vectors.

    Built from the real Wigner 3j tables by the standard recursion
    ``Y^{l} = sqrt(...) * C^{(l-1, 1, l)} (Y^{l-1} (x) Y^{1})``; ``Y^1`` is e3nn's
    ``(y, z, x)`` ordering scaled by ``sqrt(3)``.
    """
    from .cg import real_wigner_3j

    if not isinstance(vec, np.ndarray):  # torch tensor: same recursion on its device
        import torch

        v = vec / torch.linalg.norm(vec, dim=-1, keepdim=True)
        y1 = np.sqrt(3.0) * v[..., [1, 2, 0]]
        out = [torch.ones_like(v[..., :1])] + ([y1] if lmax >= 1 else [])
        prev = y1
        for l in range(2, lmax + 1):
            c = torch.tensor(real_wigner_3j(l - 1, 1, l), dtype=v.dtype, device=v.device)
            nxt = torch.einsum("...i,...j,ijk->...k", prev, y1, c)
            nxt = nxt * (np.sqrt(2 * l + 1) / torch.linalg.norm(nxt, dim=-1, keepdim=True))
            out.append(nxt)
            prev = nxt
        return torch.cat(out, dim=-1)

    v = vec / np.linalg.norm(vec, axis=-1, keepdims=True)
    out = [np.ones(v.shape[:-1] + (1,))]
    y1 = np.sqrt(3.0) * v[..., [1, 2, 0]]
    if lmax >= 1:
        out.append(y1)
    prev = y1
    for l in range(2, lmax + 1):
        c = real_wigner_3j(l - 1, 1, l)
        nxt = np.einsum("...i,...j,ijk->...k", prev, y1, c)
        # component normalisation: |Y^l|^2 = 2l+1
        nxt *= np.sqrt(2 * l + 1) / np.linalg.norm(nxt, axis=-1, keepdims=True)
        out.append(nxt)
        prev = nxt
    return np.concatenate(out, axis=-1)
