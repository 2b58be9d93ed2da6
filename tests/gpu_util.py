"""Helpers shared by the GPU parity tests."""

import numpy as np
import torch

import tp_oracle as O

# Normalised max error bounds: fp32 1e-5, fp64 1e-12.
TOL = {np.float32: 1e-5, np.float64: 1e-12}
TORCH_DT = {np.float32: torch.float32, np.float64: torch.float64}


def to_dev(a, dtype):
    return torch.tensor(np.asarray(a), dtype=TORCH_DT[dtype], device="cuda")


def nerr(got, want):
    if isinstance(got, torch.Tensor):
        got = got.detach().double().cpu().numpy()
    return O.normalized_max_error(got, want)


def assert_close(got, want, dtype, what):
    e = nerr(got, want)
    assert e <= TOL[dtype], f"{what}: normalised max error {e:.3e} > {TOL[dtype]:.0e}"
