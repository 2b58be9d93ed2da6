"""Shared test setup.

Markers: ``gpu`` (needs a CUDA device; run with ``-m gpu``).  The oracle under ``oracle/``
is importable here as ``tp_oracle`` -- tests are one of the few places allowed to use it.
"""

import os
import sys
from pathlib import Path

import numpy as np
import pytest

# The whole GPU session runs with the synchronous device checks on (graph validation before
# every convolution launch, status read after every launch): any kernel that flags a bad
# index or an expired pipeline wait fails its test.
os.environ.setdefault("OEQB_DEVICE_CHECKS", "1")

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = Path(__file__).resolve().parent / "golden"
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "oracle"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: test needs a CUDA GPU (B200)")


def load_golden(name):
    with np.load(GOLDEN / name, allow_pickle=False) as f:
        return {k: f[k] for k in f.files}


def golden_names(prefix):
    return sorted(p.name for p in GOLDEN.glob(f"{prefix}_*.npz"))


def oracle_problem(g):
    """Builds the oracle's problem description from a golden fixture's spec."""
    import tp_oracle as O

    ins = [(int(a), int(b), int(c), str(m), True)
           for (a, b, c), m in zip(g["instructions"], g["modes"])]
    return O.make_problem(str(g["irreps_in1"]), str(g["irreps_in2"]), str(g["irreps_out"]),
                          ins, shared_weights=bool(g["shared_weights"]))


def product_problem(g, dtype=np.float64, layout="mul_ir"):
    """Builds the package's TPProblem from a golden fixture's spec."""
    from openequivariance_b200.irreps import TPProblem

    ins = [(int(a), int(b), int(c), str(m), True)
           for (a, b, c), m in zip(g["instructions"], g["modes"])]
    return TPProblem(str(g["irreps_in1"]), str(g["irreps_in2"]), str(g["irreps_out"]), ins,
                     shared_weights=bool(g["shared_weights"]), internal_weights=False,
                     irrep_dtype=dtype, weight_dtype=dtype, layout=layout)


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")
