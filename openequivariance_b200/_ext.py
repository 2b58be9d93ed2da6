"""Loader for the native libraries.

There is no CPU fallback: if ``liboeqb200.so`` or ``libtorch_oeqb200.so`` is missing the
import of an operator fails with an explicit error (build them with
``python -c "import openequivariance_b200._build as b; b.build()"``).
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "liboeqb200.so"
TORCH_LIB_PATH = PKG / "libtorch_oeqb200.so"

_lock = threading.Lock()
_cabi = None
_torch_loaded = False


class ExtensionMissing(RuntimeError):
    pass


def cabi() -> ctypes.CDLL:
    """The C-ABI library (``include/oeqb200.h``)."""
    global _cabi
    with _lock:
        if _cabi is None:
            if not LIB_PATH.exists():
                raise ExtensionMissing(
                    f"{LIB_PATH} is missing: the CUDA extension has not been built "
                    "(run openequivariance_b200._build.build())"
                )
            lib = ctypes.CDLL(str(LIB_PATH))
            lib.oeqb_last_error.restype = ctypes.c_char_p
            lib.oeqb_version.restype = ctypes.c_char_p
            lib.oeqb_conv_workspace_bytes.restype = ctypes.c_size_t
            _cabi = lib
    return _cabi


def load_torch_ops() -> None:
    """Registers the ``torch.ops.libtorch_tp_jit.*`` operators (idempotent)."""
    global _torch_loaded
    with _lock:
        if _torch_loaded:
            return
        if not TORCH_LIB_PATH.exists():
            raise ExtensionMissing(
                f"{TORCH_LIB_PATH} is missing: the torch operator shim has not been built "
                "(run openequivariance_b200._build.build())"
            )
        import torch

        torch.ops.load_library(str(TORCH_LIB_PATH))
        _torch_loaded = True


def loaded_native_libraries():
    """Paths of this package's native libraries mapped into the process."""
    out = []
    try:
        with open("/proc/self/maps") as f:
            for line in f:
                if str(PKG) in line and line.rstrip().endswith(".so"):
                    path = line.split()[-1]
                    if path not in out:
                        out.append(path)
    except OSError:
        pass
    return out
