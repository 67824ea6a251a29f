"""Loading of the native libraries that carry the whole hot path.

``libqsa_b200.so`` holds the sm_100a kernels and the C ABI
(``include/qsa_b200.h``); ``_qsa_b200_torch.so`` registers the
``torch.ops.qsa_b200`` operators over that ABI. Both are built in-tree by
``qsa-fp8-sm89_b200/build.py``. There is no fallback: when either library is
missing, every entry point raises ``QsaBuildError``.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
LIB_PATH = PKG_DIR / "libqsa_b200.so"
TORCH_EXT_PATH = PKG_DIR / "_qsa_b200_torch.so"

_lock = threading.Lock()
_clib = None
_ops_loaded = False


class QsaBuildError(RuntimeError):
    """The native qsa_b200 libraries are missing or failed to load."""


def _missing(path: Path) -> QsaBuildError:
    return QsaBuildError(
        f"{path.name} not found in {path.parent}; build it with "
        "`python qsa-fp8-sm89_b200/build.py` (there is no CPU fallback)")


def load_clib() -> ctypes.CDLL:
    """The C-ABI library, loaded once per process."""
    global _clib
    with _lock:
        if _clib is None:
            if not LIB_PATH.exists():
                raise _missing(LIB_PATH)
            _clib = ctypes.CDLL(str(LIB_PATH))
        return _clib


def load_torch_ops():
    """Registers ``torch.ops.qsa_b200`` (loads the extension once)."""
    global _ops_loaded
    import torch

    with _lock:
        if not _ops_loaded:
            if not TORCH_EXT_PATH.exists():
                raise _missing(TORCH_EXT_PATH)
            torch.ops.load_library(str(TORCH_EXT_PATH))
            _ops_loaded = True
    return torch.ops.qsa_b200
