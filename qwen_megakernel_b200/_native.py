"""Loading of the in-tree native libraries.

There is no fallback: if the libraries are missing or fail to load, every
entry point that needs them raises.  ``ops()`` returns
``torch.ops.qwen_megakernel_C`` (the reference's operator namespace,
qwen_megakernel/model.py:18); ``cdll()`` returns the C-ABI library via ctypes.
"""

from __future__ import annotations

import ctypes
import os
import threading

from .build import LIB_PATH, OPS_PATH

_lock = threading.Lock()
_ops_loaded = False
_cdll = None


class NativeLibraryMissing(RuntimeError):
    pass


def _require(path: str) -> None:
    if not os.path.exists(path):
        raise NativeLibraryMissing(
            f"qwen_megakernel_b200: native library {path} is not built; "
            "run `python -m qwen_megakernel_b200.build` (nvcc, sm_100a)"
        )


def ops():
    """Load qwen_megakernel_C.so once and return torch.ops.qwen_megakernel_C."""
    global _ops_loaded
    import torch

    with _lock:
        if not _ops_loaded:
            _require(LIB_PATH)
            _require(OPS_PATH)
            torch.ops.load_library(OPS_PATH)
            _ops_loaded = True
    return torch.ops.qwen_megakernel_C


def cdll() -> ctypes.CDLL:
    """Load libqwen_megakernel.so (C ABI) once via ctypes."""
    global _cdll
    with _lock:
        if _cdll is None:
            _require(LIB_PATH)
            lib = ctypes.CDLL(LIB_PATH)
            lib.qmk_version.restype = ctypes.c_char_p
            lib.qmk_error_string.restype = ctypes.c_char_p
            lib.qmk_error_string.argtypes = [ctypes.c_int]
            lib.qmk_get_last_error_message.restype = ctypes.c_char_p
            lib.qmk_workspace_bytes.restype = ctypes.c_size_t
            lib.qmk_attention_splits.argtypes = [ctypes.c_int, ctypes.c_int]
            lib.qmk_describe_partition.argtypes = [
                ctypes.c_int,
                ctypes.c_int,
                ctypes.c_int,
                ctypes.POINTER(ctypes.c_int),
                ctypes.c_int,
            ]
            _cdll = lib
    return _cdll


def loaded_library_paths() -> list[str]:
    """Paths of this package's native libraries mapped into the process."""
    out = []
    try:
        with open("/proc/self/maps") as f:
            for line in f:
                for p in (LIB_PATH, OPS_PATH):
                    if line.rstrip().endswith(p) and p not in out:
                        out.append(p)
    except OSError:
        pass
    return out
