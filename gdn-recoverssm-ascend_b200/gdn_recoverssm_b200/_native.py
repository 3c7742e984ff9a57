"""Loading of the native libraries.  There is no fallback: if the CUDA build is
missing, every op raises instead of silently running something else.

* ``ops()``  -> ``torch.ops.gdn_recoverssm_ac`` (registered by ``_C.so``)
* ``capi()`` -> ``ctypes.CDLL`` of ``libgdn_rssm_b200.so`` (the C ABI)
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import torch

_PKG = Path(__file__).resolve().parent
TORCH_LIB = _PKG / "_C.so"
CAPI_LIB = _PKG / "libgdn_rssm_b200.so"
ABI_VERSION = 1

_lock = threading.Lock()
_ops = None
_capi = None


class NativeLibraryMissing(RuntimeError):
    """The sm_100a build of this package is not present."""


def _missing(path):
    return NativeLibraryMissing(
        f"GDN RecoverSSM: native library {path.name} is not built; run "
        "`python -m gdn_recoverssm_b200.build` (nvcc, sm_100a).  There is no CPU "
        "or Triton fallback."
    )


def ops():
    """The registered torch op namespace, loading ``_C.so`` on first use."""
    global _ops
    if _ops is None:
        with _lock:
            if _ops is None:
                if not TORCH_LIB.exists():
                    raise _missing(TORCH_LIB)
                torch.ops.load_library(str(TORCH_LIB))
                ns = torch.ops.gdn_recoverssm_ac
                if int(ns.abi_version()) != ABI_VERSION:
                    raise RuntimeError("GDN RecoverSSM: native ABI version mismatch")
                _ops = ns
    return _ops


def capi():
    """The C ABI library (ctypes), loaded on first use."""
    global _capi
    if _capi is None:
        with _lock:
            if _capi is None:
                if not CAPI_LIB.exists():
                    raise _missing(CAPI_LIB)
                _capi = ctypes.CDLL(str(CAPI_LIB))
    return _capi


def loaded_libraries():
    """Paths of the native libraries this process has loaded so far."""
    out = []
    if _ops is not None:
        out.append(str(TORCH_LIB))
    if _capi is not None or _ops is not None:
        out.append(str(CAPI_LIB))
    return out
