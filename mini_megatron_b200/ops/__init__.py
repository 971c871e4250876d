"""Access to the sm_100a kernels (``mini_megatron_b200._C``).

The extension is built in-tree (``python setup.py build_ext --inplace``).  On a
machine with a CUDA device the native path is mandatory: if the extension is
missing, :func:`native` raises instead of silently falling back to PyTorch.
CPU tensors never reach these kernels; the PyTorch code paths in the model
modules are the CPU oracle used by the unit tests.
"""
from __future__ import annotations

import importlib
import os

_C = None
_IMPORT_ERROR = None


def native():
    """Return the compiled extension module or raise with a build hint."""
    global _C, _IMPORT_ERROR
    if _C is None:
        try:
            _C = importlib.import_module("mini_megatron_b200._C")
            if os.environ.get("MMB_CRASH_TRACE") == "1":
                _C.install_crash_handler()
        except ImportError as exc:  # pragma: no cover - exercised only without a build
            _IMPORT_ERROR = exc
            raise RuntimeError(
                "mini_megatron_b200._C is not built; run `python setup.py build_ext --inplace` "
                f"(sm_100a). Import error: {exc}") from exc
    return _C


def available() -> bool:
    try:
        native()
        return True
    except RuntimeError:
        return False


def check_errors():
    """Raise if any kernel recorded a bounded-wait timeout since the last clear."""
    C = native()
    code = C.get_error()
    if code:
        C.clear_error()
        raise RuntimeError(f"device kernel reported error code {code} (bounded wait timed out)")
