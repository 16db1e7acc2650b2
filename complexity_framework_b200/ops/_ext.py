"""Loader of the in-tree sm_100a extension ``complexity_framework_b200._C``.

The extension is built in place (``python setup.py build_ext --inplace``).
On a machine with a CUDA device the fused ops require it and raise when it
is missing; there is no silent eager fallback on CUDA.
"""
from __future__ import annotations

import importlib

_C = None
_ERR: Exception | None = None


def load():
    """Return the compiled extension module, or None if it is not built."""
    global _C, _ERR
    if _C is None and _ERR is None:
        try:
            _C = importlib.import_module("complexity_framework_b200._C")
        except Exception as exc:  # pragma: no cover - depends on the build
            _ERR = exc
    return _C


def require():
    """Return the extension or raise a clear error naming the build command."""
    mod = load()
    if mod is None:
        raise RuntimeError(
            "complexity_framework_b200._C is not built; run "
            "`python setup.py build_ext --inplace` (sm_100a) first"
        ) from _ERR
    return mod


def available() -> bool:
    return load() is not None


def check_errors(device: int = 0) -> None:
    """Raise if any kernel on ``device`` recorded a device-side error.

    Kernels never trap: a bounded wait that expires, or a failed bounds
    check, writes ``(code, site, block, count)`` into a per-device error word.
    Reading it synchronises the device.
    """
    import torch

    buf = require().error_buffer(device)
    vals = buf.cpu().tolist()
    if vals[0] != 0:
        buf.zero_()
        raise RuntimeError(
            f"device error code={vals[0]} site={vals[1]} block={vals[2]} count={vals[3]}"
        )
