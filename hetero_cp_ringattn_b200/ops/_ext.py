"""Loader of the in-tree sm_100a extension (`hetero_cp_ringattn_b200._C`).

On a machine with a GPU the extension is mandatory: `native()` raises if it cannot be imported,
so a GPU run can never silently fall back to a PyTorch path. On a CPU-only machine (build checks,
CPU-rank tests) `available()` is False and callers use the reference ops for CPU tensors.
"""

from __future__ import annotations

import importlib

from ..errors import NativeExtensionMissing

_mod = None
_err = None


def _load():
    global _mod, _err
    if _mod is not None or _err is not None:
        return _mod
    try:
        import torch  # noqa: F401  (loads libc10 / libtorch that the extension links against)
        _mod = importlib.import_module("hetero_cp_ringattn_b200._C")
    except Exception as e:  # pragma: no cover - exercised only when the build is missing
        _err = e
    return _mod


def available() -> bool:
    return _load() is not None


def native():
    m = _load()
    if m is None:
        raise NativeExtensionMissing(
            "the sm_100a extension hetero_cp_ringattn_b200._C is not built "
            f"(run `python setup.py build_ext --inplace`): {_err}")
    return m


def so_path() -> str | None:
    m = _load()
    return getattr(m, "__file__", None) if m is not None else None
