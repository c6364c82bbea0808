"""Loader of the host runtime library `hetero_cp_ringattn_b200._host` (C++, no CUDA).

The planning and bookkeeping that every rank and the coordinator run on the CPU live there:
ring layouts, capacity chunking and KV byte admission, the frozen KV-growth schedule, the KV page
allocator and the batch scheduler's queue. The Python modules `parallel.strategy`,
`parallel.capacity`, `parallel.schedule`, `kv.arena` and `serve.scheduler` are thin bindings of
it. It is built with the sm_100a extension (`python setup.py build_ext --inplace`) and is
required on every machine, with or without a GPU.
"""

from __future__ import annotations

import importlib

from .errors import NativeExtensionMissing

_mod = None


def lib():
    global _mod
    if _mod is None:
        try:
            _mod = importlib.import_module("hetero_cp_ringattn_b200._host")
        except ImportError as e:
            raise NativeExtensionMissing(
                "the host runtime library hetero_cp_ringattn_b200._host is not built "
                f"(run `python setup.py build_ext --inplace`): {e}") from e
    return _mod
