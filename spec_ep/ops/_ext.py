"""Loader for the in-tree sm_100a extension ``spec_ep._C``.

The extension is built with ``python setup.py build_ext --inplace`` (or
``__graft_entry__.build()``). There is no fallback: on a machine with a GPU a missing
or stale extension raises immediately, so a test can never pass on a silent eager path.
"""
from __future__ import annotations

import importlib

_C = None
_ERR: Exception | None = None


def load():
    """Return the compiled module, raising a clear error if it is unavailable."""
    global _C, _ERR
    if _C is not None:
        return _C
    try:
        import torch  # noqa: F401  (loads libc10 / libtorch, which the extension links against)

        _C = importlib.import_module("spec_ep._C")
    except Exception as e:  # pragma: no cover - depends on the build
        _ERR = e
        raise RuntimeError(
            "spec_ep._C (sm_100a kernels) is not built or failed to load; run "
            "`python setup.py build_ext --inplace`. Original error: %r" % (e,)
        ) from e
    return _C


def available() -> bool:
    try:
        load()
        return True
    except RuntimeError:
        return False
