"""Loader for the native sm_100a extension ``kore_b200._C``.

CUDA tensors always go through the native kernels. If the extension is
missing while a CUDA tensor reaches an op, the op raises: there is no silent
eager fallback on a GPU. CPU tensors use the plain PyTorch definitions in
``kore_b200.ops.reference`` (used by CPU tests and gloo runs).
"""
from __future__ import annotations

import importlib

_C = None
_err: Exception | None = None
_launches = 0


class _Counted:
    """Wraps the extension so every native entry point call (each launches
    exactly one of our kernels) is counted; used for launch accounting."""

    def __init__(self, mod):
        self._mod = mod
        self._cache = {}

    def __getattr__(self, name):
        fn = self._cache.get(name)
        if fn is None:
            raw = getattr(self._mod, name)
            if not callable(raw) or name == "read_and_clear_device_error":
                return raw

            def fn(*a, _raw=raw, **k):
                global _launches
                _launches += 1
                return _raw(*a, **k)

            self._cache[name] = fn
        return fn


def launch_count() -> int:
    return _launches


def reset_launch_count() -> None:
    global _launches
    _launches = 0


def native():
    """Return the loaded extension module or raise with the build command."""
    global _C, _err
    if _C is not None:
        return _C
    if _err is None:
        try:
            _C = _Counted(importlib.import_module("kore_b200._C"))
            return _C
        except Exception as e:  # noqa: BLE001 - recorded and re-raised below
            _err = e
    raise RuntimeError(
        "kore_b200 native extension is not built or failed to load "
        f"({_err!r}); run `python setup.py build_ext --inplace` in the repo root"
    )


def available() -> bool:
    try:
        native()
        return True
    except RuntimeError:
        return False


def check_device_error() -> int:
    """Synchronize and return (and clear) the kernels' device error word.

    1 = an mbarrier wait timed out, 2 = a peer-flag wait timed out."""
    return int(native().read_and_clear_device_error())
