"""Loader for the in-tree native extensions.

The CUDA kernels live in ``kapsl_sdk_b200._cuda`` (built by ``setup.py`` /
``__graft_entry__.build``).  On a machine with a GPU a missing extension is an
error, never a silent fallback: every GPU op in :mod:`kapsl_sdk_b200.ops` calls
:func:`cuda_ops`, which raises if the shared object cannot be imported.
"""
from __future__ import annotations

import importlib
import os

_cuda_mod = None
_native_mod = None
_cuda_err: Exception | None = None


def cuda_ops():
    """Return the compiled sm_100a kernel module or raise ``RuntimeError``."""
    global _cuda_mod, _cuda_err
    if _cuda_mod is not None:
        return _cuda_mod
    try:
        import torch  # noqa: F401  (the extension links against libtorch)

        _cuda_mod = importlib.import_module("kapsl_sdk_b200._cuda")
    except Exception as e:  # pragma: no cover - depends on the build
        _cuda_err = e
        raise RuntimeError(
            "kapsl_sdk_b200._cuda is not built or failed to load "
            f"({e!r}); run `python setup.py build_ext --inplace` (sm_100a)"
        ) from e
    return _cuda_mod


def native():
    """Return the C++ runtime module (wire codec, block allocator, SHM, servers)."""
    global _native_mod
    if _native_mod is None:
        try:
            _native_mod = importlib.import_module("kapsl_sdk_b200._native")
        except Exception as e:
            raise RuntimeError(
                f"kapsl_sdk_b200._native is not built ({e!r}); run `python setup.py build_ext --inplace`"
            ) from e
    return _native_mod


def cuda_available() -> bool:
    """True when torch sees a CUDA device (the kernels then must load)."""
    if os.environ.get("KAPSL_FORCE_CPU") == "1":
        return False
    import torch

    return torch.cuda.is_available()


def launch_count() -> int:
    """Kernels launched through kapsl's own CUDA extension so far (host count)."""
    if _cuda_mod is None:
        return 0
    return int(_cuda_mod.launch_count())
