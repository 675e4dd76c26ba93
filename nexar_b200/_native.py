"""Loaders for the in-tree native extensions.

Both modules are built by ``python setup.py build_ext --inplace``. A missing
extension raises immediately: there is no Python fallback for any kernel.
"""
from __future__ import annotations

import functools


@functools.lru_cache(maxsize=None)
def cuda():
    """The sm_100a device runtime (``nexar_b200._cuda``)."""
    import torch  # noqa: F401  (loads libc10/libtorch for the extension)
    try:
        from . import _cuda  # type: ignore
    except ImportError as e:  # pragma: no cover - exercised only on broken installs
        raise RuntimeError(
            "nexar_b200._cuda is not built; run `python setup.py build_ext --inplace` "
            "(or __graft_entry__.build()) before using device features") from e
    return _cuda


@functools.lru_cache(maxsize=None)
def host():
    """The C++ host runtime (``nexar_b200._host``)."""
    import torch  # noqa: F401
    try:
        from . import _host  # type: ignore
    except ImportError as e:  # pragma: no cover
        raise RuntimeError(
            "nexar_b200._host is not built; run `python setup.py build_ext --inplace`") from e
    return _host


def launch_count() -> int:
    """Number of nexar_b200 kernels launched by this process so far."""
    return int(cuda().launch_count())
