"""Loader for the in-tree sm_100a kernel library.

The compiled module ``swarm_inference_lab_b200._C`` is built in place by
``python setup.py build_ext --inplace`` (or ``__graft_entry__.build()``).  On a
machine with a CUDA device the kernels are mandatory: :func:`ext` raises
instead of silently falling back to PyTorch, so a missing build can never
masquerade as a passing GPU run.
"""
from __future__ import annotations

import importlib
import threading

import torch

_lock = threading.Lock()
_mod = None
_proxy = None
_err: Exception | None = None

# Number of kernel launches issued through this library in the current
# process (each binding call launches exactly one kernel).  CUDA-graph replays
# do not pass through Python, so per-step counts are taken while capturing.
LAUNCHES = [0]


class _Counting:
    """Attribute proxy over the compiled module that counts launches."""

    def __init__(self, mod):
        self._mod = mod

    def __getattr__(self, name):
        fn = getattr(self._mod, name)

        def call(*args, **kw):
            LAUNCHES[0] += 1
            return fn(*args, **kw)

        return call


def launch_count() -> int:
    return LAUNCHES[0]


def ext():
    """Return the compiled kernel module, raising a clear error if it is missing."""
    global _mod, _proxy, _err
    if _proxy is not None:
        return _proxy
    with _lock:
        if _mod is None:
            try:
                _mod = importlib.import_module("swarm_inference_lab_b200._C")
            except Exception as exc:  # pragma: no cover - depends on the build
                _err = exc
                raise RuntimeError(
                    "swarm_inference_lab_b200._C is not built; run "
                    "`python setup.py build_ext --inplace` (sm_100a) first"
                ) from exc
            _proxy = _Counting(_mod)
    return _proxy


def available() -> bool:
    try:
        ext()
        return True
    except RuntimeError:
        return False


def require_cuda(t: torch.Tensor) -> None:
    if not t.is_cuda:
        raise ValueError("sm_100a kernels need CUDA tensors")
