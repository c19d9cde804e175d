"""Loader of the in-tree sm_100a extension.

The compiled module is imported straight from ``ops/_build/_mxk.so``. On a machine with a GPU,
every CUDA op requires it: a missing or stale build raises instead of silently falling back.
"""

from __future__ import annotations

import importlib.util
import os
import threading

import torch

from .build import BUILD_DIR, EXT_NAME

_EXT = None
_LOCK = threading.Lock()
_ERR: dict[int, torch.Tensor] = {}


def ext():
    global _EXT
    if _EXT is None:
        with _LOCK:
            if _EXT is None:
                path = os.path.join(BUILD_DIR, EXT_NAME + ".so")
                if not os.path.exists(path):
                    raise RuntimeError(
                        f"sm_100a extension not built ({path} missing); run "
                        "`python -m marin_experiments_b200.ops.build`"
                    )
                spec = importlib.util.spec_from_file_location(EXT_NAME, path)
                mod = importlib.util.module_from_spec(spec)
                spec.loader.exec_module(mod)
                _EXT = mod
    return _EXT


def available() -> bool:
    return os.path.exists(os.path.join(BUILD_DIR, EXT_NAME + ".so"))


def err_flag(device: torch.device) -> torch.Tensor:
    """Per-device int32 flag the kernels set when a bounded wait times out."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    t = _ERR.get(idx)
    if t is None:
        t = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", idx))
        _ERR[idx] = t
    return t


class KernelTimeoutError(RuntimeError):
    pass


def check_kernel_errors(device: torch.device | None = None) -> None:
    """Synchronise and raise if any kernel recorded a timed-out wait (then clear the flag)."""
    devs = [device.index] if device is not None else list(_ERR)
    for idx in devs:
        t = _ERR.get(idx)
        if t is None:
            continue
        code = int(t.item())
        if code != 0:
            t.zero_()
            raise KernelTimeoutError(f"cuda:{idx}: kernel wait timed out (code {code})")
