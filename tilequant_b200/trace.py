"""NVTX ranges around the path's host-side steps, so profiler timelines show which
projection, prefill or decode step a kernel belongs to.  Off unless ``TQ_NVTX=1`` (or
``set_enabled(True)``); when off, ``nvtx_range`` hands back one shared no-op context."""

from __future__ import annotations

import contextlib
import os

_enabled = os.environ.get("TQ_NVTX", "0") == "1"
_NOOP = contextlib.nullcontext()


def set_enabled(on: bool) -> None:
    global _enabled
    _enabled = bool(on)


def enabled() -> bool:
    return _enabled


@contextlib.contextmanager
def _range(name: str):
    import torch

    torch.cuda.nvtx.range_push(name)
    try:
        yield
    finally:
        torch.cuda.nvtx.range_pop()


def nvtx_range(name: str):
    return _range(name) if _enabled else _NOOP


def traced(name: str):
    """Decorator: the call runs inside ``nvtx_range(name)`` when ranges are on."""
    import functools

    def deco(fn):
        @functools.wraps(fn)
        def wrapper(*args, **kwargs):
            if not _enabled:
                return fn(*args, **kwargs)
            with _range(name):
                return fn(*args, **kwargs)

        return wrapper

    return deco
