"""Optional NVTX ranges around the engine's calls, for a profiler's timeline
(Nsight Systems, or ``ncu --nvtx --nvtx-include <name>/`` to capture the
kernels of one call).

Off by default, and free when off: unless ``ASTRA_NVTX`` is set to a value
other than ``0`` when the package is imported, ``traced`` returns each method
unchanged.  When on, every traced call runs inside
``torch.cuda.nvtx.range_push(name)`` / ``range_pop()``, named after the
reference method it replaces (``AddTwoSidedQuotes``, ``GetBBOs``,
``ApplyPlayerTrading``, ...).  A range marks the host call; the kernels it
launches run asynchronously on the market's stream.
"""
from __future__ import annotations

import functools
import os

ENABLED = os.environ.get("ASTRA_NVTX", "0") not in ("", "0")


def traced(name: str):
    """Decorator: wrap the method in an NVTX range called `name` when
    ``ASTRA_NVTX`` is on; otherwise return it as it is."""
    def wrap(fn):
        if not ENABLED:
            return fn
        import torch

        @functools.wraps(fn)
        def inner(*args, **kwargs):
            torch.cuda.nvtx.range_push(name)
            try:
                return fn(*args, **kwargs)
            finally:
                torch.cuda.nvtx.range_pop()
        return inner
    return wrap
