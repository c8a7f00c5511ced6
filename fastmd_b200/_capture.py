"""Python garbage collection around CUDA-graph captures.

A CUDA graph that has become unreachable is released when Python's collector finds it; if that happens
while another graph is being captured, its release (not a capturable operation) invalidates the capture.
``quiet_gc()`` collects first, so such graphs die before the capture starts, and keeps the collector off
until the capture ends."""
from __future__ import annotations

import contextlib
import gc


@contextlib.contextmanager
def quiet_gc():
    gc.collect()
    enabled = gc.isenabled()
    gc.disable()
    try:
        yield
    finally:
        if enabled:
            gc.enable()
