"""NVTX ranges with a CPU-side mirror.

``nvtx_range(label)`` pushes an NVTX range when CUDA is present and, when CPU tracing is
switched on, also records (label, start, end, step id parsed from the label) so that a run
leaves ``{prefix}_nvtx_cpu.json`` behind for offline analysis without a profiler.

Reference: python/minisgl/utils/torch_utils.py:26-59 (nvtx_range / nvtx_annotate),
python/minisgl/utils/cpu_trace.py:19-182.
"""
from __future__ import annotations

import functools
import json
import os
import re
import threading
import time
from contextlib import contextmanager
from typing import Dict, List

_ENABLED_NVTX = os.environ.get("FASTAFD_NVTX", "0") == "1"
_STEP_RE = re.compile(r"step[=_]?(\d+)")


class CpuTrace:
    """Thread-safe in-memory list of closed ranges."""

    def __init__(self):
        self.enabled = os.environ.get("FASTAFD_NVTX_CPU_TRACE", "0") == "1"
        self.events: List[Dict] = []
        self._lock = threading.Lock()

    def add(self, label: str, t0: float, t1: float) -> None:
        m = _STEP_RE.search(label)
        with self._lock:
            self.events.append({"name": label, "ts_us": t0 * 1e6, "dur_us": (t1 - t0) * 1e6,
                                "tid": threading.get_ident(), "step": int(m.group(1)) if m else None})

    def dump(self, prefix: str) -> str:
        path = f"{prefix}_nvtx_cpu.json"
        with self._lock, open(path, "w") as f:
            json.dump({"traceEvents": self.events}, f)
        return path

    def clear(self) -> None:
        with self._lock:
            self.events.clear()


CPU_TRACE = CpuTrace()


def set_nvtx(enabled: bool) -> None:
    global _ENABLED_NVTX
    _ENABLED_NVTX = enabled


@contextmanager
def nvtx_range(label: str):
    if not _ENABLED_NVTX and not CPU_TRACE.enabled:
        yield
        return
    pushed = False
    if _ENABLED_NVTX:
        import torch

        if torch.cuda.is_available():
            torch.cuda.nvtx.range_push(label)
            pushed = True
    t0 = time.perf_counter()
    try:
        yield
    finally:
        if pushed:
            import torch

            torch.cuda.nvtx.range_pop()
        if CPU_TRACE.enabled:
            CPU_TRACE.add(label, t0, time.perf_counter())


def nvtx_annotate(fmt: str):
    """Decorator: wraps a method in a range whose label is ``fmt.format(*args)`` of the call's
    positional arguments after ``self`` (e.g. ``"AFD_AG_Attn_{}"`` with the layer index)."""
    def deco(fn):
        @functools.wraps(fn)
        def wrapper(self, *args, **kw):
            try:
                label = fmt.format(*args)
            except (IndexError, KeyError):
                label = fmt
            with nvtx_range(label):
                return fn(self, *args, **kw)
        return wrapper
    return deco
