"""Colour logger, rank-0 logging, and buffered per-process log files.

Reference: python/minisgl/utils/logger.py, python/minisgl/afd_support.py:107-193 (log_line).
"""
from __future__ import annotations

import atexit
import logging
import os
import sys
import threading
import time
from typing import Optional

_COLORS = {"DEBUG": "\033[36m", "INFO": "\033[32m", "WARNING": "\033[33m", "ERROR": "\033[31m", "CRITICAL": "\033[35m"}


class _Fmt(logging.Formatter):
    def format(self, record):
        c = _COLORS.get(record.levelname, "") if sys.stderr.isatty() else ""
        r = "\033[0m" if c else ""
        return f"{c}[{time.strftime('%H:%M:%S')}|{record.name}|{record.levelname[0]}]{r} {record.getMessage()}"


def init_logger(name: str, level: Optional[str] = None) -> logging.Logger:
    log = logging.getLogger(name)
    if not log.handlers:
        h = logging.StreamHandler()
        h.setFormatter(_Fmt())
        log.addHandler(h)
        log.propagate = False
    log.setLevel(level or os.environ.get("FASTAFD_LOG_LEVEL", "INFO"))
    return log


def info_rank0(log: logging.Logger, msg: str, rank: Optional[int] = None) -> None:
    if (rank if rank is not None else int(os.environ.get("RANK", "0"))) == 0:
        log.info(msg)


class BufferedLogFile:
    """Append-only log file with an in-memory buffer flushed every `interval_s` or `max_lines`
    (hot loops must not pay a write syscall per line)."""

    def __init__(self, path: str, interval_s: float = 1.0, max_lines: int = 256):
        self.path, self.interval_s, self.max_lines = path, interval_s, max_lines
        self._buf, self._lock, self._last = [], threading.Lock(), time.monotonic()
        os.makedirs(os.path.dirname(path) or ".", exist_ok=True)
        atexit.register(self.flush)

    def line(self, text: str) -> None:
        with self._lock:
            self._buf.append(f"{time.time():.6f} {text}\n")
            due = len(self._buf) >= self.max_lines or time.monotonic() - self._last >= self.interval_s
        if due:
            self.flush()

    def flush(self) -> None:
        with self._lock:
            if not self._buf:
                return
            data, self._buf, self._last = "".join(self._buf), [], time.monotonic()
        with open(self.path, "a") as f:
            f.write(data)
