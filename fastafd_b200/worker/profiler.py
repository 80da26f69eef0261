"""Profiler capture window by step id.

Workers started under a profiler with ``capture-range=cudaProfilerApi`` record only between
``cudaProfilerStart`` and ``cudaProfilerStop``. The window is named by global step ids
(``FASTAFD_CONTROL_PROFILE_START_STEP`` / ``_STOP_STEP``, or a command from the coordinator),
so that all ranks capture the same steps.

Reference: python/minisgl/afd_profiler.py:11-103, python/minisgl/afd_worker_base.py:1083-1113.
"""
from __future__ import annotations

from typing import Optional

from ..env import ENV


class StepProfiler:
    def __init__(self, start_step: Optional[int] = None, stop_step: Optional[int] = None, backend=None):
        self.start_step = ENV.PROFILE_START_STEP.value if start_step is None else start_step
        self.stop_step = ENV.PROFILE_STOP_STEP.value if stop_step is None else stop_step
        self.active = False
        self._backend = backend

    def _api(self):
        if self._backend is not None:
            return self._backend
        import torch

        return torch.cuda.profiler

    def on_step(self, step_id: int) -> None:
        """Call before executing step `step_id`."""
        if self.start_step < 0:
            return
        if not self.active and step_id == self.start_step:
            self._api().start()
            self.active = True
        elif self.active and self.stop_step >= 0 and step_id >= self.stop_step:
            self._api().stop()
            self.active = False

    def close(self) -> None:
        if self.active:
            self._api().stop()
            self.active = False
