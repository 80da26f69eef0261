"""Statistics of a benchmark run: step time over the pure-decode window, per-GPU throughput,
wall period, and the pass verdict against a recorded value.

Throughput counts every GPU, attention and expert alike:

    tok/s/GPU = b / step_time * r / (r + 1)

with ``b`` requests per attention GPU and ``r`` the attention:expert GPU ratio (1 for a 4+4 split,
3 for 6+2). A speculative run multiplies by the measured tokens per verify step.

Step times come from the coordinator's ``[afd-step-time] step=.. phase=.. bucket=.. ms=..`` lines
(``FASTAFD_STEP_TIMES=1``) or from the JSON line that ``bench.py`` prints.
Reference: scripts/benchmark/run_stats.py:84-89 and scripts/benchmark/README.md:63-78.
"""
from __future__ import annotations

import json
import re
import statistics
from dataclasses import dataclass
from typing import Dict, Iterable, List, Optional, Sequence, Tuple

_STEP_RE = re.compile(r"\[afd-step-time\] step=(\d+) phase=(\w+) bucket=(\d+) num_mb=(\d+) ms=([0-9.]+) real=(\[[^\]]*\]|\d+)")


@dataclass(frozen=True)
class StepSample:
    step: int
    phase: str
    bucket: int
    num_mb: int
    ms: float
    real: int


def parse_step_lines(lines: Iterable[str]) -> List[StepSample]:
    out = []
    for ln in lines:
        m = _STEP_RE.search(ln)
        if m:
            real = sum(int(v) for v in m[6].strip("[]").split(",") if v.strip())      # per-lane list or a total
            out.append(StepSample(int(m[1]), m[2], int(m[3]), int(m[4]), float(m[5]), real))
    return out


def decode_window(samples: Sequence[StepSample], full_batch: Optional[int] = None) -> List[StepSample]:
    """Decode steps after the last prefill step, at the full batch (`real` requests, default the
    largest seen), consecutive in step id."""
    last_prefill = max((i for i, s in enumerate(samples) if s.phase != "decode"), default=-1)
    tail = [s for s in samples[last_prefill + 1:] if s.phase == "decode"]
    if not tail:
        return []
    want = full_batch if full_batch is not None else max(s.real for s in tail)
    best: List[StepSample] = []
    run: List[StepSample] = []
    for s in tail:
        if s.real == want and (not run or s.step == run[-1].step + 1):
            run.append(s)
        else:
            if len(run) > len(best):
                best = run
            run = [s] if s.real == want else []
    return run if len(run) > len(best) else best


def step_mean(samples: Sequence[StepSample], skip: int = 2) -> float:
    """Mean step time (ms) over the window, dropping the first `skip` steps (graph warm-up)."""
    w = [s.ms for s in samples[skip:]] or [s.ms for s in samples]
    if not w:
        raise ValueError("no decode steps in the window")
    return statistics.fmean(w)


def wall_period(step_ids: Sequence[int], timestamps_s: Sequence[float]) -> float:
    """Seconds per step as the inverse slope of step id over wall time (least squares); counts
    host time between steps, which the per-step timer does not see."""
    n = len(step_ids)
    if n < 2:
        raise ValueError("need at least two points")
    mx, my = statistics.fmean(timestamps_s), statistics.fmean(step_ids)
    sxx = sum((x - mx) ** 2 for x in timestamps_s)
    sxy = sum((x - mx) * (y - my) for x, y in zip(timestamps_s, step_ids))
    if sxx == 0 or sxy == 0:
        raise ValueError("degenerate timestamps")
    return sxx / sxy


def throughput_per_gpu(batch_per_attn_gpu: int, step_ms: float, attn_gpus: int, expert_gpus: int,
                       tokens_per_step: float = 1.0) -> float:
    """tok/s/GPU over all GPUs; ``tokens_per_step`` > 1 for speculative decoding."""
    total = batch_per_attn_gpu * attn_gpus * tokens_per_step / (step_ms / 1e3)
    return total / (attn_gpus + expert_gpus)


def verdict(measured: float, recorded: Optional[float], tolerance: float = 0.03) -> Tuple[str, Optional[float]]:
    """('pass' | 'fail' | 'unrecorded', relative deviation)."""
    if recorded is None or recorded <= 0:
        return "unrecorded", None
    dev = measured / recorded - 1.0
    return ("pass" if abs(dev) <= tolerance else "fail"), dev


def from_bench_json(line: str) -> Dict[str, float]:
    d = json.loads(line)
    return {"step_ms": float(d["ms_per_step"]), "tok_s": float(d["value"]), "tok_s_per_gpu": float(d["value"]) / d["n_gpus"],
            "e2e_step_ms": float(d.get("e2e", {}).get("ms_per_step", float("nan")))}
