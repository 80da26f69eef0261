"""Typed environment variables (an override layer on top of the typed configuration).

Every knob is ``FASTAFD_<NAME>``; for users coming from the reference the same knob is also
read from ``MINISGL_AFD_<NAME>`` / ``MINISGL_<NAME>`` when the new name is unset.

Reference: python/minisgl/env.py (EnvVar wrappers, ENV singleton, afd_env).
"""
from __future__ import annotations

import os
from typing import Callable, Generic, Optional, TypeVar

T = TypeVar("T")


def _to_bool(s: str) -> bool:
    return s.strip().lower() in ("1", "true", "yes", "on")


class EnvVar(Generic[T]):
    def __init__(self, name: str, default: T, parse: Callable[[str], T], aliases=()):
        self.name, self.default, self.parse, self.aliases = name, default, parse, tuple(aliases)

    def names(self):
        return (f"FASTAFD_{self.name}", f"MINISGL_AFD_{self.name}", f"MINISGL_{self.name}") + self.aliases

    @property
    def value(self) -> T:
        for n in self.names():
            raw = os.environ.get(n)
            if raw is not None and raw != "":
                try:
                    return self.parse(raw)
                except ValueError as e:
                    raise ValueError(f"bad value for {n}: {raw!r}") from e
        return self.default

    def __bool__(self) -> bool:
        return bool(self.value)


class _Env:
    """The registry of knobs. Names follow the reference's registry
    (python/minisgl/ray_env_keys.py) where the knob still exists in this design."""
    FLAG_TIMEOUT_S = EnvVar("FLAG_TIMEOUT_S", 20.0, float)
    STARTUP_TIMEOUT_S = EnvVar("STARTUP_TIMEOUT_S", 1800.0, float)
    DIST_TIMEOUT = EnvVar("DIST_TIMEOUT", 600.0, float)
    LOG_STEPS = EnvVar("LOG_STEPS", False, _to_bool)
    STEP_TIMES = EnvVar("STEP_TIMES", False, _to_bool)
    PAGE_AUDIT = EnvVar("PAGE_AUDIT", False, _to_bool)
    COMM_TRACE = EnvVar("COMM_TRACE", False, _to_bool)
    NVTX = EnvVar("NVTX", False, _to_bool)
    NVTX_CPU_TRACE = EnvVar("NVTX_CPU_TRACE", False, _to_bool)
    MAX_COMM_TOKENS = EnvVar("MAX_COMM_TOKENS", 2048, int)
    PREFIX_CACHE = EnvVar("PREFIX_CACHE", "naive", str)
    MODE = EnvVar("MODE", "afd", str)                      # afd | cad
    SPEC = EnvVar("SPEC", False, _to_bool)
    SPEC_BLOCK = EnvVar("SPEC_BLOCK", 4, int)
    SPEC_DRAFT = EnvVar("SPEC_DRAFT", "", str)
    SPEC_SIM_ACCEPT = EnvVar("SPEC_SIM_ACCEPT", 0.0, float)
    SPEC_SIM_SEED = EnvVar("SPEC_SIM_SEED", 0, int)
    CAD_HANG_TIMEOUT_NS = EnvVar("CAD_HANG_TIMEOUT_NS", 300_000_000_000, int)
    CAD_INIT_TIMEOUT_S = EnvVar("CAD_INIT_TIMEOUT_S", 900.0, float)
    CAD_O_DTYPE = EnvVar("CAD_O_DTYPE", "bfloat16", str)
    PROFILE_START_STEP = EnvVar("CONTROL_PROFILE_START_STEP", -1, int)
    PROFILE_STOP_STEP = EnvVar("CONTROL_PROFILE_STOP_STEP", -1, int)
    LOG_DIR = EnvVar("LOG_DIR", "", str)


ENV = _Env()

# Knobs of the hot path that are read where they act (some of them in C, by getenv), with the reference's
# name for the same switch where it has one. `apply_reference_aliases` copies a reference name that is set
# onto the new name that is not, once, when the package is imported.
HOT_PATH_KNOBS = {
    "FASTAFD_PDL": "programmatic dependent launch of the decode-path kernels (default 1)",
    "FASTAFD_DIRECT": "slot-claiming N2M exchange (default 1; 0 = receive slots + group/gather)",
    "FASTAFD_TP_FUSED": "attention-TP collectives fused with the GEMMs over the fabric (default 1; 0 = NCCL)",
    "FASTAFD_OWN_DENSE": "own tcgen05 kernel for dense projections (1 = bf16 and FP8, fp8 = FP8 only; default library)",
    "FASTAFD_L2_PREFETCH_MB": "weights the gate/up GEMM pulls into L2 while it waits for its predecessor (default 64)",
    "FASTAFD_LANE_STREAMS": "every micro-batch's attention-side chain on its own stream (default 0)",
    "FASTAFD_ROUTE_TPC": "tokens per CTA of the route kernel (default 4)",
    "FASTAFD_ROUTE_CLUSTER": "CTAs that share a token group's expert range in the route kernel (default by gate size)",
    "FASTAFD_COMM_TRACE": "device-side timeline of the N2M / M2N exchange",
}
REFERENCE_ALIASES = {
    "MINISGL_PDL": "FASTAFD_PDL",
    "MINISGL_AFD_LANE_COMPUTE_STREAMS": "FASTAFD_LANE_STREAMS",
    "MINISGL_MEGAMOE_EG_PREFETCH_MB": "FASTAFD_L2_PREFETCH_MB",
    "MINISGL_MEGAMOE_AG_TIMING": "FASTAFD_COMM_TRACE",
    "MINISGL_MEGAMOE_EG_TIMING": "FASTAFD_COMM_TRACE",
}


def apply_reference_aliases(environ=None) -> dict:
    """For every reference name that is set while its new name is not, set the new name to the same
    value. Returns what was copied (new name -> value)."""
    environ = os.environ if environ is None else environ
    copied = {}
    for old, new in REFERENCE_ALIASES.items():
        v = environ.get(old)
        if v not in (None, "") and environ.get(new) in (None, ""):
            environ[new] = v
            copied[new] = v
    return copied


def afd_env(suffix: str, default: Optional[str] = None) -> Optional[str]:
    """Raw lookup of an AFD knob by suffix (FASTAFD_<suffix>, then MINISGL_AFD_<suffix>)."""
    for n in (f"FASTAFD_{suffix}", f"MINISGL_AFD_{suffix}"):
        if os.environ.get(n):
            return os.environ[n]
    return default
