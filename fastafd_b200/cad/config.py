"""CAD configuration from the environment, with a strict parser: unknown values are refused instead of silently
falling back, and a CAD key without CAD mode is refused too (a job-script mistake). Every key answers to the
``FASTAFD_`` name and to the reference's ``MINISGL_AFD_`` name, and takes the reference's spellings of the values
(``bf16``, ``window``, ``megamoe_dual``).

  MODE                  afd (default, also unset / "") | cad
  CAD_O_DTYPE           bfloat16 | bf16, float32 | fp32: dtype of the attention output rows sent back
  CAD_HOP               kernel | window: put / wait kernels over the peer-mapped window; copy: plain copies + flag kernels
  CAD_MOE               dual | megamoe_dual: every model rank is a dispatch source and an expert rank at once
  CAD_HANG_TIMEOUT_NS   limit of every flag wait; a wait that runs out sets the window's err word
  CAD_INIT_TIMEOUT_S    how long the coordinator lets the ranks take over the CAD init
  CAD_ATTN_PER_MODEL    attention ranks per model rank of a deployment built inside one process

Reference: python/minisgl/cad/config.py:1-97.
"""
from __future__ import annotations

import os
from dataclasses import dataclass
from typing import Dict, Mapping, Optional

_MODES = ("afd", "cad")
_DTYPES = {"bfloat16": "bfloat16", "bf16": "bfloat16", "float32": "float32", "fp32": "float32"}
_HOPS = {"kernel": "kernel", "window": "kernel", "copy": "copy"}
_MOES = {"dual": "dual", "megamoe_dual": "dual"}
_CAD_SUFFIXES = ("CAD_O_DTYPE", "CAD_HOP", "CAD_MOE", "CAD_HANG_TIMEOUT_NS", "CAD_INIT_TIMEOUT_S", "CAD_ATTN_PER_MODEL")


class CadConfigError(ValueError):
    pass


def _names(suffix: str):
    return (f"FASTAFD_{suffix}", f"MINISGL_AFD_{suffix}")


def _get(env: Mapping[str, str], suffix: str) -> Optional[str]:
    for n in _names(suffix):
        v = env.get(n)
        if v not in (None, ""):
            return v.strip()
    return None


@dataclass(frozen=True)
class CadConfig:
    mode: str = "afd"
    o_dtype: str = "bfloat16"        # dtype of the attention output rows sent back
    hop: str = "kernel"              # kernel: fused wait+copy+flag kernels; copy: plain copies + flag kernels
    moe: str = "dual"                # every model rank dispatches its own rows and serves its slice of the experts
    hang_timeout_ns: int = 300_000_000_000
    init_timeout_s: float = 900.0
    attn_per_model: int = 1          # attention GPUs serving one model GPU

    @property
    def enabled(self) -> bool:
        return self.mode == "cad"

    @staticmethod
    def from_env(environ: Optional[Mapping[str, str]] = None) -> "CadConfig":
        env = os.environ if environ is None else environ

        def pick(suffix, default, allowed=None, cast=str):
            raw = _get(env, suffix)
            if raw is None:
                return default
            try:
                val = cast(raw)
            except ValueError as e:
                raise CadConfigError(f"{suffix}={raw!r} is not a valid {cast.__name__}") from e
            if allowed is None:
                return val
            if val not in allowed:
                extra = " (DeepEP is not an expert path of this framework)" if (suffix, val) == ("CAD_MOE", "deepep") else ""
                raise CadConfigError(f"{suffix}={raw!r}: expected one of {', '.join(allowed)}{extra}")
            return allowed[val] if isinstance(allowed, dict) else val

        mode = pick("MODE", "afd", _MODES)
        if mode != "cad":
            stray = [n for s in _CAD_SUFFIXES for n in _names(s) if env.get(n)]
            if stray:
                raise CadConfigError(f"{', '.join(stray)} set without MODE=cad")
            return CadConfig()
        cfg = CadConfig(mode=mode, o_dtype=pick("CAD_O_DTYPE", "bfloat16", _DTYPES), hop=pick("CAD_HOP", "kernel", _HOPS),
                        moe=pick("CAD_MOE", "dual", _MOES),
                        hang_timeout_ns=pick("CAD_HANG_TIMEOUT_NS", 300_000_000_000, None, int),
                        init_timeout_s=pick("CAD_INIT_TIMEOUT_S", 900.0, None, float),
                        attn_per_model=pick("CAD_ATTN_PER_MODEL", 1, None, int))
        if cfg.hang_timeout_ns <= 0 or cfg.init_timeout_s <= 0 or cfg.attn_per_model < 1:
            raise CadConfigError("CAD time-outs and attn_per_model must be positive")
        return cfg

    def env(self) -> Dict[str, str]:
        """The environment that reproduces this configuration in a child process (empty when CAD is off)."""
        if not self.enabled:
            return {}
        return {"FASTAFD_MODE": "cad", "FASTAFD_CAD_O_DTYPE": self.o_dtype, "FASTAFD_CAD_HOP": self.hop,
                "FASTAFD_CAD_MOE": self.moe, "FASTAFD_CAD_HANG_TIMEOUT_NS": str(self.hang_timeout_ns),
                "FASTAFD_CAD_INIT_TIMEOUT_S": str(self.init_timeout_s), "FASTAFD_CAD_ATTN_PER_MODEL": str(self.attn_per_model)}
