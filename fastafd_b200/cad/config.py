"""CAD configuration from the environment, with a strict parser: unknown values are refused
instead of silently falling back. Reference: python/minisgl/cad/config.py:75-97."""
from __future__ import annotations

import os
from dataclasses import dataclass

_MODES = ("afd", "cad")
_DTYPES = ("bfloat16", "float32")
_HOPS = ("kernel", "copy")


class CadConfigError(ValueError):
    pass


def _get(names, default):
    for n in names:
        v = os.environ.get(n)
        if v not in (None, ""):
            return v
    return default


@dataclass(frozen=True)
class CadConfig:
    mode: str = "afd"
    o_dtype: str = "bfloat16"        # dtype of the attention output rows sent back
    hop: str = "kernel"              # kernel: fused wait+copy+flag kernels; copy: plain copies + flag kernels
    hang_timeout_ns: int = 300_000_000_000
    init_timeout_s: float = 900.0
    attn_per_model: int = 1          # attention GPUs serving one model GPU

    @property
    def enabled(self) -> bool:
        return self.mode == "cad"

    @staticmethod
    def from_env() -> "CadConfig":
        def pick(suffix, default, allowed=None, cast=str):
            raw = _get((f"FASTAFD_{suffix}", f"MINISGL_AFD_{suffix}"), None)
            if raw is None:
                return default
            try:
                val = cast(raw)
            except ValueError as e:
                raise CadConfigError(f"{suffix}={raw!r} is not a valid {cast.__name__}") from e
            if allowed is not None and val not in allowed:
                raise CadConfigError(f"{suffix}={raw!r}: expected one of {', '.join(allowed)}")
            return val
        cfg = CadConfig(mode=pick("MODE", "afd", _MODES), o_dtype=pick("CAD_O_DTYPE", "bfloat16", _DTYPES),
                        hop=pick("CAD_HOP", "kernel", _HOPS),
                        hang_timeout_ns=pick("CAD_HANG_TIMEOUT_NS", 300_000_000_000, None, int),
                        init_timeout_s=pick("CAD_INIT_TIMEOUT_S", 900.0, None, float),
                        attn_per_model=pick("CAD_ATTN_PER_MODEL", 1, None, int))
        if cfg.hang_timeout_ns <= 0 or cfg.init_timeout_s <= 0 or cfg.attn_per_model < 1:
            raise CadConfigError("CAD time-outs and attn_per_model must be positive")
        return cfg
