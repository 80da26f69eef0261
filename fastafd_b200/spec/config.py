"""Speculative-decoding settings from flags and environment.

Environment (each also answers to the ``MINISGL_AFD_`` prefix): ``FASTAFD_SPEC`` switches it on,
``FASTAFD_SPEC_BLOCK`` = tokens verified per step (draft tokens + 1, default 4),
``FASTAFD_SPEC_DRAFT`` = draft checkpoint directory ("" = random-init draft head, for timing runs),
``FASTAFD_SPEC_SIM_ACCEPT`` = mean accepted tokens per step to simulate (0 = real greedy acceptance),
``FASTAFD_SPEC_SIM_SEED``. Flags (``--spec-block``, ``--spec-draft-path``) win over the environment.

Reference: python/minisgl/spec/config.py:44-67 (afd_spec_config), :85-124 (acceptance rule).
"""
from __future__ import annotations

from dataclasses import dataclass

from ..env import ENV


class SpecConfigError(ValueError):
    pass


@dataclass(frozen=True)
class SpecConfig:
    enabled: bool = False
    block: int = 0                 # verified tokens per step (draft tokens + 1); 0 when off
    draft_path: str = ""
    sim_accept: float = 0.0        # 0 = real acceptance
    sim_seed: int = 0

    @property
    def num_draft_tokens(self) -> int:
        return max(self.block - 1, 0)

    def validate(self) -> "SpecConfig":
        if not self.enabled:
            return self
        if not 2 <= self.block <= 16:
            raise SpecConfigError(f"spec block must be 2..16 (draft tokens + 1), got {self.block}")
        if self.sim_accept and not 1.0 <= self.sim_accept <= self.block:
            raise SpecConfigError(f"simulated acceptance must lie in [1, block={self.block}], got {self.sim_accept}")
        return self

    @staticmethod
    def from_env(block_flag: int = 0, draft_flag: str = "") -> "SpecConfig":
        """Flags first, then the environment; returns a disabled config when neither asks for it."""
        on = block_flag > 1 or bool(ENV.SPEC.value)
        if not on:
            return SpecConfig()
        block = block_flag if block_flag > 1 else int(ENV.SPEC_BLOCK.value)
        return SpecConfig(True, block, draft_flag or str(ENV.SPEC_DRAFT.value), float(ENV.SPEC_SIM_ACCEPT.value),
                          int(ENV.SPEC_SIM_SEED.value)).validate()
