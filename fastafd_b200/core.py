"""Request-level value types shared by the scheduler, coordinator and workers.

Reference: python/minisgl/core.py (SamplingParams :16, Req :29, Batch :72).
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import List, Tuple


@dataclass
class SamplingParams:
    temperature: float = 0.0
    top_k: int = -1
    top_p: float = 1.0
    ignore_eos: bool = False
    max_tokens: int = 1024
    stop_token_ids: Tuple[int, ...] = ()

    @property
    def is_greedy(self) -> bool:
        return (self.temperature <= 0.0 or self.top_k == 1) and self.top_p == 1.0


@dataclass
class Req:
    """One running request as the scheduler sees it.

    ``cached_len`` tokens already have KV in the cache; ``device_len`` is the length
    after the step being planned; ``table_idx`` is the row of the page table / token
    pool that the request owns on its attention lane."""
    uid: int
    input_ids: List[int]
    sampling: SamplingParams
    table_idx: int = -1
    cached_len: int = 0
    output_ids: List[int] = field(default_factory=list)
    finished: bool = False
    lane: int = 0
    pages: List[int] = field(default_factory=list)
    prefix_hit: int = 0

    @property
    def prompt_len(self) -> int:
        return len(self.input_ids)

    @property
    def total_len(self) -> int:
        return len(self.input_ids) + len(self.output_ids)

    @property
    def remaining_prefill(self) -> int:
        return max(0, self.prompt_len - self.cached_len)

    @property
    def max_total_len(self) -> int:
        return self.prompt_len + self.sampling.max_tokens

    def all_ids(self) -> List[int]:
        return self.input_ids + self.output_ids
