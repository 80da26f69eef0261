"""Validation of the ``input_ids`` request extension (token ids used verbatim).
Reference: python/minisgl/server/prompt_ids.py."""
from __future__ import annotations

from typing import List, Sequence


def validate_prompt_ids(ids: Sequence[int], vocab_size: int, max_seq_len: int) -> List[int]:
    if not isinstance(ids, (list, tuple)) or len(ids) == 0:
        raise ValueError("input_ids must be a non-empty list of integers")
    out = []
    for i in ids:
        if isinstance(i, bool) or not isinstance(i, int):
            raise ValueError("input_ids must contain integers only")
        if i < 0 or i >= vocab_size:
            raise ValueError(f"input id {i} outside the vocabulary [0, {vocab_size})")
        out.append(int(i))
    if len(out) >= max_seq_len:
        raise ValueError(f"prompt of {len(out)} tokens does not fit max_seq_len {max_seq_len}")
    return out
