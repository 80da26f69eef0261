"""Decode graph bucket ladders and micro-batch splitting.

Reference: python/minisgl/afd_support.py:549-619 (_normalize_decode_graph_bs,
compute_decode_graph_sizes, select_decode_graph_bs) and
python/minisgl/afd_scheduler.py:372-417,868-940 (_compute_microbatch_offsets,
_balanced_decode_padded_reqs, _select_padded_size).
"""
from __future__ import annotations

from typing import List, Sequence, Tuple


def default_decode_buckets(max_bs: int) -> List[int]:
    """[1, 2, 4] + every 8 up to 256 + every 16 above, capped at max_bs (max_bs included)."""
    sizes = [s for s in (1, 2, 4) if s <= max_bs]
    sizes += list(range(8, min(max_bs, 256) + 1, 8))
    if max_bs > 256:
        sizes += list(range(272, max_bs + 1, 16))
    if max_bs not in sizes:
        sizes.append(max_bs)
    return sorted(set(sizes))


def normalize_buckets(explicit: Sequence[int], max_bs: int) -> List[int]:
    if not explicit:
        return default_decode_buckets(max_bs)
    out = sorted({int(b) for b in explicit if int(b) > 0})
    if not out:
        raise ValueError("decode graph bucket list is empty")
    return out


def select_bucket(real_per_mb: int, buckets: Sequence[int]) -> int:
    """Smallest captured size >= real_per_mb (largest bucket if none fits: caller must split)."""
    for b in buckets:
        if b >= real_per_mb:
            return b
    raise ValueError(f"{real_per_mb} requests per micro-batch exceed the largest bucket {buckets[-1]}")


def per_mb_real(num_real: int, num_mb: int) -> int:
    return max(1, (num_real + num_mb - 1) // num_mb)


def balanced_split(num_real: int, num_mb: int) -> List[int]:
    """Real requests per micro-batch, spread evenly so that no micro-batch is all padding
    unless there are fewer requests than micro-batches."""
    base, rem = divmod(num_real, num_mb)
    return [base + (1 if i < rem else 0) for i in range(num_mb)]


def split_prefill(extend_lens: Sequence[int], num_mb: int) -> List[Tuple[int, int]]:
    """Split a prefill batch into num_mb contiguous request ranges at the request boundaries
    closest to equal token counts. Returns [(start, end)) per micro-batch (may be empty)."""
    n = len(extend_lens)
    total = sum(extend_lens)
    bounds = [0]
    acc, idx = 0, 0
    for m in range(1, num_mb):
        target = total * m / num_mb
        while idx < n and abs(acc + extend_lens[idx] - target) <= abs(acc - target):
            acc += extend_lens[idx]
            idx += 1
        bounds.append(idx)
    bounds.append(n)
    return [(bounds[i], bounds[i + 1]) for i in range(num_mb)]
