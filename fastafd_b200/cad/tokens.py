"""Token path of a model rank in a core-attention-disaggregated decode step.

The model rank embeds, applies the final norm and the LM head, and samples (greedy) for the rows of all its
``r`` peers. A micro-batch of a step with bucket ``B`` has ``r * B`` rows on the model rank, peer ``p``'s rows
at ``p*B .. (p+1)*B``; over a step the rows are micro-batch major, so request ``i`` of peer ``p`` in
micro-batch ``m`` sits at row ``(m*r + p)*B + i``. Rows without a request are padding: token 0 at position 0,
and their sampled token goes to a dump slot.

Where the input token comes from: every request owns a *last-token slot* on its model rank
(``peer * table_rows + request-table row``, stable while the request lives). The coordinator sends the input
token when the host has it (the first decode step after a prefill, whose token the attention rank sampled), else
-1, and the row then takes what the previous decode step sampled for the request and left in its slot. Decode
steps therefore follow one another without a host round trip.

All per-step state is a set of fixed-size device tensors filled by plain copies, so a step can be captured in a
CUDA graph. Sampling is greedy only: a graph replays the same random numbers, so requests that want random
sampling are refused at admission.

Reference: python/minisgl/cad/tokens.py:15-152.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, List, Sequence

import numpy as np
import torch

ROW_FIELDS = ("peer", "mb", "i", "table_row", "position", "host_token")


@dataclass(frozen=True)
class CadRow:
    """One request of a decode step, as its model rank sees it."""
    peer: int            # position of its attention rank among the model rank's peers
    mb: int
    i: int               # index inside that peer's micro-batch (< bucket)
    table_row: int       # its row in the lane's request table
    position: int        # position of the step's input token (= KV length before the step)
    host_token: int      # the input token, or -1: take the token the previous step sampled


def pack_rows(rows: Sequence[CadRow]) -> np.ndarray:
    """Rows as one int32 array [n, 6] (the wire form; column order = ROW_FIELDS)."""
    return np.asarray([[getattr(q, f) for f in ROW_FIELDS] for q in rows], np.int32).reshape(-1, len(ROW_FIELDS))


def unpack_rows(arr: np.ndarray) -> List[CadRow]:
    return [CadRow(*(int(v) for v in line)) for line in np.asarray(arr).reshape(-1, len(ROW_FIELDS))]


def row_index(r: int, bucket: int, mb: int, peer: int, i: int) -> int:
    if not (0 <= peer < r and 0 <= i < bucket and mb >= 0):
        raise ValueError(f"row (mb {mb}, peer {peer}, i {i}) outside {r} peers x bucket {bucket}")
    return (mb * r + peer) * bucket + i


def host_token(known_ids: Sequence[int], position: int) -> int:
    """The input token at `position` if the host knows it, else -1."""
    return int(known_ids[position]) if 0 <= position < len(known_ids) else -1


class CadTokenPath:
    def __init__(self, r: int, num_mb: int, t_max: int, table_rows: int, device="cpu"):
        self.r, self.num_mb, self.t_max, self.table_rows = r, num_mb, t_max, table_rows
        self.device = torch.device(device)
        T = num_mb * r * t_max
        self.dump_slot = r * table_rows
        z = lambda n, dt: torch.zeros(n, dtype=dt, device=self.device)  # noqa: E731
        self.host_ids, self.pos, self.out = z(T, torch.int32), z(T, torch.int32), z(T, torch.int32)
        self.slot = torch.full((T,), self.dump_slot, dtype=torch.int64, device=self.device)
        self.last = z(self.dump_slot + 1, torch.int32)
        self.bucket = 0

    # ------------------------------------------------------------------ host side of a step
    def bind(self, bucket: int) -> None:
        if not 0 < bucket <= self.t_max:
            raise ValueError(f"bucket {bucket} outside 1..{self.t_max}")
        self.bucket = bucket

    @property
    def rows(self) -> int:
        """Rows of a step at the bound bucket."""
        return self.num_mb * self.r * self.bucket

    def mb_rows(self, mb: int) -> slice:
        n = self.r * self.bucket
        return slice(mb * n, (mb + 1) * n)

    def peer_rows(self, mb: int, peer: int) -> slice:
        a = (mb * self.r + peer) * self.bucket
        return slice(a, a + self.bucket)

    def host_arrays(self, rows: Sequence[CadRow]):
        """(ids, slot, pos, where): the step's three input arrays with padding filled in, and the row of each
        request in the order given."""
        n = self.rows
        ids, slot, pos = np.zeros(n, np.int32), np.full(n, self.dump_slot, np.int64), np.zeros(n, np.int32)
        where: List[int] = []
        for q in rows:
            if q.mb >= self.num_mb or not 0 <= q.table_row < self.table_rows:
                raise ValueError(f"{q}: micro-batch or table row outside {self.num_mb} / {self.table_rows}")
            k = row_index(self.r, self.bucket, q.mb, q.peer, q.i)
            if slot[k] != self.dump_slot:
                raise ValueError(f"two requests on row {k}")
            ids[k], slot[k], pos[k] = q.host_token, q.peer * self.table_rows + q.table_row, q.position
            where.append(k)
        if len(set(slot[where].tolist())) != len(where):
            raise ValueError("one request appears twice in a step")
        return ids, slot, pos, where

    def stage(self, rows: Sequence[CadRow]) -> List[int]:
        """Copy a step's rows to the device (pinned source on CUDA, no host sync)."""
        ids, slot, pos, where = self.host_arrays(rows)
        n = self.rows
        for dst, src in ((self.host_ids, ids), (self.slot, slot), (self.pos, pos)):
            t = torch.from_numpy(src)
            if dst.is_cuda:
                t = t.pin_memory()
            dst[:n].copy_(t, non_blocking=dst.is_cuda)
        return where

    def stage_padding(self) -> None:
        """A step of padding rows only (warm-up, graph capture)."""
        n = self.rows
        self.host_ids[:n].zero_()
        self.pos[:n].zero_()
        self.slot[:n].fill_(self.dump_slot)

    # ------------------------------------------------------------------ device side (fixed shapes)
    def input_ids(self) -> torch.Tensor:
        n = self.rows
        host = self.host_ids[:n]
        return torch.where(host >= 0, host, self.last.index_select(0, self.slot[:n]))

    def positions(self) -> torch.Tensor:
        return self.pos[:self.rows]

    def record(self, tokens: torch.Tensor) -> None:
        """Keep the step's sampled tokens: per row for the reply, per request slot for the next step."""
        n = self.rows
        self.out[:n].copy_(tokens.to(torch.int32))
        self.last.index_copy_(0, self.slot[:n], self.out[:n])


def tokens_by_peer(out_host: Sequence[int], r: int, num_mb: int, bucket: int) -> Dict[int, np.ndarray]:
    """A step's sampled tokens regrouped per peer in the lane scheduler's order (micro-batch major, bucket
    padded): what each lane's `complete` takes."""
    out = np.asarray(out_host, np.int32).reshape(num_mb, r, bucket)
    return {p: out[:, p, :].reshape(-1).copy() for p in range(r)}
