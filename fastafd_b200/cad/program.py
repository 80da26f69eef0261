"""Fixed per-GPU task programs of one CAD decode step, and the proof obligations on flags.

attention GPU : for layer, for mb:  pre(l, mb) ; attn(l, mb)
model GPU     : embed ; hqkv(0, *) ; for layer: { hpost(l, mb) ; ffn(l, mb) ; hqkv(l+1, mb) }... ;
                final ; sample

Every hop is "put rows, then release flag = epoch + 1" on the sender and "acquire-wait flag"
on the receiver. ``flag_traffic`` lists, for a program pair, every release and every wait;
``check_balanced`` asserts that each flag is released exactly once and waited exactly once
per step, which is what makes epoch-stamped flags reusable without resets.

Reference: python/minisgl/cad/program.py:53-107.
"""
from __future__ import annotations

from collections import Counter
from dataclasses import dataclass
from typing import List, Tuple


@dataclass(frozen=True)
class Task:
    kind: str           # embed | hqkv | pre | attn | hpost | ffn | final | sample
    layer: int = -1
    mb: int = -1


def attention_program(num_layers: int, num_mb: int) -> List[Task]:
    return [t for l in range(num_layers) for mb in range(num_mb) for t in (Task("pre", l, mb), Task("attn", l, mb))]


def model_program(num_layers: int, num_mb: int) -> List[Task]:
    prog = [Task("embed")] + [Task("hqkv", 0, mb) for mb in range(num_mb)]
    for l in range(num_layers):
        for mb in range(num_mb):
            prog += [Task("hpost", l, mb), Task("ffn", l, mb)]
            if l + 1 < num_layers:
                prog.append(Task("hqkv", l + 1, mb))
    return prog + [Task("final"), Task("sample")]


def flag_traffic(num_layers: int, num_mb: int, attn_ranks: int) -> Tuple[List[tuple], List[tuple]]:
    """(releases, waits) as (flag name, layer, mb, attention rank) tuples for one step."""
    rel, wait = [], []
    for t in model_program(num_layers, num_mb):
        if t.kind == "hqkv":
            rel += [("qkv", t.layer, t.mb, a) for a in range(attn_ranks)]
        elif t.kind == "hpost":
            wait += [("o", t.layer, t.mb, a) for a in range(attn_ranks)]
    for a in range(attn_ranks):
        for t in attention_program(num_layers, num_mb):
            if t.kind == "pre":
                wait.append(("qkv", t.layer, t.mb, a))
            elif t.kind == "attn":
                rel.append(("o", t.layer, t.mb, a))
    return rel, wait


def check_balanced(num_layers: int, num_mb: int, attn_ranks: int) -> None:
    rel, wait = flag_traffic(num_layers, num_mb, attn_ranks)
    cr, cw = Counter(rel), Counter(wait)
    if set(cr) != set(cw):
        raise AssertionError(f"flags released but never waited (or the reverse): {set(cr) ^ set(cw)}")
    bad = [k for k in cr if cr[k] != 1 or cw[k] != 1]
    if bad:
        raise AssertionError(f"flags not released once / waited once per step: {bad[:4]}")
