"""Prompt bases for long-context benchmarks: `count` prompts of exactly `target_tokens` tokens each.

Two sources, no network:

* ``--source-dir``: every ``*.txt`` file below it is tokenised (``--tokenizer`` = a directory with a
  tokenizer, through `fastafd_b200.tokenizer.load_tokenizer`) and cut into contiguous chunks; a prompt is
  one contiguous chunk of one document, nothing is added to it (no headers, no instructions, no padding).
* without it: token ids with the statistics that matter to a serving engine (a Zipf unigram
  distribution over the vocabulary and locally repeated phrases, so that a radix prefix cache and a
  router see neither uniform noise nor one constant), drawn from ``--seed`` only.

The output is JSON lines ``{"input_ids": [...]}``; `load` reads it back and the HTTP load client takes
it with ``--prompt-file``. The same seed always gives the same file.

Reference: scripts/data_gen/generate_realistic_long_prompts.py (contiguous slices of real documents at a
target token length, deterministic in the seed; that script downloads its corpus).
"""
from __future__ import annotations

import argparse
import json
import random
from pathlib import Path
from typing import Iterable, List, Optional, Sequence


_ZIPF_TABLES: dict = {}


def _zipf_table(usable: int):
    """Cumulative integer weights of ranks 1..usable under a Zipf law with exponent 1 (weight 2^40 // r):
    integers only, so the same seed gives the same prompts on every platform."""
    t = _ZIPF_TABLES.get(usable)
    if t is None:
        cum, total = [], 0
        for r in range(1, usable + 1):
            total += (1 << 40) // r
            cum.append(total)
        t = _ZIPF_TABLES[usable] = (cum, total)
    return t


def zipf_prompt(rng: random.Random, n: int, vocab: int, phrase_prob_pct: int = 15, first_id: int = 16) -> List[int]:
    """n token ids: ranks drawn from a Zipf law (rank r with weight 1/r, mapped to ids scattered over
    the vocabulary), and with probability `phrase_prob_pct` % a phrase of 3-12 tokens seen earlier in
    the same prompt is repeated (natural text re-uses its own n-grams). Integer arithmetic only."""
    import bisect

    usable = max(vocab - first_id, 2)
    cum, total = _zipf_table(usable)
    stride = 2654435761 % usable or 1        # scatter ranks over the id space (a rank is not an id)
    out: List[int] = []
    while len(out) < n:
        if len(out) > 32 and rng.randrange(100) < phrase_prob_pct:
            ln = rng.randint(3, 12)
            st = rng.randrange(0, len(out) - ln)
            out.extend(out[st:st + ln])
        else:
            rank = bisect.bisect_right(cum, rng.randrange(total))
            out.append(first_id + (rank * stride) % usable)
    return out[:n]


def synthetic(count: int, target_tokens: int, vocab: int, seed: int, shared_prefix: int = 0) -> List[List[int]]:
    """`shared_prefix` > 0: every prompt starts with the same tokens (a system prompt), the case a
    prefix cache is built for."""
    rng = random.Random(seed)
    prefix = zipf_prompt(rng, shared_prefix, vocab) if shared_prefix else []
    return [prefix + zipf_prompt(rng, target_tokens - len(prefix), vocab) for _ in range(count)]


def slices_of_documents(docs: Iterable[Sequence[int]], count: int, target_tokens: int, seed: int,
                        min_source_tokens: int = 0) -> List[List[int]]:
    """Contiguous chunks of `target_tokens` tokens, documents taken round-robin so that one long
    document does not fill the whole base; a document shorter than a chunk (or than
    `min_source_tokens`) is skipped."""
    rng = random.Random(seed)
    pool = [list(d) for d in docs if len(d) >= max(target_tokens, min_source_tokens)]
    if not pool:
        raise ValueError(f"no source document has {max(target_tokens, min_source_tokens)} tokens")
    chunks: List[List[List[int]]] = []
    for d in pool:
        off = rng.randrange(0, (len(d) - target_tokens) % target_tokens + 1)
        chunks.append([d[i:i + target_tokens] for i in range(off, len(d) - target_tokens + 1, target_tokens)])
    out: List[List[int]] = []
    i = 0
    while len(out) < count and any(chunks):
        c = chunks[i % len(chunks)]
        if c:
            out.append(c.pop(0))
        i += 1
    if len(out) < count:
        raise ValueError(f"sources yield only {len(out)} chunks of {target_tokens} tokens, {count} wanted")
    return out


def save(prompts: Sequence[Sequence[int]], path: Path) -> None:
    path.parent.mkdir(parents=True, exist_ok=True)
    with open(path, "w") as f:
        for p in prompts:
            f.write(json.dumps({"input_ids": list(p)}) + "\n")


def load(path: str, max_prompts: int = 0, max_tokens: int = 0) -> List[List[int]]:
    out = []
    with open(path) as f:
        for line in f:
            line = line.strip()
            if not line:
                continue
            ids = json.loads(line)["input_ids"]
            out.append(ids[:max_tokens] if max_tokens else ids)
            if max_prompts and len(out) >= max_prompts:
                break
    return out


POOLS_FILE = Path(__file__).with_name("prompt_pools.json")


def pool_name(model: str, isl: int, rows: int) -> str:
    return f"{model}_isl{isl}_r{rows}"


def build_pool(model: str, isl: int, rows: int, out_dir: Path, registry: Optional[dict] = None) -> dict:
    """One prompt pool of a benchmark model: `rows` synthetic prompts of `isl` tokens over the model's
    vocabulary, from the registry's seed. The file's sha256 is compared with the registered one: the
    recorded step times were measured on exactly these prompts (`ok` False = a different file)."""
    import hashlib

    from ..config import get_model_config

    reg = json.loads(POOLS_FILE.read_text()) if registry is None else registry
    name = pool_name(model, isl, rows)
    entry = reg["pools"].get(name, {})
    preset = reg["models"][model]
    seed = int(entry.get("seed", reg.get("seed", 20260527)))
    path = out_dir / (name + ".jsonl")
    save(synthetic(rows, isl, get_model_config(preset).vocab_size, seed), path)
    digest = hashlib.sha256(path.read_bytes()).hexdigest()
    want = entry.get("sha256")
    return {"pool": name, "path": str(path), "sha256": digest, "registered": want, "ok": want in (None, digest)}


def pools_main(argv: Sequence[str]) -> int:
    """python -m fastafd_b200.benchmark.long_prompts build-pools --model qwen3-235b --out DIR --pool 8192:128 ..."""
    ap = argparse.ArgumentParser(prog="fastafd_b200.benchmark.long_prompts build-pools")
    ap.add_argument("--model", required=True, help="a key of prompt_pools.json 'models'")
    ap.add_argument("--out", required=True, type=Path)
    ap.add_argument("--pool", action="append", default=[], help="ISL:ROWS (repeatable)")
    a = ap.parse_args(argv)
    bad = 0
    for spec in a.pool:
        isl, rows = (int(x) for x in spec.split(":"))
        res = build_pool(a.model, isl, rows, a.out)
        print(json.dumps(res))
        bad += 0 if res["ok"] else 1
    return 1 if bad else 0


def main(argv: Optional[Sequence[str]] = None) -> int:
    import sys

    argv = list(sys.argv[1:] if argv is None else argv)
    if argv and argv[0] == "build-pools":
        return pools_main(argv[1:])
    ap = argparse.ArgumentParser(prog="fastafd_b200.benchmark.long_prompts")
    ap.add_argument("--target-tokens", type=int, default=8192)
    ap.add_argument("--count", type=int, default=512)
    ap.add_argument("--output", required=True, type=Path)
    ap.add_argument("--seed", type=int, default=20260527)
    ap.add_argument("--vocab", type=int, default=151936, help="synthetic mode: size of the id space")
    ap.add_argument("--shared-prefix", type=int, default=0, help="synthetic mode: tokens shared by every prompt")
    ap.add_argument("--source-dir", type=Path, default=None, help="slice the *.txt files below this directory instead")
    ap.add_argument("--tokenizer", default="", help="tokenizer directory for --source-dir")
    ap.add_argument("--min-source-tokens", type=int, default=0)
    a = ap.parse_args(argv)
    if a.source_dir is not None:
        from ..tokenizer import load_tokenizer

        tok = load_tokenizer(a.tokenizer)
        docs = [tok.encode(p.read_text(errors="ignore")) for p in sorted(a.source_dir.rglob("*.txt"))]
        prompts = slices_of_documents(docs, a.count, a.target_tokens, a.seed, a.min_source_tokens)
    else:
        prompts = synthetic(a.count, a.target_tokens, a.vocab, a.seed, a.shared_prefix)
    save(prompts, a.output)
    print(json.dumps({"output": str(a.output), "prompts": len(prompts), "tokens_each": a.target_tokens}))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
