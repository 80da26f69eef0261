"""Load-generating client for the HTTP server: sends `n` requests with random token ids over
``/v1/chat/completions`` (the ``input_ids`` extension), records the arrival time of every
streamed chunk, and reports time to first token (TTFT), time per output token (TPOT) and
throughput.

    python -m fastafd_b200.benchmark.client --port 1919 --num 64 --prompt-len 1024 --max-tokens 128

A recorded arrival trace can be replayed instead of a closed batch:

    python -m fastafd_b200.benchmark.client --port 1919 --trace trace.jsonl --time-scale 0.5 --max-requests 200

Trace lines are JSON objects with ``timestamp`` (ms since the first request), ``input_length`` and
``output_length`` (the Mooncake / Qwen trace layout); prompts are random ids of the recorded lengths.

Reference: python/minisgl/benchmark/client.py:18-60 (per-request tick lists), :407-500 (trace
readers and scaling), perf.py.
"""
from __future__ import annotations

import argparse
import asyncio
import json
import random
import time
from dataclasses import dataclass, field
from typing import List, Optional


@dataclass
class RequestTrace:
    start: float
    ticks: List[float] = field(default_factory=list)     # arrival time of each content chunk
    tokens: int = 0
    error: str = ""

    @property
    def ttft(self) -> float:
        return self.ticks[0] - self.start if self.ticks else float("nan")

    @property
    def tpot(self) -> float:
        if len(self.ticks) < 2:
            return float("nan")
        return (self.ticks[-1] - self.ticks[0]) / (len(self.ticks) - 1)


@dataclass(frozen=True)
class TraceEntry:
    at_s: float           # arrival offset from the start of the replay
    input_length: int
    output_length: int


def read_trace(path: str) -> List[TraceEntry]:
    """One JSON object per line: timestamp (ms), input_length, output_length. Lines that lack a
    field or have non-positive lengths are skipped; arrivals are re-based to start at 0."""
    out = []
    with open(path) as f:
        for line in f:
            line = line.strip()
            if not line:
                continue
            try:
                o = json.loads(line)
                e = TraceEntry(float(o["timestamp"]) / 1e3, int(o["input_length"]), int(o["output_length"]))
            except (ValueError, KeyError, TypeError):
                continue
            if e.input_length > 0 and e.output_length > 0:
                out.append(e)
    out.sort(key=lambda e: e.at_s)
    t0 = out[0].at_s if out else 0.0
    return [TraceEntry(e.at_s - t0, e.input_length, e.output_length) for e in out]


def scale_trace(entries: List[TraceEntry], time_scale: float = 1.0, max_requests: int = 0, max_input: int = 0,
                max_output: int = 0) -> List[TraceEntry]:
    """Compress or stretch arrivals by `time_scale` (0.5 = twice the request rate), keep the first
    `max_requests`, and clip lengths to what the server under test accepts."""
    out = entries[:max_requests] if max_requests > 0 else list(entries)
    return [TraceEntry(e.at_s * time_scale, min(e.input_length, max_input) if max_input > 0 else e.input_length,
                       min(e.output_length, max_output) if max_output > 0 else e.output_length) for e in out]


def summarize(traces: List[RequestTrace], wall_s: float) -> dict:
    ok = [t for t in traces if not t.error and t.ticks]
    def pct(xs, p):
        xs = sorted(x for x in xs if x == x)
        return xs[min(len(xs) - 1, int(p * len(xs)))] if xs else float("nan")
    ttft = [t.ttft for t in ok]
    tpot = [t.tpot for t in ok]
    toks = sum(t.tokens for t in ok)
    return {"requests": len(traces), "failed": len(traces) - len(ok), "output_tokens": toks, "wall_s": round(wall_s, 3),
            "tok_per_s": round(toks / wall_s, 2) if wall_s > 0 else 0.0,
            "ttft_ms_p50": round(pct(ttft, 0.5) * 1e3, 2), "ttft_ms_p99": round(pct(ttft, 0.99) * 1e3, 2),
            "tpot_ms_p50": round(pct(tpot, 0.5) * 1e3, 3), "tpot_ms_p99": round(pct(tpot, 0.99) * 1e3, 3)}


async def _one(session, url: str, ids: List[int], max_tokens: int) -> RequestTrace:
    tr = RequestTrace(start=time.perf_counter())
    body = {"input_ids": ids, "max_tokens": max_tokens, "temperature": 0, "ignore_eos": True, "return_token_ids": True}
    try:
        async with session.post(url, json=body) as resp:
            async for raw in resp.content:
                line = raw.decode().strip()
                if not line.startswith("data: "):
                    continue
                payload = line[6:]
                if payload == "[DONE]":
                    break
                obj = json.loads(payload)
                if "error" in obj:
                    tr.error = obj["error"]
                    break
                ids_out = obj["choices"][0].get("token_ids") or []
                if ids_out:
                    tr.ticks.append(time.perf_counter())
                    tr.tokens += len(ids_out)
    except Exception as e:  # connection errors are part of the report, not a crash
        tr.error = f"{type(e).__name__}: {e}"
    return tr


async def run(host: str, port: int, num: int, prompt_len: int, max_tokens: int, vocab: int, seed: int = 0,
              prompts: Optional[List[List[int]]] = None) -> dict:
    """A closed batch of `num` requests sent at once. `prompts`: token ids to send (cycled when there
    are fewer than `num`), e.g. a prompt base of benchmark/long_prompts.py; else uniform random ids."""
    import aiohttp

    rng = random.Random(seed)
    url = f"http://{host}:{port}/v1/chat/completions"
    t0 = time.perf_counter()
    async with aiohttp.ClientSession(timeout=aiohttp.ClientTimeout(total=None)) as s:
        traces = await asyncio.gather(*[_one(s, url, prompts[i % len(prompts)] if prompts else
                                             [rng.randrange(vocab) for _ in range(prompt_len)], max_tokens)
                                        for i in range(num)])
    return summarize(list(traces), time.perf_counter() - t0)


async def replay(host: str, port: int, entries: List[TraceEntry], vocab: int, seed: int = 0) -> dict:
    """Open-loop replay: every request is sent at its recorded arrival time whatever the state of
    the earlier ones."""
    import aiohttp

    rng = random.Random(seed)
    url = f"http://{host}:{port}/v1/chat/completions"
    t0 = time.perf_counter()

    async def later(session, e: TraceEntry):
        await asyncio.sleep(max(0.0, e.at_s - (time.perf_counter() - t0)))
        return await _one(session, url, [rng.randrange(vocab) for _ in range(e.input_length)], e.output_length)

    async with aiohttp.ClientSession(timeout=aiohttp.ClientTimeout(total=None)) as s:
        traces = await asyncio.gather(*[later(s, e) for e in entries])
    return summarize(list(traces), time.perf_counter() - t0)


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=1919)
    ap.add_argument("--num", type=int, default=32)
    ap.add_argument("--prompt-len", type=int, default=128)
    ap.add_argument("--max-tokens", type=int, default=32)
    ap.add_argument("--vocab", type=int, default=1024)
    ap.add_argument("--prompt-file", default="", help="JSON lines of {input_ids}: a prompt base of benchmark/long_prompts.py")
    ap.add_argument("--trace", default="", help="JSONL arrival trace to replay instead of a closed batch")
    ap.add_argument("--time-scale", type=float, default=1.0)
    ap.add_argument("--max-requests", type=int, default=0)
    ap.add_argument("--max-input", type=int, default=0)
    ap.add_argument("--max-output", type=int, default=0)
    a = ap.parse_args(argv)
    if a.trace:
        entries = scale_trace(read_trace(a.trace), a.time_scale, a.max_requests, a.max_input, a.max_output)
        print(json.dumps(asyncio.run(replay(a.host, a.port, entries, a.vocab))))
        return
    prompts = None
    if a.prompt_file:
        from .long_prompts import load

        prompts = load(a.prompt_file, max_prompts=a.num, max_tokens=a.max_input)
    print(json.dumps(asyncio.run(run(a.host, a.port, a.num, a.prompt_len, a.max_tokens, a.vocab, prompts=prompts))))


if __name__ == "__main__":
    main()
