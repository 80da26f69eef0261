"""Load-generating client for the HTTP server: sends `n` requests with random token ids over
``/v1/chat/completions`` (the ``input_ids`` extension), records the arrival time of every
streamed chunk, and reports time to first token (TTFT), time per output token (TPOT) and
throughput.

    python -m fastafd_b200.benchmark.client --port 1919 --num 64 --prompt-len 1024 --max-tokens 128

Reference: python/minisgl/benchmark/client.py:18-60 (per-request tick lists), perf.py.
"""
from __future__ import annotations

import argparse
import asyncio
import json
import random
import statistics
import time
from dataclasses import dataclass, field
from typing import List


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


async def run(host: str, port: int, num: int, prompt_len: int, max_tokens: int, vocab: int, seed: int = 0) -> dict:
    import aiohttp

    rng = random.Random(seed)
    url = f"http://{host}:{port}/v1/chat/completions"
    t0 = time.perf_counter()
    async with aiohttp.ClientSession(timeout=aiohttp.ClientTimeout(total=None)) as s:
        traces = await asyncio.gather(*[_one(s, url, [rng.randrange(vocab) for _ in range(prompt_len)], max_tokens)
                                        for _ in range(num)])
    return summarize(list(traces), time.perf_counter() - t0)


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=1919)
    ap.add_argument("--num", type=int, default=32)
    ap.add_argument("--prompt-len", type=int, default=128)
    ap.add_argument("--max-tokens", type=int, default=32)
    ap.add_argument("--vocab", type=int, default=1024)
    a = ap.parse_args(argv)
    print(json.dumps(asyncio.run(run(a.host, a.port, a.num, a.prompt_len, a.max_tokens, a.vocab))))


if __name__ == "__main__":
    main()
