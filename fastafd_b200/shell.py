"""Interactive shell: type a prompt, get the completion, keep the conversation.

    python -m fastafd_b200.shell --model-path tiny-qwen3-moe --device cpu --max-tokens 32

Commands: ``/reset`` forgets the conversation, ``/exit`` (or end of input) leaves.
Reference: python/minisgl/shell.py (terminal front end of the engine).
"""
from __future__ import annotations

import argparse
import sys
from typing import List, Optional, Sequence, TextIO

from .core import SamplingParams


def run_shell(llm, max_tokens: int = 64, temperature: float = 0.0, inp: TextIO = sys.stdin,
              out: TextIO = sys.stdout, prompt: str = ">>> ") -> int:
    """Read-eval loop over `llm.generate`; the running conversation (token ids) is the context
    of the next turn. Returns the number of turns answered."""
    history: List[int] = []
    turns = 0
    sp = SamplingParams(max_tokens=max_tokens, temperature=temperature)
    while True:
        out.write(prompt)
        out.flush()
        line = inp.readline()
        if not line:
            break
        line = line.strip()
        if not line:
            continue
        if line in ("/exit", "/quit"):
            break
        if line == "/reset":
            history = []
            out.write("(conversation cleared)\n")
            continue
        ids = list(llm.tokenizer.encode(line))
        room = llm.rt.max_seq_len - max_tokens - 1
        ctx = (history + ids)[-max(room, 1):]          # keep the most recent tokens that fit
        res = llm.generate([ctx], sp)[0]
        history = ctx + list(res["token_ids"])
        out.write(str(res["text"]) + "\n")
        turns += 1
    return turns


def main(argv: Optional[Sequence[str]] = None) -> int:
    ap = argparse.ArgumentParser(prog="fastafd_b200.shell")
    ap.add_argument("--model-path", "--model", dest="model_path", default="tiny-qwen3-moe")
    ap.add_argument("--device", default=None)
    ap.add_argument("--max-tokens", type=int, default=64)
    ap.add_argument("--temperature", type=float, default=0.0)
    ap.add_argument("--max-seq-len", type=int, default=0)
    a = ap.parse_args(argv)
    from .llm import LLM

    kw = {"max_seq_len": a.max_seq_len} if a.max_seq_len else {}
    llm = LLM(a.model_path, device=a.device, **kw)
    run_shell(llm, a.max_tokens, a.temperature)
    return 0


if __name__ == "__main__":
    sys.exit(main())
