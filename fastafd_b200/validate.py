"""Alignment check of the serving path against the PyTorch oracle.

    python -m fastafd_b200.validate --model tiny-qwen3-moe --prompts 4 --prompt-len 32 --decode 16
    python -m fastafd_b200.validate --model-path /models/Qwen3-30B-A3B --device cuda:0 --decode 8

Generates greedily with the engine (fused kernels, CUDA graphs, micro-batches) and with the
single-process PyTorch model (`reference/model_ref.py`) from the same weights, and reports the
fraction of identical tokens, the first divergence of every prompt and a pass/fail verdict
against `--min-match`. On CPU in fp32 the two paths must agree token for token; in bf16 on a GPU
near-ties in the logits may flip a token, after which the continuations differ, so the
comparison there is by prefix.
Reference: scripts/validate (alignment of the reference against vLLM); here the oracle is the
PyTorch model, since no second serving stack exists in the image.
"""
from __future__ import annotations

import argparse
import json
import sys

import torch


def first_divergence(a, b) -> int:
    for i, (x, y) in enumerate(zip(a, b)):
        if x != y:
            return i
    return min(len(a), len(b))


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="fastafd_b200.validate")
    ap.add_argument("--model", default="tiny-qwen3-moe", help="preset name (random-init weights)")
    ap.add_argument("--model-path", default="", help="HF checkpoint directory (overrides --model)")
    ap.add_argument("--device", default="cuda:0" if torch.cuda.is_available() else "cpu")
    ap.add_argument("--prompts", type=int, default=4)
    ap.add_argument("--prompt-len", type=int, default=32)
    ap.add_argument("--decode", type=int, default=16)
    ap.add_argument("--num-mb", type=int, default=2)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--min-match", type=float, default=-1.0, help="default: 1.0 on CPU, 0.8 on CUDA")
    a = ap.parse_args(argv)

    from .config import ModelConfig, RuntimeConfig, get_model_config
    from .core import SamplingParams
    from .engine import AfdEngine, SpmdDriver
    from .protocol import AfdTopology

    cfg = ModelConfig.from_hf(a.model_path) if a.model_path else get_model_config(a.model)
    g = torch.Generator().manual_seed(a.seed)
    prompts = [torch.randint(0, cfg.vocab_size, (a.prompt_len,), generator=g).tolist() for _ in range(a.prompts)]
    sp = SamplingParams(max_tokens=a.decode, ignore_eos=True)

    def generate(device: str, graph: bool, with_oracle: bool):
        rt = RuntimeConfig(model_path=a.model_path or a.model, num_mb=a.num_mb, page_size=16,
                           max_running_requests=max(a.prompts, 2), max_seq_len=a.prompt_len + a.decode + 16,
                           cuda_graph_max_bs=max(a.prompts, 2), device=device,
                           dtype="float32" if device == "cpu" else "bfloat16", use_cuda_graph=graph, moe_block_tok=16)
        eng = AfdEngine(cfg, rt, AfdTopology(colocated=True), 0, device, seed=a.seed)
        try:
            out = SpmdDriver(eng).generate(prompts, sp)
            ref_out = None
            if with_oracle:
                # the plain full-sequence forward of the same weights (no paging, no micro-batches)
                from .reference.model_ref import greedy_generate_reference

                ref_out = greedy_generate_reference(cfg, eng.attn.model, [eng.expert_stage], prompts, a.decode)
            return out, ref_out
        finally:
            eng.close()

    if a.device == "cpu":
        served, oracle = generate("cpu", False, True)
    else:
        served, _ = generate(a.device, True, False)
        _, oracle = generate("cpu", False, True)
    total = sum(len(o) for o in oracle)
    same = sum(x == y for s, o in zip(served, oracle) for x, y in zip(s, o))
    div = [first_divergence(s, o) for s, o in zip(served, oracle)]
    need = a.min_match if a.min_match >= 0 else (1.0 if a.device == "cpu" else 0.8)
    ok = same >= need * total
    print(json.dumps({"model": a.model_path or a.model, "device": a.device, "tokens": total, "identical": same,
                      "match": round(same / max(total, 1), 4), "first_divergence": div, "min_match": need,
                      "verdict": "pass" if ok else "fail"}))
    return 0 if ok else 1


if __name__ == "__main__":
    sys.exit(main())
