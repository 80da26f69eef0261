"""Alignment check of the serving path against the PyTorch oracle.

    python -m fastafd_b200.validate --model tiny-qwen3-moe --prompts 4 --prompt-len 32 --decode 16
    python -m fastafd_b200.validate --model-path /models/Qwen3-30B-A3B --device cuda:0 --decode 8

Generates greedily with the engine (fused kernels, CUDA graphs, micro-batches) and with the
single-process PyTorch model (`reference/model_ref.py`) from the same weights, and reports the
fraction of identical tokens, the first divergence of every prompt, the rank of every served token
in the oracle's logits when the served continuation is teacher-forced through it (top-1 / top-10 /
top-100 hit rates, the reference's alignment gate) and a pass/fail verdict against `--min-match`
and the rank thresholds. On CPU in fp32 the two paths must agree token for token; in bf16 on a GPU
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


def library_reference(model_path: str, prompts, served, decode: int):
    """(greedy continuations of the `transformers` model, rank scores of the served continuations under it).
    Whole-sequence forward passes in fp32 on the CPU, no cache: slow and simple on purpose.
    Reference: scripts/validate/compare_minisgl_vllm.py (alignment against an independent implementation; there vLLM,
    here the library that defines the checkpoint format)."""
    from transformers import AutoModelForCausalLM

    model = AutoModelForCausalLM.from_pretrained(model_path, dtype=torch.float32).eval()
    oracle, ranks = [], []
    with torch.no_grad():
        for p, s in zip(prompts, served):
            ids = list(p)
            for _ in range(decode):
                ids.append(int(model(input_ids=torch.tensor([ids])).logits[0, -1].argmax()))
            oracle.append(ids[len(p):])
            logits = model(input_ids=torch.tensor([list(p) + list(s)])).logits[0]       # teacher-forced on what was served
            r = []
            for i, tok in enumerate(s):
                row = logits[len(p) - 1 + i]
                r.append(int((row > row[tok]).sum()))          # 0 = the library's own greedy choice
            ranks.append(r)
    flat = [x for r in ranks for x in r]
    n = max(len(flat), 1)
    return oracle, {"ranks": ranks, "tokens": len(flat), "top1_agreement_rate": sum(x == 0 for x in flat) / n,
                    "top10_hit_rate": sum(x < 10 for x in flat) / n, "top100_hit_rate": sum(x < 100 for x in flat) / n}


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
    ap.add_argument("--min-top1", type=float, default=-1.0, help="rank gate: share of emitted tokens that are the "
                                                                 "oracle's own choice (default 1.0 on CPU, 0.9 on CUDA)")
    ap.add_argument("--min-top10", type=float, default=0.99, help="rank gate: share within the oracle's top 10")
    ap.add_argument("--min-top100", type=float, default=1.0, help="rank gate: share within the oracle's top 100")
    ap.add_argument("--against", default="oracle", choices=["oracle", "transformers"],
                    help="what the served tokens are compared with: this package's whole-sequence PyTorch forward of the "
                         "same weights, or the `transformers` implementation of the model loading the same directory "
                         "(CPU, fp32): an implementation that shares no code with this package")
    a = ap.parse_args(argv)

    from .config import ModelConfig, RuntimeConfig, get_model_config
    from .core import SamplingParams
    from .engine import AfdEngine, SpmdDriver
    from .protocol import AfdTopology

    cfg = get_model_config(a.model_path or a.model)
    if a.against == "transformers" and not a.model_path:
        ap.error("--against transformers needs --model-path (a checkpoint directory both sides can load)")
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
            return out, ref_out, eng

        finally:
            eng.close()

    if a.against == "transformers":
        served, _, _ = generate(a.device, a.device != "cpu", False)
        oracle, score = library_reference(a.model_path, prompts, served, a.decode)
    else:
        if a.device == "cpu":
            served, oracle, ref_eng = generate("cpu", False, True)
        else:
            served, _, _ = generate(a.device, True, False)
            _, oracle, ref_eng = generate("cpu", False, True)
        # rank gate: the served continuation, teacher-forced through the oracle (the weights outlive close())
        from .reference.model_ref import score_continuations

        score = score_continuations(cfg, ref_eng.attn.model, [ref_eng.expert_stage], prompts, served)
    need1 = a.min_top1 if a.min_top1 >= 0 else (1.0 if a.device == "cpu" else 0.9)
    rank_ok = (score["top1_agreement_rate"] >= need1 and score["top10_hit_rate"] >= a.min_top10
               and score["top100_hit_rate"] >= a.min_top100)
    total = sum(len(o) for o in oracle)
    same = sum(x == y for s, o in zip(served, oracle) for x, y in zip(s, o))
    div = [first_divergence(s, o) for s, o in zip(served, oracle)]
    need = a.min_match if a.min_match >= 0 else (1.0 if a.device == "cpu" else 0.8)
    ok = same >= need * total and rank_ok
    print(json.dumps({"model": a.model_path or a.model, "device": a.device, "against": a.against, "tokens": total, "identical": same,
                      "match": round(same / max(total, 1), 4), "first_divergence": div, "min_match": need,
                      "overall_top1_agreement_rate": round(score["top1_agreement_rate"], 4),
                      "overall_top10_hit_rate": round(score["top10_hit_rate"], 4),
                      "overall_top100_hit_rate": round(score["top100_hit_rate"], 4),
                      "rank_gate": {"min_top1": need1, "min_top10": a.min_top10, "min_top100": a.min_top100,
                                    "worst_rank": max((x for r in score["ranks"] for x in r), default=0)},
                      "verdict": "pass" if ok else "fail"}))
    return 0 if ok else 1


if __name__ == "__main__":
    sys.exit(main())
