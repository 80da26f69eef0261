"""One tiny prefill + decode run of the flagship MoE model on ``cuda:0`` through the full
serving path (scheduler, paged KV, ping-pong pipeline, fused dispatch / grouped GEMM / combine
kernels, CUDA graph). Two checks: the graph-replayed run emits the same tokens as eager
launches, and the eager run's logits match the whole-sequence fp32 reference forward on the same
bf16-rounded weights (teacher-forced on the GPU's tokens; argmax equal wherever the reference's
top-2 gap exceeds the tolerance)."""
from __future__ import annotations

import torch


def run_smoke() -> None:
    from .config import PRESETS, RuntimeConfig
    from .core import SamplingParams
    from .engine import AfdEngine, SpmdDriver
    from .protocol import AfdTopology
    from .reference.model_ref import bf16_rounded_copy, logit_check

    cfg = PRESETS["tiny-qwen3-moe"]
    g = torch.Generator().manual_seed(0)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (32, 31, 20, 7)]
    sp = SamplingParams(max_tokens=8, ignore_eos=True)

    def run(graph: bool, tap: bool):
        rt = RuntimeConfig(model_path="tiny-qwen3-moe", num_mb=2, page_size=16, num_pages=64, max_running_requests=8,
                           max_seq_len=128, cuda_graph_max_bs=8, device="cuda", moe_block_tok=16, use_cuda_graph=graph)
        eng = AfdEngine(cfg, rt, AfdTopology(colocated=True), 0, "cuda:0", seed=0)
        if tap:
            eng.attn.logit_tap = []
        out = SpmdDriver(eng).generate(prompts, sp)
        taps = eng.attn.logit_tap
        eng.close()
        return out, taps

    out, _ = run(graph=True, tap=False)
    assert all(len(o) == 8 for o in out), out
    eager, taps = run(graph=False, tap=True)
    assert eager == out, ("graph replay and eager launches disagree", out, eager)
    rt_cpu = RuntimeConfig(model_path="tiny-qwen3-moe", num_mb=2, page_size=16, num_pages=64, max_running_requests=8,
                           max_seq_len=128, cuda_graph_max_bs=8, device="cpu", dtype="float32", use_cuda_graph=False)
    ref_eng = AfdEngine(cfg, rt_cpu, AfdTopology(colocated=True), 0, "cpu", seed=0)
    stats = logit_check(cfg, bf16_rounded_copy(ref_eng.attn.model), [bf16_rounded_copy(ref_eng.expert_stage)],
                        prompts, eager, taps)
    print(f"smoke: graph == eager tokens; logits vs reference forward: {stats}; first request: {out[0]}")
    assert stats["positions"] == len(prompts) * 8, stats
