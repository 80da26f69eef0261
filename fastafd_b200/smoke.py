"""One tiny prefill + decode run of the flagship MoE model on ``cuda:0`` through the full
serving path (scheduler, paged KV, ping-pong pipeline, fused dispatch / grouped GEMM / combine
kernels, CUDA graph), checked against the CPU fp32 oracle."""
from __future__ import annotations

import torch


def run_smoke() -> None:
    from .config import PRESETS, RuntimeConfig
    from .core import SamplingParams
    from .engine import AfdEngine, SpmdDriver
    from .protocol import AfdTopology

    cfg = PRESETS["tiny-qwen3-moe"]
    rt = RuntimeConfig(model_path="tiny-qwen3-moe", num_mb=2, page_size=16, num_pages=64, max_running_requests=8,
                       max_seq_len=128, cuda_graph_max_bs=8, device="cuda", moe_block_tok=16)
    eng = AfdEngine(cfg, rt, AfdTopology(colocated=True), 0, "cuda:0", seed=0)
    g = torch.Generator().manual_seed(0)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (32, 32, 20, 7)]
    out = SpmdDriver(eng).generate(prompts, SamplingParams(max_tokens=8, ignore_eos=True))
    assert all(len(o) == 8 for o in out), out
    rt_cpu = RuntimeConfig(model_path="tiny-qwen3-moe", num_mb=2, page_size=16, num_pages=64, max_running_requests=8,
                           max_seq_len=128, cuda_graph_max_bs=8, device="cpu", dtype="float32", use_cuda_graph=False)
    ref_eng = AfdEngine(cfg, rt_cpu, AfdTopology(colocated=True), 0, "cpu", seed=0)
    exp = SpmdDriver(ref_eng).generate(prompts, SamplingParams(max_tokens=8, ignore_eos=True))
    same = sum(a == b for o, e in zip(out, exp) for a, b in zip(o, e))
    total = sum(len(e) for e in exp)
    print(f"smoke: {same}/{total} greedy tokens equal to the CPU fp32 oracle; first request: {out[0]}")
    assert same >= total // 2, (out, exp)
    eng.close()
