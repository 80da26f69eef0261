"""Single-process CPU engine: end-to-end generation through scheduler + attention worker +
local experts, against a straightforward full-sequence forward of the same weights."""
import torch

from fastafd_b200.config import PRESETS, RuntimeConfig
from fastafd_b200.core import SamplingParams
from fastafd_b200.engine import AfdEngine, SpmdDriver
from fastafd_b200.protocol import AfdTopology
from fastafd_b200.reference.model_ref import greedy_generate_reference


def _rt(**kw):
    base = dict(model_path="tiny-qwen3-moe", num_mb=2, page_size=16, num_pages=64, max_running_requests=8,
                max_seq_len=128, cuda_graph_max_bs=8, device="cpu", dtype="float32", use_cuda_graph=False)
    base.update(kw)
    return RuntimeConfig(**base)


def test_tiny_moe_generation_matches_full_forward():
    cfg = PRESETS["tiny-qwen3-moe"]
    eng = AfdEngine(cfg, _rt(), AfdTopology(colocated=True), 0, "cpu", seed=0)
    g = torch.Generator().manual_seed(0)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (32, 32, 17, 5)]
    out = SpmdDriver(eng).generate(prompts, SamplingParams(max_tokens=6, ignore_eos=True))
    exp = greedy_generate_reference(cfg, eng.attn.model, [eng.expert_stage], prompts, 6)
    assert out == exp


def test_chunked_prefill_and_single_mb():
    cfg = PRESETS["tiny-qwen3-moe"]
    eng = AfdEngine(cfg, _rt(num_mb=1, max_batched_tokens=16), AfdTopology(colocated=True), 0, "cpu", seed=1, max_comm_tokens=16)
    g = torch.Generator().manual_seed(1)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (40, 9)]
    out = SpmdDriver(eng).generate(prompts, SamplingParams(max_tokens=4, ignore_eos=True))
    exp = greedy_generate_reference(cfg, eng.attn.model, [eng.expert_stage], prompts, 4)
    assert out == exp
