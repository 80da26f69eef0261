"""Speculative decoding: acceptance rule, simulated acceptance, and the end-to-end property
that greedy verification is lossless (same tokens as plain greedy decoding), on CPU."""
import numpy as np
import pytest
import torch

from fastafd_b200.config import PRESETS, RuntimeConfig
from fastafd_b200.core import SamplingParams
from fastafd_b200.engine import AfdEngine, SpmdDriver
from fastafd_b200.protocol import AfdTopology
from fastafd_b200.reference import ops_ref as ref
from fastafd_b200.spec.attn_side import simulated_accept


def test_greedy_accept_rule():
    target = torch.tensor([[5, 6, 7, 8], [5, 6, 7, 8], [1, 2, 3, 4]])
    draft = torch.tensor([[5, 6, 7], [5, 9, 7], [0, 2, 3]])
    n, emitted = ref.greedy_accept(draft, target)
    assert n.tolist() == [4, 2, 1]
    assert emitted.tolist() == [[5, 6, 7, 8], [5, 6, -1, -1], [1, -1, -1, -1]]


def test_simulated_acceptance_mean():
    rng = np.random.default_rng(0)
    n = simulated_accept(20000, 4, 1.8, rng)
    assert n.min() >= 1 and n.max() <= 2 and abs(n.mean() - 1.8) < 0.02
    assert simulated_accept(10, 4, 9.0, rng).max() == 4


def _rt(**kw):
    base = dict(model_path="tiny-qwen3-moe", num_mb=2, page_size=16, num_pages=96, max_running_requests=8,
                max_seq_len=160, cuda_graph_max_bs=8, device="cpu", dtype="float32", use_cuda_graph=False)
    base.update(kw)
    return RuntimeConfig(**base)


@pytest.mark.parametrize("block", [2, 4])
def test_speculative_greedy_output_equals_plain_greedy(block):
    cfg = PRESETS["tiny-qwen3-moe"]
    g = torch.Generator().manual_seed(0)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (30, 7, 18)]
    sp = SamplingParams(max_tokens=11, ignore_eos=True)
    plain = SpmdDriver(AfdEngine(cfg, _rt(), AfdTopology(colocated=True), 0, "cpu", seed=0)).generate(prompts, sp)
    eng = AfdEngine(cfg, _rt(spec_block=block), AfdTopology(colocated=True), 0, "cpu", seed=0)
    spec = SpmdDriver(eng).generate(prompts, sp)
    assert spec == plain
    assert eng.attn.spec.accept_hist.sum() > 0 and 1.0 <= eng.attn.spec.mean_accept() <= block


def test_self_draft_accepts_everything():
    """With a draft that always proposes what the target will say (here: drafts planted from a
    plain run), every block is accepted in full."""
    target = torch.tensor([[3, 4, 5, 6]])
    n, _ = ref.greedy_accept(target[:, :3], target)
    assert n.tolist() == [4]


def test_spec_config_from_flags_and_environment(monkeypatch):
    from fastafd_b200.server.args import parse_args
    from fastafd_b200.spec.config import SpecConfig, SpecConfigError

    for k in ("FASTAFD_SPEC", "FASTAFD_SPEC_BLOCK", "FASTAFD_SPEC_DRAFT", "FASTAFD_SPEC_SIM_ACCEPT", "MINISGL_AFD_SPEC"):
        monkeypatch.delenv(k, raising=False)
    assert SpecConfig.from_env() == SpecConfig()                                   # off by default
    c = SpecConfig.from_env(block_flag=4, draft_flag="/d")
    assert c.enabled and c.block == 4 and c.num_draft_tokens == 3 and c.draft_path == "/d"
    monkeypatch.setenv("MINISGL_AFD_SPEC", "1")                                    # the reference's name works too
    monkeypatch.setenv("FASTAFD_SPEC_BLOCK", "8")
    monkeypatch.setenv("FASTAFD_SPEC_SIM_ACCEPT", "1.8")
    c = SpecConfig.from_env()
    assert c.enabled and c.block == 8 and c.sim_accept == 1.8
    a = parse_args(["--model-path", "tiny-qwen3-moe", "--device", "cpu"])
    assert a.spec_block == 8                                                       # environment reached the server flags
    assert parse_args(["--model-path", "tiny-qwen3-moe", "--device", "cpu", "--spec-block", "2"]).spec_block == 2
    monkeypatch.setenv("FASTAFD_SPEC_SIM_ACCEPT", "9.5")
    with pytest.raises(SpecConfigError):
        SpecConfig.from_env()
    monkeypatch.setenv("FASTAFD_SPEC_SIM_ACCEPT", "0")
    monkeypatch.setenv("FASTAFD_SPEC_BLOCK", "1")
    with pytest.raises(SpecConfigError):
        SpecConfig.from_env()


def test_verify_steps_planned_ahead_stay_lossless():
    """The coordinator keeps two verify steps in flight: step n+1 is planned before the acceptance of
    step n is known (the committed lengths live with the attention worker, the scheduler only keeps an
    upper bound and reserves KV for it). The output must still be plain greedy decoding."""
    from fastafd_b200.coordinator import AfdCoordinator, InProcTransport

    cfg = PRESETS["tiny-qwen3-moe"]
    g = torch.Generator().manual_seed(3)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (21, 9, 30, 14)]
    sp = SamplingParams(max_tokens=13, ignore_eos=True)
    plain = SpmdDriver(AfdEngine(cfg, _rt(), AfdTopology(colocated=True), 0, "cpu", seed=0)).generate(prompts, sp)
    rt = _rt(spec_block=4, async_pending_steps=3)
    eng = AfdEngine(cfg, rt, AfdTopology(colocated=True), 0, "cpu", seed=0)

    class Deferred(InProcTransport):
        """Executes a step when it is sent (like a worker queueing it on the GPU) but hands the reply
        over only when the coordinator polls after it has filled its window."""

    got = {i: [] for i in range(len(prompts))}
    coord = AfdCoordinator(cfg, rt, AfdTopology(colocated=True), Deferred({0: eng}), num_pages=96,
                           max_comm_tokens=eng.max_comm_tokens,
                           on_tokens=lambda items: [got[u].extend(t) for u, t, _ in items])
    assert coord.pending == 2
    seen_two_in_flight = False
    for i, p in enumerate(prompts):
        coord.add_request(i, p, sp)
    while not coord.idle():
        coord.step_loop_once(block=True)
        seen_two_in_flight |= len(coord.inflight) >= 1 and any(r.phase == "verify" for r in coord.inflight)
    assert [got[i] for i in range(len(prompts))] == plain
    assert seen_two_in_flight
    # acceptance statistics: every token but each request's first (sampled by its prefill) came out of a verify step
    st = coord.spec_stats()
    assert st["verify_steps"] > 0 and st["tokens"] == sum(len(t) - 1 for t in plain)
    assert 1.0 <= st["mean_accepted"] <= 4.0 and st["rows"] <= st["tokens"]
