"""Coordinator behaviour on CPU: overlap window, dummy lanes, admission, failure detection
(injected on the host: a fake worker that stops replying, a worker that reports an error
status), admission stall, shutdown idempotence."""
import numpy as np
import pytest
import torch

from fastafd_b200.config import PRESETS, RuntimeConfig
from fastafd_b200.coordinator import AfdCoordinator, CoordinatorError, InProcTransport, WorkerTransport
from fastafd_b200.core import SamplingParams
from fastafd_b200.engine import AfdEngine, SpmdDriver
from fastafd_b200.protocol import AfdTopology, AgStepReply, EgStepReply, WorkerFailure
from fastafd_b200.scheduler.lane import AdmissionError


def _rt(**kw):
    base = dict(model_path="tiny-qwen3-moe", num_mb=2, page_size=16, num_pages=64, max_running_requests=8,
                max_seq_len=128, cuda_graph_max_bs=8, device="cpu", dtype="float32", use_cuda_graph=False)
    base.update(kw)
    return RuntimeConfig(**base)


class FakeWorkers(WorkerTransport):
    """Workers that answer every plan with token 7 (or misbehave on request)."""

    def __init__(self, drop_rank=None, bad_status_rank=None, fail_rank=None):
        self.out, self.drop_rank, self.bad_status_rank, self.fail_rank = [], drop_rank, bad_status_rank, fail_rank
        self.sent = []

    def send_step(self, step_id, ag_plans, eg_plans):
        self.sent.append((step_id, sorted(ag_plans), sorted(eg_plans)))
        for r, (plan, _) in ag_plans.items():
            if r == self.drop_rank:
                continue
            if r == self.fail_rank:
                self.out.append(WorkerFailure(rank=r, error="boom"))
                continue
            n = sum(len(mb.rows) for mb in plan.mbs)
            self.out.append(AgStepReply(step_id=step_id, rank=r, next_tokens=np.full(n, 7, np.int32),
                                        status=2 if r == self.bad_status_rank else 0))
        for r in eg_plans:
            self.out.append(EgStepReply(step_id=step_id, rank=r))

    def poll(self, timeout_s):
        out, self.out = self.out, []
        return out


def test_coordinator_matches_spmd_driver_on_cpu_engine():
    cfg = PRESETS["tiny-qwen3-moe"]
    g = torch.Generator().manual_seed(0)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (20, 33, 5)]
    sp = SamplingParams(max_tokens=5, ignore_eos=True)
    exp = SpmdDriver(AfdEngine(cfg, _rt(), AfdTopology(colocated=True), 0, "cpu", seed=0)).generate(prompts, sp)
    eng = AfdEngine(cfg, _rt(), AfdTopology(colocated=True), 0, "cpu", seed=0)
    got = {i: [] for i in range(len(prompts))}
    coord = AfdCoordinator(cfg, _rt(async_pending_steps=1), AfdTopology(colocated=True), InProcTransport({0: eng}),
                           num_pages=64, max_comm_tokens=eng.max_comm_tokens,
                           on_tokens=lambda items: [got[u].extend(t) for u, t, _ in items])
    for i, p in enumerate(prompts):
        coord.add_request(i, p, sp)
    coord.run_until_idle()
    assert [got[i] for i in range(len(prompts))] == exp


def test_overlap_window_dummy_lanes_and_completion():
    cfg = PRESETS["tiny-qwen3-moe"]
    topo = AfdTopology(attn_dp=2, mlp_ep=2)
    fake = FakeWorkers()
    done = []
    coord = AfdCoordinator(cfg, _rt(async_pending_steps=3), topo, fake, num_pages=64,
                           on_tokens=lambda items: done.extend(items))
    coord.add_request(0, [1, 2, 3], SamplingParams(max_tokens=4, ignore_eos=True))   # only lane 0 gets work
    coord.run_until_idle()
    toks = [t for u, ts, _ in done for t in ts]
    assert toks == [7, 7, 7, 7] and done[-1][2] is True
    # every step went to all four ranks even though lane 1 had nothing to do
    assert all(ag == [0, 1] and eg == [2, 3] for _, ag, eg in fake.sent)
    # 1 prefill + 3 decode steps, no extra step planned past max_tokens
    assert len(fake.sent) == 4
    for l in coord.lanes:
        l.check_integrity()
        assert l.cache.free_pages == 63 and len(l.free_rows) == 8


def test_eos_found_late_drops_tokens_planned_ahead():
    cfg = PRESETS["tiny-qwen3-moe"]
    from dataclasses import replace
    cfg = replace(cfg, eos_token_ids=(7,))
    fake = FakeWorkers()
    done = []
    coord = AfdCoordinator(cfg, _rt(async_pending_steps=3), AfdTopology(attn_dp=1, mlp_ep=1), fake, num_pages=64,
                           on_tokens=lambda items: done.extend(items))
    coord.add_request(0, [1, 2, 3], SamplingParams(max_tokens=16))
    coord.run_until_idle()
    assert [t for _, ts, _ in done for t in ts] == [7]      # EOS right away; later planned steps ignored
    assert coord.lanes[0].cache.free_pages == 63


def test_silent_worker_is_reported_not_waited_for_forever():
    cfg = PRESETS["tiny-qwen3-moe"]
    coord = AfdCoordinator(cfg, _rt(), AfdTopology(attn_dp=2, mlp_ep=2), FakeWorkers(drop_rank=1), num_pages=64,
                           worker_timeout_s=0.3)
    coord.add_request(0, [1, 2, 3], SamplingParams(max_tokens=2, ignore_eos=True))
    with pytest.raises(CoordinatorError, match=r"no reply from ranks \[1\]"):
        coord.run_until_idle()
    assert "no reply" in coord.get_failure()


@pytest.mark.parametrize("kw,msg", [(dict(bad_status_rank=0), "device status 2"), (dict(fail_rank=1), "worker 1 failed: boom")])
def test_worker_error_surfaces(kw, msg):
    cfg = PRESETS["tiny-qwen3-moe"]
    coord = AfdCoordinator(cfg, _rt(), AfdTopology(attn_dp=2, mlp_ep=2), FakeWorkers(**kw), num_pages=64)
    coord.add_request(0, [1, 2, 3], SamplingParams(max_tokens=2, ignore_eos=True))
    with pytest.raises(CoordinatorError, match=msg):
        coord.run_until_idle()
    with pytest.raises(CoordinatorError):
        coord.add_request(1, [1], SamplingParams())


def test_admission_errors_and_stall():
    cfg = PRESETS["tiny-qwen3-moe"]
    coord = AfdCoordinator(cfg, _rt(num_pages=4), AfdTopology(attn_dp=1, mlp_ep=1), FakeWorkers(), num_pages=4)
    with pytest.raises(AdmissionError):
        coord.add_request(0, list(range(100)), SamplingParams(max_tokens=100))   # > max_seq_len
    with pytest.raises(AdmissionError):
        coord.add_request(1, list(range(40)), SamplingParams(max_tokens=40))     # more pages than the lane has


def test_shutdown_is_idempotent():
    class T(FakeWorkers):
        stops = 0

        def stop(self):
            self.stops += 1
    t = T()
    coord = AfdCoordinator(PRESETS["tiny-qwen3-moe"], _rt(), AfdTopology(attn_dp=1, mlp_ep=1), t, num_pages=8)
    coord.shutdown()
    coord.shutdown()
    assert t.stops == 1


@pytest.mark.parametrize("kw,want", [(dict(async_pending_steps=3), 3), (dict(async_pending_steps=0), 1),
                                     (dict(async_pending_steps=3, disable_overlap=True), 1),
                                     (dict(async_pending_steps=3, spec_block=4), 2),
                                     (dict(async_pending_steps=1, spec_block=4), 1)])
def test_overlap_policy_steps_in_flight(kw, want):
    """--afd-async-pending-steps steps are planned ahead; --afd-disable-overlap keeps one in flight;
    speculative decoding keeps at most two (the committed lengths live on the attention GPUs)."""
    from fastafd_b200.server.args import parse_args

    coord = AfdCoordinator(PRESETS["tiny-qwen3-moe"], _rt(**kw), AfdTopology(colocated=True), FakeWorkers(),
                           num_pages=64, max_comm_tokens=64)
    assert coord.pending == want
    a = parse_args(["--mode", "afd-serve", "--model-path", "tiny-qwen3-moe", "--device", "cpu", "--afd-disable-overlap",
                    "--afd-async-pending-steps", "3"])
    assert a.runtime_config().disable_overlap and a.runtime_config().async_pending_steps == 3


class RandomWorkers(WorkerTransport):
    """Workers that answer with random tokens, out of order and late: a reply is released only after a
    random number of polls, expert replies and attention replies of one step in any order."""

    def __init__(self, seed):
        import random

        self.rng, self.waiting = random.Random(seed), []

    def send_step(self, step_id, ag_plans, eg_plans):
        for r, (plan, _) in ag_plans.items():
            n = sum(len(mb.rows) for mb in plan.mbs)
            toks = np.array([self.rng.choice([3, 7, 8, 9]) for _ in range(n)], np.int32)
            self.waiting.append([self.rng.randint(0, 3), AgStepReply(step_id=step_id, rank=r, next_tokens=toks, status=0)])
        for r in eg_plans:
            self.waiting.append([self.rng.randint(0, 3), EgStepReply(step_id=step_id, rank=r)])

    def poll(self, timeout_s):
        out = []
        for item in self.waiting:
            item[0] -= 1
        self.rng.shuffle(self.waiting)
        out = [m for d, m in self.waiting if d < 0]
        self.waiting = [it for it in self.waiting if it[0] >= 0]
        return out


@pytest.mark.parametrize("seed,cache", [(1, "naive"), (2, "radix"), (3, "naive")])
def test_coordinator_soak_over_three_lanes(monkeypatch, seed, cache):
    """Three attention lanes + two expert ranks, three steps in flight, replies late and out of order,
    arrivals and aborts while steps are outstanding, page audit on in every lane: every request that was
    not aborted gets all its tokens exactly once and in the end every lane is empty."""
    import random

    monkeypatch.setenv("FASTAFD_PAGE_AUDIT", "1")
    rng = random.Random(seed)
    cfg = PRESETS["tiny-qwen3-moe"]
    topo = AfdTopology(attn_dp=3, mlp_ep=2)
    got, done = {}, set()

    def on_tokens(items):
        for uid, toks, fin in items:
            assert uid not in done, "tokens after the request finished"
            got[uid] += toks
            if fin:
                done.add(uid)

    coord = AfdCoordinator(cfg, _rt(async_pending_steps=3, cache_type=cache, max_batched_tokens=48), topo, RandomWorkers(seed),
                           num_pages=64, max_comm_tokens=64, on_tokens=on_tokens)
    limits, aborted, uid = {}, set(), 0
    shared = [40 + i for i in range(10)]
    for it in range(4000):
        if uid < 45 and rng.random() < 0.3:
            ids = (shared if rng.random() < 0.5 else []) + [rng.randrange(10, 30) for _ in range(rng.randint(1, 40))]
            sp = SamplingParams(max_tokens=rng.randint(1, 10), ignore_eos=rng.random() < 0.6)
            got[uid], limits[uid] = [], sp
            coord.add_request(uid, ids, sp)
            uid += 1
        live = [u for u in got if u not in done and u not in aborted]
        if live and rng.random() < 0.03:
            u = rng.choice(live)
            coord.abort(u)
            aborted.add(u)
        coord.step_loop_once(block=False)
        assert coord.get_failure() is None
        if uid >= 45 and coord.idle():
            break
    else:
        raise AssertionError("the coordinator did not drain")
    for u, sp in limits.items():
        if u in aborted:
            continue
        assert u in done and 1 <= len(got[u]) <= sp.max_tokens
        assert len(got[u]) == sp.max_tokens or (got[u][-1] in cfg.eos_token_ids and not sp.ignore_eos)
    for lane in coord.lanes:
        lane.audit_pages()
        assert not lane.states
    coord.shutdown()


def test_reply_latency_is_kept_per_rank_and_logged_at_shutdown(caplog):
    topo = AfdTopology(attn_dp=2, mlp_ep=2)
    coord = AfdCoordinator(PRESETS["tiny-qwen3-moe"], _rt(), topo, FakeWorkers(), num_pages=64, max_comm_tokens=64)
    coord.log_step_times = True
    coord.add_request(0, [1, 2, 3], SamplingParams(max_tokens=3, ignore_eos=True))
    coord.run_until_idle()
    summary = coord.latency_summary()
    assert sorted(summary) == [0, 1, 2, 3]                      # both attention ranks and both expert ranks
    assert all(v["replies"] == len(coord.step_times) and 0 <= v["mean_ms"] <= v["max_ms"] for v in summary.values())
    assert coord.spec_stats() == {"verify_steps": 0, "rows": 0, "tokens": 0, "mean_accepted": 0.0}
    import logging
    with caplog.at_level(logging.INFO):
        coord.shutdown()
    assert any("reply latency per rank" in r.getMessage() for r in caplog.records)


def test_hybrid_models_refuse_the_prefix_cache():
    """The recurrent state of linear-attention layers at the end of a cached prefix is kept nowhere, so a prefix hit
    would continue from a wrong state: refused at construction, by the coordinator and by the SPMD driver alike."""
    import dataclasses

    from fastafd_b200.config import get_model_config

    hybrid = dataclasses.replace(get_model_config("qwen3.5-397b-a17b-fp8"), num_layers=4, layer_types=("linear", "linear", "linear", "full"))
    topo = AfdTopology(attn_dp=1, mlp_ep=1)
    with pytest.raises(ValueError, match="cache-type naive"):
        AfdCoordinator(hybrid, _rt(cache_type="radix"), topo, FakeWorkers(), num_pages=64)
    AfdCoordinator(hybrid, _rt(cache_type="naive"), topo, FakeWorkers(), num_pages=64)
    with pytest.raises(ValueError, match="rolled back"):          # nor can rejected draft tokens be undone in that state
        AfdCoordinator(hybrid, _rt(spec_block=4), topo, FakeWorkers(), num_pages=64)
    AfdCoordinator(PRESETS["tiny-qwen3-moe"], _rt(cache_type="radix"), topo, FakeWorkers(), num_pages=64)
