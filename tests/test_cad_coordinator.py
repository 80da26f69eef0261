"""Core-attention disaggregation driven by the coordinator (CPU, every rank an object of this process):
prefill as AFD steps on the attention ranks, decode as CAD steps with the KV cache on the attention ranks and
everything else on the model ranks, steps planned ahead, a lost flag that voids one step only."""
import numpy as np
import pytest
import torch

from fastafd_b200.cad.coordinator import CadCoordinator
from fastafd_b200.cad.deploy import CadLocalWorkers
from fastafd_b200.cad.ranks import CadRanks, CadTopologyError
from fastafd_b200.cad.tokens import CadRow, CadTokenPath, host_token, pack_rows, row_index, tokens_by_peer, unpack_rows
from fastafd_b200.config import ModelConfig, RopeConfig, RuntimeConfig
from fastafd_b200.coordinator import CoordinatorError
from fastafd_b200.core import SamplingParams
from fastafd_b200.models.transformer import AttentionStage, ExpertStage
from fastafd_b200.protocol import AfdTopology, CadInitCmd, CadStepCmd, CadStepReply, decode, encode
from fastafd_b200.reference.model_ref import greedy_generate_reference

CFG = ModelConfig(architecture="MiniMaxM2ForCausalLM", num_layers=3, hidden_size=128, num_q_heads=4, num_kv_heads=2,
                  head_dim=32, vocab_size=512, num_experts=8, num_experts_per_tok=2, moe_intermediate_size=64,
                  qk_norm="cross_head", rope=RopeConfig(5e6, 16), scoring="sigmoid", router_bias=True, router_fp32=True,
                  eos_token_ids=())


def _rt(**kw):
    base = dict(model_path="tiny", num_mb=2, page_size=16, num_pages=64, max_running_requests=8, max_seq_len=128,
                cuda_graph_max_bs=8, device="cpu", dtype="float32", use_cuda_graph=False, async_pending_steps=3,
                max_batched_tokens=64)
    base.update(kw)
    return RuntimeConfig(**base)


# ------------------------------------------------------------------------- rank arithmetic
def test_ranks_and_peers():
    rk = CadRanks.of(AfdTopology(attn_dp=4, mlp_ep=2))
    assert (rk.num_attn, rk.num_model, rk.r, rk.world) == (4, 2, 2, 6)
    assert rk.model_ranks() == [4, 5] and rk.peers_of(1) == [2, 3]
    assert [rk.model_of(a) for a in range(4)] == [4, 4, 5, 5] and [rk.peer_index(a) for a in range(4)] == [0, 1, 0, 1]
    assert rk.role(3) == "attn" and rk.role(4) == "model" and rk.model_index(5) == 1
    for bad in (AfdTopology(colocated=True), AfdTopology(attn_dp=2, attn_tp=2, mlp_ep=2), AfdTopology(attn_dp=3, mlp_ep=2)):
        with pytest.raises(CadTopologyError):
            CadRanks.of(bad)
    with pytest.raises(CadTopologyError):
        rk.model_of(4)


# ------------------------------------------------------------------------- token path
def test_token_path_takes_the_host_token_or_the_last_sampled_one():
    tp = CadTokenPath(r=2, num_mb=2, t_max=4, table_rows=9)
    tp.bind(2)
    assert tp.rows == 8 and tp.mb_rows(1) == slice(4, 8) and tp.peer_rows(1, 1) == slice(6, 8)
    assert row_index(2, 2, 1, 1, 0) == 6
    rows = [CadRow(0, 0, 0, 3, 10, 41), CadRow(1, 0, 1, 3, 7, 42), CadRow(1, 1, 0, 5, 2, 43)]
    where = tp.stage(unpack_rows(pack_rows(rows)))
    assert where == [0, 3, 6]
    assert tp.input_ids().tolist() == [41, 0, 0, 42, 0, 0, 43, 0] and tp.positions().tolist() == [10, 0, 0, 7, 0, 0, 2, 0]
    tp.record(torch.arange(100, 108))
    assert tp.last[0 * 9 + 3] == 100 and tp.last[1 * 9 + 3] == 103 and tp.last[1 * 9 + 5] == 106
    # next step: no host tokens, other rows of the bucket: each request finds its own last token
    tp.stage([CadRow(1, 0, 0, 5, 3, -1), CadRow(0, 1, 1, 3, 11, -1), CadRow(1, 1, 1, 3, 8, 77)])
    ids = tp.input_ids().tolist()
    assert ids[row_index(2, 2, 0, 1, 0)] == 106 and ids[row_index(2, 2, 1, 0, 1)] == 100 and ids[row_index(2, 2, 1, 1, 1)] == 77
    by = tokens_by_peer(list(range(8)), 2, 2, 2)
    assert by[0].tolist() == [0, 1, 4, 5] and by[1].tolist() == [2, 3, 6, 7]
    assert host_token([5, 6, 7], 2) == 7 and host_token([5, 6, 7], 3) == -1
    with pytest.raises(ValueError):
        tp.stage([CadRow(0, 0, 0, 3, 1, 1), CadRow(0, 0, 0, 4, 1, 1)])          # one row twice
    with pytest.raises(ValueError):
        tp.stage([CadRow(0, 0, 0, 3, 1, 1), CadRow(0, 1, 0, 3, 1, 1)])          # one request twice
    with pytest.raises(ValueError):
        tp.stage([CadRow(0, 0, 2, 3, 1, 1)])                                      # index outside the bucket
    tp.stage_padding()
    assert tp.input_ids().tolist() == [0] * 8


def test_cad_messages_survive_the_wire():
    cmd = decode(encode(CadStepCmd(step_id=4, bucket=2, rows=pack_rows([CadRow(1, 0, 1, 3, 7, -1)]))))
    assert unpack_rows(cmd.rows) == [CadRow(1, 0, 1, 3, 7, -1)] and cmd.plan is None
    rep = decode(encode(CadStepReply(step_id=4, rank=5, tokens={0: np.arange(3, dtype=np.int32)}, err=0)))
    assert rep.tokens[0].tolist() == [0, 1, 2]
    init = decode(encode(CadInitCmd(buckets=[1, 2, 4], t_max=4, table_rows=9, num_mb=2)))
    assert init.buckets == [1, 2, 4] and init.use_graph


# ------------------------------------------------------------------------- end to end
def _run(topo, prompts, max_tokens, **rtkw):
    rt = _rt(**rtkw)
    workers = CadLocalWorkers(CFG, rt, topo, seed=4)
    got, done = {}, set()

    def on_tokens(items):
        for uid, toks, fin in items:
            got.setdefault(uid, []).extend(toks)
            if fin:
                done.add(uid)

    coord = CadCoordinator(CFG, rt, topo, workers, num_pages=workers.num_pages, max_comm_tokens=64, on_tokens=on_tokens)
    for uid, p in enumerate(prompts):
        coord.add_request(uid, p, SamplingParams(max_tokens=max_tokens[uid], ignore_eos=True))
    return coord, workers, got, done


def _oracle(prompts, max_tokens):
    stage = AttentionStage(CFG, "cpu", torch.float32).init_random(4)
    experts = ExpertStage(CFG, "cpu", torch.float32).init_random(4)
    full = greedy_generate_reference(CFG, stage, [experts], prompts, max(max_tokens))
    return [t[:n] for t, n in zip(full, max_tokens)]


@pytest.mark.parametrize("attn,model,pending", [(2, 1, 3), (4, 2, 2), (2, 2, 1)])
def test_served_through_the_coordinator_equals_the_reference(attn, model, pending):
    g = torch.Generator().manual_seed(attn * 10 + model)
    lens = [5, 9, 17, 3, 12, 7, 21]
    prompts = [torch.randint(0, CFG.vocab_size, (n,), generator=g).tolist() for n in lens]
    max_tokens = [6, 1, 4, 8, 5, 2, 7]
    coord, workers, got, done = _run(AfdTopology(attn_dp=attn, mlp_ep=model), prompts, max_tokens, async_pending_steps=pending)
    coord.run_until_idle()
    assert done == set(range(len(prompts)))
    assert [got[u] for u in range(len(prompts))] == _oracle(prompts, max_tokens)
    assert workers.steps_run >= max(max_tokens) - 1 and not coord.aborted_steps
    for lane in coord.lanes:
        lane.audit_pages()
        assert not lane.states


def test_requests_that_arrive_during_decode_join_without_disturbing_the_others():
    g = torch.Generator().manual_seed(3)
    prompts = [torch.randint(0, CFG.vocab_size, (n,), generator=g).tolist() for n in (6, 11, 4, 15, 8)]
    max_tokens = [9, 7, 8, 5, 6]
    coord, workers, got, done = _run(AfdTopology(attn_dp=2, mlp_ep=1), prompts[:2], max_tokens[:2])
    for _ in range(4):
        coord.step_loop_once(block=True)
    for uid in (2, 3, 4):                     # late arrivals: prefill steps now interleave with CAD steps in flight
        coord.add_request(uid, prompts[uid], SamplingParams(max_tokens=max_tokens[uid], ignore_eos=True))
        coord.step_loop_once(block=True)
    coord.run_until_idle()
    assert [got[u] for u in range(5)] == _oracle(prompts, max_tokens)


def test_random_sampling_and_speculation_are_refused():
    coord, *_ = _run(AfdTopology(attn_dp=2, mlp_ep=1), [], [])
    with pytest.raises(CoordinatorError):
        coord.add_request(0, [1, 2, 3], SamplingParams(max_tokens=4, temperature=0.8))
    with pytest.raises(ValueError):
        CadCoordinator(CFG, _rt(spec_block=4), AfdTopology(attn_dp=2, mlp_ep=1), CadLocalWorkers(CFG, _rt(), AfdTopology(attn_dp=2, mlp_ep=1)),
                       num_pages=64)


@pytest.mark.parametrize("flag", [("qkv", 1, 0), ("o", 2, 1)])
def test_a_lost_flag_voids_one_step_and_the_deployment_keeps_serving(flag):
    g = torch.Generator().manual_seed(9)
    prompts = [torch.randint(0, CFG.vocab_size, (n,), generator=g).tolist() for n in (6, 9, 5, 8)]
    max_tokens = [8, 8, 8, 8]
    coord, workers, got, done = _run(AfdTopology(attn_dp=2, mlp_ep=1), prompts, max_tokens, async_pending_steps=1)
    while workers.steps_run < 2:
        coord.step_loop_once(block=True)
    workers.drop_next(1, flag)                # the next release of this flag on lane 1's window never happens
    coord.run_until_idle()
    assert len(coord.aborted_steps) == 1 and coord.get_failure() is None
    # who was stuck on what: a lost qkv flag stops its attention rank, and the model rank (rank 2) then waits for that rank's o rows
    assert workers.last_blocked[2] == ("o", flag[1], flag[2]) and (flag[0] == "o" or workers.last_blocked[1] == flag)
    want = _oracle(prompts, max_tokens)
    assert done == {0, 1, 2, 3}
    for u in range(4):                        # ended early, and what they did produce is right
        assert len(got[u]) < 8 and got[u] == want[u][:len(got[u])]
    # the deployment serves on: new requests run to the end with the right tokens
    more = [torch.randint(0, CFG.vocab_size, (n,), generator=g).tolist() for n in (7, 10)]
    for i, p in enumerate(more):
        coord.add_request(10 + i, p, SamplingParams(max_tokens=5, ignore_eos=True))
    coord.run_until_idle()
    assert [got[10], got[11]] == _oracle(more, [5, 5])
    for lane in coord.lanes:
        lane.audit_pages()
        assert not lane.states


def test_offline_api_in_cad_mode(monkeypatch):
    """`LLM(...)` with the mode switch of the reference's environment: same tokens as the colocated engine."""
    from fastafd_b200.llm import LLM

    prompts = [[5, 9, 2, 44, 17], [8, 3], [61, 62, 63, 64, 65, 66, 67]]
    sp = SamplingParams(max_tokens=6, ignore_eos=True)
    base = LLM("tiny-qwen3-moe", device="cpu", num_pages=64, max_seq_len=128)
    want = [o["token_ids"] for o in base.generate(prompts, sp)]
    base.shutdown()
    monkeypatch.setenv("MINISGL_AFD_MODE", "cad")
    monkeypatch.setenv("FASTAFD_CAD_ATTN_PER_MODEL", "2")
    llm = LLM("tiny-qwen3-moe", device="cpu", num_pages=64, max_seq_len=128, num_mb=2)
    assert type(llm.coordinator).__name__ == "CadCoordinator" and llm.topo.attn_dp == 2
    got = [o["token_ids"] for o in llm.generate(prompts, sp)]
    llm.shutdown()
    assert got == want


@pytest.mark.parametrize("seed,cache", [(1, "naive"), (2, "radix")])
def test_soak_with_arrivals_aborts_and_shared_prefixes(monkeypatch, seed, cache):
    """Requests arrive and are aborted while prefill steps and CAD steps are in flight, some prompts share a
    prefix (under the radix cache their first pages are reused on the attention rank), page audit on: every
    request that was not aborted produces exactly the reference's tokens."""
    import random

    monkeypatch.setenv("FASTAFD_PAGE_AUDIT", "1")
    rng = random.Random(seed)
    shared = [rng.randrange(CFG.vocab_size) for _ in range(20)]
    prompts, max_tokens = [], []
    for _ in range(14):
        own = [rng.randrange(CFG.vocab_size) for _ in range(rng.randint(1, 14))]
        prompts.append((shared if rng.random() < 0.5 else []) + own)
        max_tokens.append(rng.randint(1, 7))
    want = _oracle(prompts, max_tokens)
    coord, workers, got, done = _run(AfdTopology(attn_dp=2, mlp_ep=1), [], [], cache_type=cache, max_batched_tokens=24)
    nxt, aborted = 0, set()
    for _ in range(3000):
        if nxt < len(prompts) and rng.random() < 0.4:
            coord.add_request(nxt, prompts[nxt], SamplingParams(max_tokens=max_tokens[nxt], ignore_eos=True))
            nxt += 1
        live = [u for u in range(nxt) if u not in done and u not in aborted]
        if live and rng.random() < 0.04:
            u = rng.choice(live)
            coord.abort(u)
            aborted.add(u)
        coord.step_loop_once(block=False)
        if nxt == len(prompts) and coord.idle():
            break
    else:
        raise AssertionError("did not drain")
    assert not coord.aborted_steps and len(aborted) < len(prompts)
    for u in range(len(prompts)):
        if u in aborted:
            assert got.get(u, []) == want[u][:len(got.get(u, []))]
        else:
            assert got[u] == want[u], u
    for lane in coord.lanes:
        lane.audit_pages()
        assert not lane.states


@pytest.mark.timeout(300)
@pytest.mark.parametrize("attn,model", [(2, 1), (2, 2)], ids=["2-attention-1-model", "2-attention-2-model"])
def test_served_cad_deployment_of_separate_processes(monkeypatch, attn, model):
    """HTTP -> tokenizer -> CAD coordinator -> ZeroMQ -> attention rank processes (KV cache, attention core) and
    model rank processes (dense layers, a slice of the experts each, sampling) over gloo: the greedy tokens
    are those of the colocated engine."""
    import requests

    from fastafd_b200.llm import LLM
    from fastafd_b200.server.args import parse_args
    from fastafd_b200.server.launch import local_endpoint
    from fastafd_b200.server.supervisor import LocalSupervisor

    prompts = [[5, 9, 2, 44, 17], [8, 3, 11], [61, 62, 63, 64, 65, 66, 67], [7]]
    base = LLM("tiny-qwen3-moe", device="cpu", num_pages=64, max_seq_len=128)
    want = [o["token_ids"] for o in base.generate(prompts, SamplingParams(max_tokens=5, ignore_eos=True))]
    base.shutdown()
    monkeypatch.setenv("FASTAFD_MODE", "cad")
    args = parse_args(["--mode", "afd-serve", "--model-path", "tiny-qwen3-moe", "--device", "cpu", "--afd-num-mb", "2",
                       "--afd-attn-dp-size", str(attn), "--afd-mlp-ep-size", str(model), "--num-pages", "64",
                       "--max-seq-len-override", "128", "--afd-max-running-requests", "8", "--cuda-graph-max-bs", "8"])
    sup = LocalSupervisor(args)
    with local_endpoint(args, sup) as url:
        got = []
        for p in prompts:
            r = requests.post(url + "/v1/chat/completions", json={"input_ids": p, "max_tokens": 5, "temperature": 0,
                                                                  "ignore_eos": True, "return_token_ids": True, "stream": False},
                              timeout=200).json()
            got.append(r["choices"][0]["token_ids"])
        batch = requests.post(url + "/v1/chat/completions/batch", json={"prompts": ["ab", "cde", "f"], "max_tokens": 3, "temperature": 0,
                                                                       "ignore_eos": True, "return_token_ids": True}, timeout=200).json()
        hot = requests.post(url + "/v1/chat/completions", json={"input_ids": [1, 2], "max_tokens": 2, "temperature": 0.9,
                                                                "stream": False}, timeout=60)
        assert sup.get_failures() == []
    assert got == want
    assert [len(c["token_ids"]) for c in batch["choices"]] == [3, 3, 3]
    assert "greedily" in hot.text            # random sampling is refused with a reason, the server keeps running


def test_an_init_that_never_finishes_is_reported_with_the_ranks_that_owe_it():
    from fastafd_b200.cad.coordinator import CadTransport
    from fastafd_b200.protocol import AgStepReply, EgStepReply, WorkerReady

    class HalfReady(CadTransport):
        """Answers prefill steps; acknowledges the CAD init on ranks 0 and 2 only; never answers a CAD step."""
        def __init__(self):
            self.out = []
        def send_cad_init(self, cmd):
            self.out += [WorkerReady(rank=0, role="cad-attn"), WorkerReady(rank=2, role="cad-model")]
        def send_step(self, step_id, ag_plans, eg_plans):
            for r, (plan, _) in ag_plans.items():
                n = sum(len(mb.rows) for mb in plan.mbs)
                self.out.append(AgStepReply(step_id=step_id, rank=r, next_tokens=np.full(n, 7, np.int32)))
            self.out += [EgStepReply(step_id=step_id, rank=r) for r in eg_plans]
        def send_cad_step(self, step_id, attn_cmds, model_cmds):
            pass
        def poll(self, timeout_s):
            out, self.out = self.out, []
            return out

    topo = AfdTopology(attn_dp=2, mlp_ep=1)
    coord = CadCoordinator(CFG, _rt(), topo, HalfReady(), num_pages=64, max_comm_tokens=64, cad_init_timeout_s=0.0)
    coord.add_request(0, [1, 2, 3], SamplingParams(max_tokens=4, ignore_eos=True))
    with pytest.raises(CoordinatorError, match=r"CAD init: ranks \[1\] did not finish"):
        coord.run_until_idle()
    assert coord.cad_ready == {0, 2}
