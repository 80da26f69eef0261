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


def _published_draft(path, cfg, *, hidden, heads, kv_heads, head_dim, inter, draft_vocab, layer_ids, with_embedding=False, with_head=True):
    """A draft directory in the layout of published EAGLE-3 heads: its own config.json, `midlayer.*` keys with separate
    q/k/v and gate/up, `fc`, `norm`, a small-vocabulary `lm_head` with `d2t` offsets (and the unused `t2d` mask)."""
    import json
    import os

    from safetensors.torch import save_file

    os.makedirs(path, exist_ok=True)
    json.dump({"architectures": ["LlamaForCausalLMEagle3"], "hidden_size": hidden, "num_attention_heads": heads,
               "num_key_value_heads": kv_heads, "head_dim": head_dim, "intermediate_size": inter, "num_hidden_layers": 1,
               "vocab_size": cfg.vocab_size, "draft_vocab_size": draft_vocab, "rms_norm_eps": 1e-5, "rope_theta": 50000.0,
               "eagle_config": {"eagle_aux_hidden_state_layer_ids": list(layer_ids), "use_aux_hidden_state": True}},
              open(os.path.join(path, "config.json"), "w"))
    g = torch.Generator().manual_seed(5)
    r = lambda *s: torch.randn(*s, generator=g) * 0.05  # noqa: E731
    sd = {"fc.weight": r(hidden, 3 * hidden), "norm.weight": torch.ones(hidden),
          "midlayer.input_layernorm.weight": torch.ones(hidden), "midlayer.hidden_norm.weight": torch.ones(hidden),
          "midlayer.post_attention_layernorm.weight": torch.ones(hidden),
          "midlayer.self_attn.q_proj.weight": r(heads * head_dim, 2 * hidden),
          "midlayer.self_attn.k_proj.weight": r(kv_heads * head_dim, 2 * hidden),
          "midlayer.self_attn.v_proj.weight": r(kv_heads * head_dim, 2 * hidden),
          "midlayer.self_attn.o_proj.weight": r(hidden, heads * head_dim),
          "midlayer.mlp.gate_proj.weight": r(inter, hidden), "midlayer.mlp.up_proj.weight": r(inter, hidden),
          "midlayer.mlp.down_proj.weight": r(hidden, inter)}
    if with_head:
        sd["lm_head.weight"] = r(draft_vocab, hidden)
        picks = torch.randperm(cfg.vocab_size, generator=g)[:draft_vocab].sort().values          # draft id -> target id
        sd["d2t"] = picks - torch.arange(draft_vocab)
        mask = torch.zeros(cfg.vocab_size, dtype=torch.bool)
        mask[picks] = True
        sd["t2d"] = mask
    if with_embedding:
        sd["embed_tokens.weight"] = r(cfg.vocab_size, hidden)
    save_file(sd, os.path.join(path, "model.safetensors"))
    return sd


@pytest.mark.parametrize("with_embedding,with_head", [(False, True), (True, False)])
def test_published_draft_head_layout_is_loaded_from_its_own_config(tmp_path, with_embedding, with_head):
    """A draft head whose sizes differ from what the target would suggest (heads, head dim, MLP width, a 100-token
    draft vocabulary with a d2t map, its own auxiliary layers and rotary base), without an embedding of its own
    (the target's is shared) or without an LM head (the target's is used): the engine takes every size from the
    head's config.json, and greedy verification stays lossless whatever the head proposes."""
    from fastafd_b200.spec.eagle3 import Eagle3Config

    cfg = PRESETS["tiny-qwen3-moe"]
    path = str(tmp_path / "draft")
    dv = 100 if with_head else cfg.vocab_size
    sd = _published_draft(path, cfg, hidden=cfg.hidden_size, heads=2, kv_heads=1, head_dim=32, inter=96, draft_vocab=dv,
                          layer_ids=(0, 1, 2) if cfg.num_layers >= 3 else (0, 0, 1), with_embedding=with_embedding, with_head=with_head)
    dc = Eagle3Config.from_dir(path, cfg)
    assert (dc.num_q_heads, dc.num_kv_heads, dc.head_dim, dc.intermediate_size, dc.draft_vocab) == (2, 1, 32, 96, dv)
    assert dc.rope_theta == 50000.0 and dc.rms_eps == 1e-5 and dc.target_vocab == cfg.vocab_size
    g = torch.Generator().manual_seed(0)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (30, 7, 18)]
    sp = SamplingParams(max_tokens=9, ignore_eos=True)
    plain = SpmdDriver(AfdEngine(cfg, _rt(), AfdTopology(colocated=True), 0, "cpu", seed=0)).generate(prompts, sp)
    eng = AfdEngine(cfg, _rt(spec_block=3, spec_draft_path=path), AfdTopology(colocated=True), 0, "cpu", seed=0)
    draft = eng.attn.spec.draft
    assert draft.cfg == dc and list(eng.attn.spec.capture_layers) == list(dc.target_layers)
    if with_head:
        assert draft.d2t.tolist() == (sd["d2t"] + torch.arange(dv)).tolist() and draft.w["lm_head.weight"].shape[0] == dv
        assert draft.w["embed_tokens.weight"] is eng.attn.model.w["model.embed_tokens.weight"]      # shared, not copied
    else:
        assert draft.w["lm_head.weight"].shape[0] == cfg.vocab_size and draft.d2t.tolist() == list(range(cfg.vocab_size))
        assert torch.equal(draft.w["embed_tokens.weight"], sd["embed_tokens.weight"])
    assert SpmdDriver(eng).generate(prompts, sp) == plain


def test_draft_config_refusals(tmp_path, monkeypatch):
    import json

    from fastafd_b200.spec.eagle3 import Eagle3Config

    cfg = PRESETS["tiny-qwen3-moe"]
    path = str(tmp_path / "d")
    _published_draft(path, cfg, hidden=cfg.hidden_size, heads=2, kv_heads=1, head_dim=32, inter=96, draft_vocab=50, layer_ids=(0, 1, 2))
    base = json.load(open(path + "/config.json"))

    def with_(**kw):
        c = dict(base)
        c.update(kw)
        json.dump(c, open(path + "/config.json", "w"))

    monkeypatch.setenv("MINISGL_AFD_SPEC_EAGLE3_LAYERS", "2,1,0")
    assert Eagle3Config.from_dir(path, cfg).target_layers == (2, 1, 0)             # the reference's override knob
    monkeypatch.delenv("MINISGL_AFD_SPEC_EAGLE3_LAYERS")
    for bad, pattern in ((dict(num_hidden_layers=2), "layers"), (dict(hidden_size=cfg.hidden_size * 2), "hidden size"),
                         (dict(rope_scaling={"rope_type": "yarn", "factor": 4.0}), "rotary scaling"),
                         (dict(eagle_config={"use_aux_hidden_state": False}), "auxiliary"),
                         (dict(eagle_config={"eagle_aux_hidden_state_layer_ids": [0, 1, 99]}), "auxiliary layers")):
        with_(**bad)
        with pytest.raises(ValueError, match=pattern):
            Eagle3Config.from_dir(path, cfg)
    big = PRESETS["qwen3-30b-a3b"]                      # no ids: the default rule, which needs a deep enough target
    with_(eagle_config={}, hidden_size=big.hidden_size)
    assert Eagle3Config.from_dir(path, big).target_layers == (1, big.num_layers // 2 - 1, big.num_layers - 4)
