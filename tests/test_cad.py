"""Core-attention disaggregation on CPU: several "ranks" as plain objects sharing tensors.
Checks the flag program (every flag released once and waited once), strict config parsing,
token-identical decode vs the whole-sequence reference, and a host-injected lost flag that
must end as a clean, recoverable abort."""
import dataclasses

import pytest
import torch

from fastafd_b200.cad.config import CadConfig, CadConfigError
from fastafd_b200.cad.program import attention_program, check_balanced, flag_traffic, model_program
from fastafd_b200.cad.runtime import CadRuntime, CadStepAborted
from fastafd_b200.config import ModelConfig, RopeConfig
from fastafd_b200.models.transformer import AttentionStage, ExpertStage
from fastafd_b200.reference.model_ref import greedy_generate_reference

CFG = ModelConfig(architecture="MiniMaxM2ForCausalLM", num_layers=3, hidden_size=128, num_q_heads=4, num_kv_heads=2,
                  head_dim=32, vocab_size=512, num_experts=8, num_experts_per_tok=2, moe_intermediate_size=64,
                  qk_norm="cross_head", rope=RopeConfig(5e6, 16), scoring="sigmoid", router_bias=True, router_fp32=True)


def test_programs_and_flag_balance():
    assert len(attention_program(3, 2)) == 12
    kinds = [t.kind for t in model_program(2, 1)]
    assert kinds == ["embed", "hqkv", "hpost", "ffn", "hqkv", "hpost", "ffn", "final", "sample"]
    rel, wait = flag_traffic(3, 2, 2)
    assert len(rel) == len(wait) == 2 * 3 * 2 * 2
    check_balanced(4, 2, 3)


def test_config_is_strict(monkeypatch):
    for k in list(__import__("os").environ):
        if k.startswith(("FASTAFD_CAD_", "MINISGL_AFD_CAD_")) or k in ("FASTAFD_MODE", "MINISGL_AFD_MODE"):
            monkeypatch.delenv(k)
    assert not CadConfig.from_env().enabled and CadConfig.from_env().env() == {}
    monkeypatch.setenv("FASTAFD_MODE", "cad")
    monkeypatch.setenv("FASTAFD_CAD_HANG_TIMEOUT_NS", "1000")
    c = CadConfig.from_env()
    assert c.enabled and c.hang_timeout_ns == 1000
    monkeypatch.setenv("FASTAFD_CAD_O_DTYPE", "fp4")
    with pytest.raises(CadConfigError):
        CadConfig.from_env()
    monkeypatch.setenv("FASTAFD_CAD_O_DTYPE", "float32")
    monkeypatch.setenv("FASTAFD_MODE", "banana")
    with pytest.raises(CadConfigError):
        CadConfig.from_env()


def test_config_takes_the_reference_names_and_spellings():
    """The environment of a reference CAD benchmark configuration parses as it is; a CAD key without CAD mode, an
    expert path that does not exist here and a malformed number are refused with the key named."""
    ref_env = {"MINISGL_AFD_MODE": "cad", "MINISGL_AFD_CAD_HANG_TIMEOUT_NS": "300000000000", "MINISGL_AFD_CAD_HOP": "window",
               "MINISGL_AFD_CAD_INIT_TIMEOUT_S": "900", "MINISGL_AFD_CAD_MOE": "megamoe_dual", "MINISGL_AFD_CAD_O_DTYPE": "bf16"}
    c = CadConfig.from_env(ref_env)
    assert c == CadConfig(mode="cad", o_dtype="bfloat16", hop="kernel", moe="dual", hang_timeout_ns=300_000_000_000, init_timeout_s=900.0)
    assert CadConfig.from_env(c.env()) == c                       # what a child process is given parses back to the same
    with pytest.raises(CadConfigError, match="without MODE=cad"):
        CadConfig.from_env({"MINISGL_AFD_CAD_HOP": "window"})
    with pytest.raises(CadConfigError, match="DeepEP"):
        CadConfig.from_env(dict(ref_env, MINISGL_AFD_CAD_MOE="deepep"))
    with pytest.raises(CadConfigError, match="CAD_HANG_TIMEOUT_NS"):
        CadConfig.from_env(dict(ref_env, MINISGL_AFD_CAD_HANG_TIMEOUT_NS="soon"))
    assert not CadConfig.from_env({"MINISGL_AFD_MODE": ""}).enabled


def _runtime(r=2, timeout=2.0):
    stage = AttentionStage(CFG, "cpu", torch.float32).init_random(4)
    experts = ExpertStage(CFG, "cpu", torch.float32).init_random(4)
    rt = CadRuntime(CFG, stage, experts, CadConfig(mode="cad", attn_per_model=r), num_mb=2, max_tokens=4, page_size=16,
                    num_pages=16, wait_timeout_s=timeout)
    return rt, stage, experts


def _step_inputs(tokens_by_req, pos):
    B = len(tokens_by_req)
    half = B // 2
    mbs = []
    for lo, hi in ((0, half), (half, B)):
        ids = torch.tensor(tokens_by_req[lo:hi], dtype=torch.int32)
        n = hi - lo
        pt = (torch.arange(lo, hi, dtype=torch.int32)[:, None] * 2 + 1 + torch.arange(2, dtype=torch.int32)[None])
        mbs.append((ids, torch.full((n,), pos, dtype=torch.int32), pt, torch.arange(lo, hi) % 2))
    return mbs


def test_cad_decode_matches_reference():
    rt, stage, experts = _runtime()
    g = torch.Generator().manual_seed(1)
    prompts = [torch.randint(0, CFG.vocab_size, (7,), generator=g).tolist() for _ in range(4)]
    seqs = [list(p) for p in prompts]
    out = None
    for pos in range(7 + 5):
        cur = [s[pos] for s in seqs]
        nxt = torch.cat(rt.decode_step(_step_inputs(cur, pos))).tolist()
        if pos >= 6:
            for s, t in zip(seqs, nxt):
                s.append(int(t))
    got = [s[7:7 + 5] for s in seqs]
    assert got == greedy_generate_reference(CFG, stage, [experts], prompts, 5)
    assert all(w.epoch == 12 for w in rt.windows)


def test_lost_flag_aborts_step_and_runtime_recovers():
    rt, _, _ = _runtime(timeout=0.2)
    ok = rt.decode_step(_step_inputs([1, 2, 3, 4], 0))
    with pytest.raises(CadStepAborted):
        rt.decode_step(_step_inputs([5, 6, 7, 8], 1), drop=("o", 1, 0))      # attention rank "forgets" one release
    assert all(int(w.err[0]) == 1 for w in rt.windows)
    with pytest.raises(CadStepAborted):                                      # later steps see err and do not spin
        rt.decode_step(_step_inputs([5, 6, 7, 8], 1))
    rt.reset_error()
    again = rt.decode_step(_step_inputs([5, 6, 7, 8], 1))
    assert len(again) == 2 and len(ok) == 2
