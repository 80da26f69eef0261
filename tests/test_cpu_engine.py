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


def test_radix_prefix_cache_through_the_engine_gives_the_same_tokens_and_shares_pages():
    """Two waves of requests with a long common prefix: with the radix cache the second wave reuses
    the first wave's KV pages (fewer prefill tokens are computed) and must produce exactly the
    tokens of the naive ledger."""
    cfg = PRESETS["tiny-qwen3-moe"]
    g = torch.Generator().manual_seed(5)
    prefix = torch.randint(0, cfg.vocab_size, (48,), generator=g).tolist()
    waves = [[prefix + torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (5, 9)] for _ in range(2)]
    sp = SamplingParams(max_tokens=5, ignore_eos=True)

    def run(cache_type):
        eng = AfdEngine(cfg, _rt(cache_type=cache_type, num_pages=96), AfdTopology(colocated=True), 0, "cpu", seed=0)
        drv = SpmdDriver(eng)
        outs = [drv.generate(w, sp) for w in waves]
        lane = drv.lanes[0]
        lane.check_integrity()
        return outs, lane

    naive, _ = run("naive")
    radix, lane = run("radix")
    assert radix == naive
    assert lane.cache.cached_pages >= len(prefix) // 16          # the shared prefix stayed cached
    assert lane.prefix_hit_len(prefix + [1, 2, 3]) >= (len(prefix) // 16) * 16


def test_validate_cli_reports_full_agreement_on_cpu(capsys):
    import json

    from fastafd_b200 import validate

    rc = validate.main(["--device", "cpu", "--prompts", "2", "--prompt-len", "12", "--decode", "5"])
    out = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert rc == 0 and out["verdict"] == "pass" and out["match"] == 1.0 and out["tokens"] == 10
    assert out["overall_top1_agreement_rate"] == 1.0 and out["overall_top100_hit_rate"] == 1.0
    assert out["rank_gate"]["worst_rank"] == 0
    assert validate.first_divergence([1, 2, 3], [1, 2, 4]) == 2 and validate.first_divergence([1], [1, 2]) == 1


def test_rank_scoring_of_continuations_sees_a_foreign_token():
    """The rank gate: the oracle's own greedy continuation scores rank 0 everywhere; replacing one token by
    the oracle's least likely one shows up as one position outside the top 100."""
    from fastafd_b200.reference.model_ref import forward_logits, greedy_generate_reference, score_continuations

    cfg = PRESETS["tiny-qwen3-moe"]
    eng = AfdEngine(cfg, _rt(), AfdTopology(colocated=True), 0, "cpu", seed=0)
    stage, experts = eng.attn.model, [eng.expert_stage]
    prompts = [[5, 9, 200, 31], [7, 7, 7, 1, 2]]
    outs = greedy_generate_reference(cfg, stage, experts, prompts, 4)
    good = score_continuations(cfg, stage, experts, prompts, outs)
    assert good["tokens"] == 8 and good["top1_agreement_rate"] == 1.0 and all(x == 0 for r in good["ranks"] for x in r)
    worst = int(forward_logits(cfg, stage, experts, prompts[0] + outs[0][:2]).argmin())
    bad_out = [outs[0][:2] + [worst] + outs[0][3:], outs[1]]
    bad = score_continuations(cfg, stage, experts, prompts, bad_out)
    assert bad["ranks"][0][2] == cfg.vocab_size - 1 and bad["top100_hit_rate"] < 1.0 and bad["top1_agreement_rate"] < 1.0
    eng.close()


def test_reference_environment_names_act_under_their_new_names():
    from fastafd_b200.env import HOT_PATH_KNOBS, REFERENCE_ALIASES, apply_reference_aliases

    env = {"MINISGL_PDL": "0", "MINISGL_MEGAMOE_EG_PREFETCH_MB": "32", "FASTAFD_L2_PREFETCH_MB": "8", "MINISGL_AFD_LANE_COMPUTE_STREAMS": ""}
    copied = apply_reference_aliases(env)
    assert copied == {"FASTAFD_PDL": "0"} and env["FASTAFD_PDL"] == "0"
    assert env["FASTAFD_L2_PREFETCH_MB"] == "8"                # the new name wins when both are set
    assert "FASTAFD_LANE_STREAMS" not in env                   # an empty value is not a setting
    assert set(REFERENCE_ALIASES.values()) <= set(HOT_PATH_KNOBS)


def test_flag_report_names_the_peers_that_are_behind():
    """Triage of a wait that ran out: the peers whose last written epoch is behind the others are the ones the wait
    was waiting for. (Plain tensors stand in for the flag words of the peer-mapped heap.)"""
    import torch

    from fastafd_b200.moe.afd_moe import flag_report

    rep = flag_report(torch.tensor([97, 96, 97, 97], dtype=torch.int32), torch.tensor([98], dtype=torch.int32), [4, 5, 6, 7])
    assert rep == {"next_epoch": 98, "flags": {4: 97, 5: 96, 6: 97, 7: 97}, "behind": [5]}
    assert flag_report(torch.tensor([3, 3], dtype=torch.int32), torch.tensor([4], dtype=torch.int32), [0, 1])["behind"] == []
    # an engine without fabric endpoints (CPU) has nothing to report and says so without raising
    from fastafd_b200.config import PRESETS, RuntimeConfig
    from fastafd_b200.engine import AfdEngine
    from fastafd_b200.protocol import AfdTopology

    rt = RuntimeConfig(num_mb=1, page_size=16, num_pages=16, max_running_requests=2, max_seq_len=64, cuda_graph_max_bs=2,
                       device="cpu", dtype="float32", use_cuda_graph=False)
    assert AfdEngine(PRESETS["tiny-qwen3-moe"], rt, AfdTopology(colocated=True), 0, "cpu").describe_waits() == {}
