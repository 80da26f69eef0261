"""A checkpoint directory given as --model-path is what gets served: the engine loads it per
role (attention stage / this rank's experts), a directory without safetensors files is refused,
and --dummy-weights serves random weights of the directory's architecture."""
import dataclasses

import pytest
import torch

from fastafd_b200.config import PRESETS, RuntimeConfig, get_model_config
from fastafd_b200.core import SamplingParams
from fastafd_b200.engine import AfdEngine, SpmdDriver, resolve_checkpoint
from fastafd_b200.models.loader import save_checkpoint
from fastafd_b200.models.transformer import AttentionStage, ExpertStage
from fastafd_b200.protocol import AfdTopology
from fastafd_b200.server.args import parse_args

CFG = dataclasses.replace(PRESETS["tiny-qwen3-moe"], num_layers=2)
PROMPTS = [[5, 9, 200, 31, 77, 4], [1000, 3, 3, 8]]


def _rt(path, device="cpu", **kw):
    base = dict(model_path=path, num_mb=2, page_size=16, num_pages=64, max_running_requests=8, max_seq_len=128,
                cuda_graph_max_bs=8, device=device, dtype="float32" if device == "cpu" else "bfloat16",
                use_cuda_graph=device != "cpu")
    base.update(kw)
    return RuntimeConfig(**base)


@pytest.fixture(scope="module")
def ckpt_dir(tmp_path_factory):
    d = tmp_path_factory.mktemp("served")
    attn = AttentionStage(CFG, "cpu", torch.float32).init_random(7)
    exp = ExpertStage(CFG, "cpu", torch.float32).init_random(7)
    save_checkpoint(CFG, attn, [exp], str(d / "model"), shard_mb=1)
    return str(d / "model")


def _generate(cfg, rt, seed=0, n=6):
    eng = AfdEngine(cfg, rt, AfdTopology(colocated=True), 0, rt.device if rt.device == "cpu" else "cuda:0", seed=seed)
    try:
        return SpmdDriver(eng).generate(PROMPTS, SamplingParams(max_tokens=n, ignore_eos=True)), eng
    finally:
        eng.close()


def test_engine_serves_the_checkpoint_not_random_weights(ckpt_dir):
    cfg = get_model_config(ckpt_dir)
    assert cfg == CFG                                           # config.json round trip
    from_ckpt, eng = _generate(cfg, _rt(ckpt_dir), seed=0)
    assert eng.checkpoint == ckpt_dir
    same_tensors, _ = _generate(CFG, _rt("tiny-qwen3-moe"), seed=7)     # the tensors the checkpoint was written from
    other_seed, _ = _generate(CFG, _rt("tiny-qwen3-moe"), seed=0)
    assert from_ckpt == same_tensors
    assert from_ckpt != other_seed


def test_directory_without_weights_is_refused_unless_dummy(tmp_path, ckpt_dir):
    import shutil

    empty = tmp_path / "only_config"
    empty.mkdir()
    shutil.copy(ckpt_dir + "/config.json", empty / "config.json")
    with pytest.raises(FileNotFoundError):
        resolve_checkpoint(_rt(str(empty)))
    assert resolve_checkpoint(_rt(str(empty), dummy_weights=True)) is None
    assert resolve_checkpoint(_rt("tiny-qwen3-moe")) is None
    out, eng = _generate(get_model_config(str(empty)), _rt(str(empty), dummy_weights=True), n=2)
    assert eng.checkpoint is None and all(len(o) == 2 for o in out)
    a = parse_args(["--model-path", str(empty), "--dummy-weights", "--device", "cpu"])
    assert a.runtime_config().dummy_weights


@pytest.mark.timeout(300)
def test_http_server_serves_the_checkpoint(ckpt_dir):
    """1 attention + 1 expert process on CPU, started from the checkpoint directory: the tokens
    that come back over HTTP are those of an engine built from the same tensors."""
    from serving_util import greedy_tokens, running_server

    expect, _ = _generate(CFG, _rt("tiny-qwen3-moe"), seed=7, n=5)
    args = parse_args(["--mode", "afd-serve", "--model-path", ckpt_dir, "--device", "cpu", "--afd-num-mb", "2",
                       "--num-pages", "64", "--max-seq-len-override", "128", "--afd-max-running-requests", "8",
                       "--cuda-graph-max-bs", "8"])
    with running_server(args) as (base, sup):
        got = [greedy_tokens(base, p, 5) for p in PROMPTS]
        assert sup.get_failures() == []
    assert got == expect


@pytest.mark.gpu
def test_block_fp8_checkpoint_on_gpu(tmp_path):
    """A block-FP8 checkpoint keeps its e4m3 bytes and exact 128x128 scales on the GPU (no
    requantisation) and decodes without a device error."""
    from fastafd_b200 import ops
    from fastafd_b200.config import QuantConfig
    from fastafd_b200.reference import ops_ref as ref

    cfg = dataclasses.replace(CFG, quant=QuantConfig("fp8"))
    attn = AttentionStage(cfg, "cpu", torch.float32).init_random(7)
    exp = ExpertStage(cfg, "cpu", torch.float32).init_random(7)
    d = str(tmp_path / "fp8")
    save_checkpoint(cfg, attn, [exp], d, fp8_experts=True, shard_mb=1)
    assert get_model_config(d).quant.is_fp8
    eng = AfdEngine(get_model_config(d), _rt(d, device="cuda"), AfdTopology(colocated=True), 0, "cuda:0")
    try:
        layer, I = exp.moe_layers[0], cfg.moe_intermediate_size
        q = torch.stack([torch.cat([ref.block_quant_fp8(exp.gate_up[layer][e, :I])[0], ref.block_quant_fp8(exp.gate_up[layer][e, I:])[0]])
                         for e in range(cfg.num_experts)])
        want = ops.interleave_gate_up(q.view(torch.uint8).cuda())
        assert torch.equal(eng.expert_stage.w13[layer].view(torch.uint8), want)
        out = SpmdDriver(eng).generate(PROMPTS, SamplingParams(max_tokens=4, ignore_eos=True))
        assert all(len(o) == 4 for o in out)
    finally:
        eng.close()
