"""Every model family through the serving path on CPU (scheduler, paged KV / GDN state,
chunked prefill, ping-pong pipeline) against the whole-sequence reference forward."""
import dataclasses

import pytest
import torch

from fastafd_b200.config import ModelConfig, QuantConfig, RopeConfig, RuntimeConfig
from fastafd_b200.core import SamplingParams
from fastafd_b200.engine import AfdEngine, SpmdDriver
from fastafd_b200.protocol import AfdTopology
from fastafd_b200.reference.model_ref import greedy_generate_reference

BASE = dict(num_layers=3, hidden_size=128, num_q_heads=4, num_kv_heads=2, head_dim=32, vocab_size=512,
            num_experts=8, num_experts_per_tok=2, moe_intermediate_size=64)

FAMILIES = {
    "qwen3_moe": ModelConfig(**BASE),
    "minimax_m2": ModelConfig(**{**BASE, "architecture": "MiniMaxM2ForCausalLM", "qk_norm": "cross_head",
                                 "rope": RopeConfig(5e6, 16), "scoring": "sigmoid", "router_bias": True, "router_fp32": True}),
    "glm4_moe": ModelConfig(**{**BASE, "architecture": "Glm4MoeForCausalLM", "qk_norm": "none", "attention_bias": True,
                               "rope": RopeConfig(1e6, 16), "intermediate_size": 96, "scoring": "sigmoid",
                               "router_bias": True, "routed_scaling_factor": 2.5, "n_group": 2, "topk_group": 1,
                               "num_shared_experts": 1, "shared_expert_intermediate_size": 64, "first_k_dense": 1}),
    "qwen35_hybrid": ModelConfig(**{**BASE, "architecture": "Qwen3_5MoeForCausalLM", "num_layers": 4,
                                    "rope": RopeConfig(1e7, 16), "num_shared_experts": 1,
                                    "shared_expert_intermediate_size": 64, "shared_expert_gate": True,
                                    "layer_types": ("linear", "linear", "linear", "full"), "gdn_num_k_heads": 2,
                                    "gdn_num_v_heads": 4, "gdn_head_k_dim": 16, "gdn_head_v_dim": 16,
                                    "gdn_conv_kernel": 4, "attn_output_gate": True, "norm_offset1": True}),
    "qwen3_dense": ModelConfig(**{**BASE, "architecture": "Qwen3ForCausalLM", "num_experts": 0, "intermediate_size": 192}),
    "llama_dense": ModelConfig(**{**BASE, "architecture": "LlamaForCausalLM", "num_experts": 0, "intermediate_size": 192,
                                  "qk_norm": "none", "tie_embeddings": True}),
}


def _rt(**kw):
    base = dict(num_mb=2, page_size=16, num_pages=64, max_running_requests=8, max_seq_len=128, cuda_graph_max_bs=8,
                device="cpu", dtype="float32", use_cuda_graph=False, max_batched_tokens=24)
    base.update(kw)
    return RuntimeConfig(**base)


@pytest.mark.parametrize("name", list(FAMILIES))
def test_family_generation_matches_reference(name):
    cfg = FAMILIES[name]
    eng = AfdEngine(cfg, _rt(), AfdTopology(colocated=True), 0, "cpu", seed=2, max_comm_tokens=16)
    g = torch.Generator().manual_seed(5)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (21, 9, 30)]
    out = SpmdDriver(eng).generate(prompts, SamplingParams(max_tokens=5, ignore_eos=True))
    stages = [eng.expert_stage] if eng.expert_stage is not None else []
    assert out == greedy_generate_reference(cfg, eng.attn.model, stages, prompts, 5)


def test_hf_config_parsing():
    qwen3 = ModelConfig.from_hf({"architectures": ["Qwen3MoeForCausalLM"], "hidden_size": 2048, "num_hidden_layers": 48,
                                 "num_attention_heads": 32, "num_key_value_heads": 4, "head_dim": 128, "vocab_size": 151936,
                                 "num_experts": 128, "num_experts_per_tok": 8, "moe_intermediate_size": 768,
                                 "rope_theta": 1e6, "norm_topk_prob": True,
                                 "quantization_config": {"quant_method": "fp8", "weight_block_size": [128, 128]}})
    assert qwen3.is_moe and qwen3.quant.is_fp8 and qwen3.quant.block == (128, 128) and qwen3.qk_norm == "head"
    mm = ModelConfig.from_hf({"architectures": ["MiniMaxM2ForCausalLM"], "hidden_size": 3072, "num_hidden_layers": 62,
                              "num_attention_heads": 48, "num_key_value_heads": 8, "head_dim": 128, "vocab_size": 200064,
                              "num_local_experts": 256, "num_experts_per_tok": 8, "intermediate_size": 1536,
                              "rotary_dim": 64, "rope_theta": 5e6})
    assert mm.scoring == "sigmoid" and mm.router_bias and mm.qk_norm == "cross_head" and mm.rotary_dim == 64
    q35 = ModelConfig.from_hf({"architectures": ["Qwen3_5MoeForConditionalGeneration"], "text_config": {
        "hidden_size": 4096, "num_hidden_layers": 8, "num_attention_heads": 32, "num_key_value_heads": 2, "head_dim": 256,
        "vocab_size": 248320, "num_experts": 512, "num_experts_per_tok": 10, "moe_intermediate_size": 1024,
        "shared_expert_intermediate_size": 1024, "full_attention_interval": 4, "partial_rotary_factor": 0.25}})
    assert q35.layer_types == ("linear", "linear", "linear", "full") * 2 and q35.rotary_dim == 64 and q35.norm_offset1
    assert q35.num_full_attn_layers == 2 and q35.kv_bytes_per_token() == 2 * 2 * 2 * 256 * 2


def test_rope_scaling_tables():
    import math

    import torch

    from fastafd_b200.reference import ops_ref as ref

    rot, theta = 64, 10000.0
    base = 1.0 / (theta ** (torch.arange(0, rot, 2, dtype=torch.float32) / rot))
    assert torch.equal(ref.scale_inv_freq(base, rot, theta, None), base)
    lin = ref.scale_inv_freq(base, rot, theta, {"rope_type": "linear", "factor": 4.0})
    assert torch.allclose(lin, base / 4)
    l3 = ref.scale_inv_freq(base, rot, theta, {"rope_type": "llama3", "factor": 8.0, "low_freq_factor": 1.0,
                                                 "high_freq_factor": 4.0, "original_max_position_embeddings": 8192})
    wave = 2 * math.pi / base
    assert torch.allclose(l3[wave < 8192 / 4], base[wave < 8192 / 4])          # short wavelengths untouched
    assert torch.allclose(l3[wave > 8192], base[wave > 8192] / 8)              # long ones slowed by the factor
    mid = (wave >= 8192 / 4) & (wave <= 8192)
    assert bool(((l3[mid] <= base[mid] + 1e-12) & (l3[mid] >= base[mid] / 8 - 1e-12)).all())
    yarn = ref.scale_inv_freq(base, rot, theta, {"rope_type": "yarn", "factor": 4.0,
                                                   "original_max_position_embeddings": 4096})
    assert torch.allclose(yarn[0], base[0]) and torch.allclose(yarn[-1], base[-1] / 4)
    assert bool((yarn[1:] / base[1:] <= yarn[:-1] / base[:-1] + 1e-7).all())   # monotone ramp
    table = ref.build_cos_sin_cache(128, rot, theta, scaling={"rope_type": "yarn", "factor": 4.0,
                                                               "original_max_position_embeddings": 4096})
    assert table.shape == (128, rot)


def test_stop_tokens_come_from_config_and_generation_config(tmp_path):
    import json

    from fastafd_b200.config import PRESETS, ModelConfig, get_model_config

    hf = PRESETS["tiny-qwen3-moe"].to_hf()
    hf["eos_token_id"] = 7
    (tmp_path / "config.json").write_text(json.dumps(hf))
    assert get_model_config(str(tmp_path)).eos_token_ids == (7,)
    (tmp_path / "generation_config.json").write_text(json.dumps({"eos_token_id": [9, 7], "temperature": 0.6}))
    assert ModelConfig.from_path(str(tmp_path)).eos_token_ids == (7, 9)
    (tmp_path / "generation_config.json").write_text(json.dumps({"eos_token_id": 11}))
    assert ModelConfig.from_path(str(tmp_path)).eos_token_ids == (7, 11)
    (tmp_path / "generation_config.json").write_text("{ not json")
    assert ModelConfig.from_path(str(tmp_path)).eos_token_ids == (7,)


def test_config_variants_that_are_not_served_as_written():
    import pytest

    from fastafd_b200.config import PRESETS, ModelConfig

    moe = PRESETS["tiny-qwen3-moe"].to_hf()
    assert ModelConfig.from_hf(dict(moe, mlp_only_layers=[], decoder_sparse_step=1)).num_experts > 0
    for bad in (dict(mlp_only_layers=[0]), dict(decoder_sparse_step=2)):
        with pytest.raises(ValueError, match="dense layers among the MoE layers"):
            ModelConfig.from_hf(dict(moe, **bad))
    mistral = dict(architectures=["MistralForCausalLM"], hidden_size=64, num_hidden_layers=2, num_attention_heads=4,
                   num_key_value_heads=2, vocab_size=256, intermediate_size=128, max_position_embeddings=32768)
    assert ModelConfig.from_hf(dict(mistral, sliding_window=4096)).max_position == 4096          # served within its window
    assert ModelConfig.from_hf(dict(mistral, sliding_window=None)).max_position == 32768
    for bad, pattern in ((dict(mlp_bias=True), "mlp_bias"), (dict(hidden_act="gelu"), "activation")):
        with pytest.raises(ValueError, match=pattern):
            ModelConfig.from_hf(dict(mistral, **bad))
    qwen2 = dict(mistral, architectures=["Qwen2ForCausalLM"], sliding_window=4096)
    assert ModelConfig.from_hf(dict(qwen2, use_sliding_window=False)).max_position == 32768       # declared but switched off
    assert ModelConfig.from_hf(dict(qwen2, use_sliding_window=True)).max_position == 4096


def test_unknown_architectures_are_refused_by_name():
    import pytest

    from fastafd_b200.config import PRESETS, SUPPORTED_ARCHITECTURES, ModelConfig

    with pytest.raises(ValueError, match="DeepseekV3ForCausalLM.*not served"):
        ModelConfig.from_hf({"architectures": ["DeepseekV3ForCausalLM"], "hidden_size": 64, "num_attention_heads": 4})
    assert all(c.architecture in SUPPORTED_ARCHITECTURES for c in PRESETS.values())


def test_tensor_parallel_size_must_divide_the_linear_attention_heads():
    import pytest

    from fastafd_b200.protocol import AfdTopology, validate_parallel_args

    ok = AfdTopology(attn_dp=1, attn_tp=2, mlp_ep=1)
    validate_parallel_args(ok, 8, 4, 2, linear_k_heads=2, linear_v_heads=4)
    with pytest.raises(ValueError, match="linear-attention key heads"):
        validate_parallel_args(AfdTopology(attn_dp=1, attn_tp=4, mlp_ep=1), 8, 4, 2, linear_k_heads=2, linear_v_heads=4)
    with pytest.raises(ValueError, match="linear-attention value heads"):
        validate_parallel_args(AfdTopology(attn_dp=1, attn_tp=4, mlp_ep=1), 8, 4, 2, linear_k_heads=4, linear_v_heads=6)
