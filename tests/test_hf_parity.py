"""Every model family against its implementation in the `transformers` library (CPU, fp32, tiny random models).

A model of the family is built with `transformers`, saved the way the library saves a checkpoint (safetensors,
the family's own key names and row layouts, the `config.json` that version of the library writes), served by
this package's engine from that directory, and the greedy continuations are compared with the library's own
forward pass token by token. This pins, per family, the config parsing, the checkpoint key mapping and row
layouts (merged projections, per-head query|gate rows, grouped gated-DeltaNet projections, depthwise conv
taps), and the model math (norm variants, partial rotary embedding, q/k norms per head and across heads,
softmax / sigmoid / grouped routing, shared experts and their gates, gated attention, gated DeltaNet).
"""
import pytest
import torch

transformers = pytest.importorskip("transformers")

from fastafd_b200.core import SamplingParams  # noqa: E402
from fastafd_b200.llm import LLM  # noqa: E402

COMMON = dict(vocab_size=256, hidden_size=64, num_hidden_layers=3, num_attention_heads=4, num_key_value_heads=2,
              max_position_embeddings=256, tie_word_embeddings=False)
GDN = dict(head_dim=16, moe_intermediate_size=32, num_experts=8, num_experts_per_tok=2, shared_expert_intermediate_size=32,
           linear_num_key_heads=2, linear_num_value_heads=4, linear_key_head_dim=16, linear_value_head_dim=16,
           linear_conv_kernel_dim=4, layer_types=["linear_attention", "linear_attention", "full_attention"])

FAMILIES = {
    "llama": ("LlamaForCausalLM", "LlamaConfig", dict(intermediate_size=128, rope_theta=10000.0)),
    "llama-tied-embeddings": ("LlamaForCausalLM", "LlamaConfig", dict(intermediate_size=128, tie_word_embeddings=True)),
    "qwen2": ("Qwen2ForCausalLM", "Qwen2Config", dict(intermediate_size=128, rope_theta=1e6)),
    "mistral": ("MistralForCausalLM", "MistralConfig", dict(intermediate_size=128, head_dim=16, sliding_window=None)),
    "qwen3": ("Qwen3ForCausalLM", "Qwen3Config", dict(intermediate_size=128, head_dim=16)),
    "qwen3-moe": ("Qwen3MoeForCausalLM", "Qwen3MoeConfig",
                  dict(intermediate_size=128, head_dim=16, moe_intermediate_size=32, num_experts=8, num_experts_per_tok=2,
                       norm_topk_prob=True, decoder_sparse_step=1, mlp_only_layers=[])),
    "glm4-moe": ("Glm4MoeForCausalLM", "Glm4MoeConfig",
                 dict(intermediate_size=128, head_dim=16, moe_intermediate_size=32, n_routed_experts=8, num_experts_per_tok=2,
                      n_shared_experts=1, n_group=2, topk_group=1, first_k_dense_replace=1, norm_topk_prob=True,
                      routed_scaling_factor=1.5, use_qk_norm=True, partial_rotary_factor=0.5)),
    "minimax-m2": ("MiniMaxM2ForCausalLM", "MiniMaxM2Config",
                   dict(intermediate_size=32, head_dim=16, num_local_experts=8, num_experts_per_tok=2, use_qk_norm=True,
                        rope_parameters={"rope_theta": 5e6, "rope_type": "default", "partial_rotary_factor": 0.5})),
    "qwen3.5-moe": ("Qwen3_5MoeForCausalLM", "Qwen3_5MoeTextConfig", dict(GDN)),
    # variants: rotary scaling rules, routing without renormalisation, attention bias, several shared experts
    "llama-rope-llama3": ("LlamaForCausalLM", "LlamaConfig",
                          dict(intermediate_size=128, rope_parameters={"rope_type": "llama3", "rope_theta": 10000.0, "factor": 8.0,
                                                                       "low_freq_factor": 1.0, "high_freq_factor": 4.0,
                                                                       "original_max_position_embeddings": 64})),
    "qwen3-rope-yarn": ("Qwen3ForCausalLM", "Qwen3Config",
                        dict(intermediate_size=128, head_dim=16, rope_parameters={"rope_type": "yarn", "rope_theta": 1e6, "factor": 4.0,
                                                                                  "original_max_position_embeddings": 64})),
    "llama-rope-linear": ("LlamaForCausalLM", "LlamaConfig",
                          dict(intermediate_size=128, rope_parameters={"rope_type": "linear", "rope_theta": 10000.0, "factor": 2.0})),
    "qwen2-tied-embeddings": ("Qwen2ForCausalLM", "Qwen2Config", dict(intermediate_size=128, tie_word_embeddings=True)),
    "glm4-moe-bias-no-qk-norm": ("Glm4MoeForCausalLM", "Glm4MoeConfig",
                                 dict(intermediate_size=128, head_dim=16, moe_intermediate_size=32, n_routed_experts=8,
                                      num_experts_per_tok=2, n_shared_experts=2, n_group=1, topk_group=1, first_k_dense_replace=0,
                                      norm_topk_prob=False, routed_scaling_factor=2.5, use_qk_norm=False, partial_rotary_factor=0.5,
                                      attention_bias=True)),
    "qwen3-moe-top3-no-renorm": ("Qwen3MoeForCausalLM", "Qwen3MoeConfig",
                                 dict(intermediate_size=128, head_dim=16, moe_intermediate_size=32, num_experts=8, num_experts_per_tok=3,
                                      norm_topk_prob=False, decoder_sparse_step=1, mlp_only_layers=[])),
    "qwen3-next": ("Qwen3NextForCausalLM", "Qwen3NextConfig", dict(GDN, decoder_sparse_step=1, mlp_only_layers=[])),
    # routing: four groups of which two are kept, top-4 of 16 experts
    "glm4-moe-groups-4-keep-2": ("Glm4MoeForCausalLM", "Glm4MoeConfig",
                                 dict(intermediate_size=128, head_dim=16, moe_intermediate_size=32, n_routed_experts=16,
                                      num_experts_per_tok=4, n_shared_experts=1, n_group=4, topk_group=2, first_k_dense_replace=1,
                                      norm_topk_prob=True, routed_scaling_factor=1.0, use_qk_norm=True, partial_rotary_factor=0.5)),
    "minimax-m2-top4-of-16": ("MiniMaxM2ForCausalLM", "MiniMaxM2Config",
                              dict(intermediate_size=32, head_dim=16, num_local_experts=16, num_experts_per_tok=4, use_qk_norm=True,
                                   rope_parameters={"rope_theta": 5e6, "rope_type": "default", "partial_rotary_factor": 0.5})),
    # four value heads per key head (the ratio of the published models), key and value head dims that differ
    "qwen3.5-moe-head-ratio-4": ("Qwen3_5MoeForCausalLM", "Qwen3_5MoeTextConfig",
                                 dict(GDN, linear_num_key_heads=2, linear_num_value_heads=8, linear_key_head_dim=32,
                                      linear_value_head_dim=16, num_attention_heads=8, num_key_value_heads=2, head_dim=32)),
    "qwen3-next-head-ratio-4": ("Qwen3NextForCausalLM", "Qwen3NextConfig",
                                dict(GDN, decoder_sparse_step=1, mlp_only_layers=[], linear_num_key_heads=2, linear_num_value_heads=8,
                                     linear_key_head_dim=32, linear_value_head_dim=16, num_attention_heads=8, num_key_value_heads=2,
                                     head_dim=32)),
}


def _library_greedy(model, prompt, n):
    """Greedy continuation by whole-sequence forward passes (no cache, no stop token)."""
    ids = list(prompt)
    with torch.no_grad():
        for _ in range(n):
            ids.append(int(model(torch.tensor([ids])).logits[0, -1].argmax()))
    return ids[len(prompt):]


@pytest.mark.parametrize("family", list(FAMILIES))
def test_served_tokens_equal_the_transformers_implementation(family, tmp_path):
    cls_name, cfg_name, extra = FAMILIES[family]
    if not (hasattr(transformers, cls_name) and hasattr(transformers, cfg_name)):
        pytest.skip(f"transformers {transformers.__version__} has no {cls_name}")
    torch.manual_seed(0)
    kw = dict(COMMON)
    kw.update(extra)
    model = getattr(transformers, cls_name)(getattr(transformers, cfg_name)(**kw)).float().eval()
    with torch.no_grad():                      # norm weights, biases, decay and routing offsets away from their defaults
        for _name, p in model.named_parameters():
            if p.dim() == 1:
                p.add_(0.1 * torch.randn_like(p))
    path = str(tmp_path / family)
    model.save_pretrained(path, safe_serialization=True)
    g = torch.Generator().manual_seed(1)
    prompts = [torch.randint(0, 256, (n,), generator=g).tolist() for n in (5, 11, 3)]
    want = [_library_greedy(model, p, 6) for p in prompts]
    llm = LLM(path, device="cpu", num_pages=64, max_seq_len=128)
    try:
        got = [o["token_ids"] for o in llm.generate(prompts, SamplingParams(max_tokens=6, ignore_eos=True))]
    finally:
        llm.shutdown()
    assert got == want


def test_q_gate_row_layout_round_trip():
    from fastafd_b200.models.loader import merge_q_gate_rows, split_q_gate_rows

    heads, d = 3, 4
    w = torch.arange(heads * 2 * d * 5, dtype=torch.float32).reshape(heads * 2 * d, 5)
    s = split_q_gate_rows(w, heads, d)
    assert torch.equal(s[:heads * d].reshape(heads, d, 5), w.reshape(heads, 2, d, 5)[:, 0])       # queries of all heads first
    assert torch.equal(s[heads * d:].reshape(heads, d, 5), w.reshape(heads, 2, d, 5)[:, 1])       # then the gates
    assert torch.equal(merge_q_gate_rows(s, heads, d), w)
    bias = torch.arange(heads * 2 * d, dtype=torch.float32)
    assert torch.equal(merge_q_gate_rows(split_q_gate_rows(bias, heads, d), heads, d), bias)


FP8_SKIP = ("embed_tokens", "lm_head", "norm", "mlp.gate.weight", "block_sparse_moe.gate.weight", "shared_expert_gate", "conv1d",
            "A_log", "dt_bias", "in_proj_a", "in_proj_b", "in_proj_ba", "e_score")


def _fp8_pair(family, tmp_path, inter):
    """(directory with block-FP8 weights + scales, the library model holding the dequantised values)."""
    import glob
    import json

    from safetensors.torch import load_file, save_file

    from fastafd_b200.reference import ops_ref as ref

    cls_name, cfg_name, extra = FAMILIES[family]
    torch.manual_seed(0)
    kw = dict(COMMON)
    kw.update(extra)
    kw["hidden_size"] = 128
    for key in ("moe_intermediate_size", "shared_expert_intermediate_size"):
        if key in kw:
            kw[key] = inter
    if family == "minimax-m2":
        kw["intermediate_size"] = inter
    cls = getattr(transformers, cls_name)
    model = cls(getattr(transformers, cfg_name)(**kw)).float().eval()
    fp8_dir, deq_dir = str(tmp_path / "fp8"), str(tmp_path / "dequantised")
    model.save_pretrained(fp8_dir, safe_serialization=True)
    model.save_pretrained(deq_dir, safe_serialization=True)
    f = glob.glob(fp8_dir + "/*.safetensors")[0]
    sd = {k: v.clone() for k, v in load_file(f).items()}
    out = {}
    for k, w in sd.items():
        if w.dim() == 2 and k.endswith(".weight") and not any(s in k for s in FP8_SKIP):
            q, s = ref.block_quant_fp8(w.float())
            out[k], out[k[:-len("weight")] + "weight_scale_inv"] = q, s.float()
            sd[k] = ref.block_dequant_fp8(q, s.float())
        else:
            out[k] = w
    save_file(out, f, metadata={"format": "pt"})
    save_file(sd, glob.glob(deq_dir + "/*.safetensors")[0], metadata={"format": "pt"})
    cfg = json.load(open(fp8_dir + "/config.json"))
    cfg["quantization_config"] = {"quant_method": "fp8", "fmt": "e4m3", "activation_scheme": "dynamic",
                                  "weight_block_size": [128, 128], "modules_to_not_convert": ["lm_head"]}
    json.dump(cfg, open(fp8_dir + "/config.json", "w"))
    return fp8_dir, cls.from_pretrained(deq_dir, dtype=torch.float32).eval()


@pytest.mark.parametrize("family", ["qwen3-moe", "glm4-moe", "minimax-m2", "qwen3.5-moe", "qwen3-next"])
def test_block_fp8_checkpoints_equal_the_library_on_the_dequantised_weights(family, tmp_path):
    """The same models with every projection and expert matrix stored as e4m3 codes + 128x128 `weight_scale_inv`
    blocks under each family's key names: serving that directory gives the tokens of the library run on the
    dequantised values (on CPU the engine computes with code x scale in fp32, so nothing else differs)."""
    cls_name, cfg_name, _ = FAMILIES[family]
    if not (hasattr(transformers, cls_name) and hasattr(transformers, cfg_name)):
        pytest.skip(f"transformers {transformers.__version__} has no {cls_name}")
    fp8_dir, model = _fp8_pair(family, tmp_path, 128)
    g = torch.Generator().manual_seed(1)
    prompts = [torch.randint(0, 256, (n,), generator=g).tolist() for n in (5, 11, 3)]
    want = [_library_greedy(model, p, 6) for p in prompts]
    llm = LLM(fp8_dir, device="cpu", num_pages=64, max_seq_len=128)
    try:
        got = [o["token_ids"] for o in llm.generate(prompts, SamplingParams(max_tokens=6, ignore_eos=True))]
    finally:
        llm.shutdown()
    assert got == want


def test_block_fp8_experts_with_ragged_gate_up_blocks_are_refused(tmp_path):
    """Gate rows and up rows become one matrix; an intermediate size that is not a multiple of the scale block
    would make them share a block of scales, so such a checkpoint is refused instead of served with wrong scales."""
    fp8_dir, _ = _fp8_pair("qwen3-moe", tmp_path, 32)
    with pytest.raises(ValueError, match="multiple of 128"):
        LLM(fp8_dir, device="cpu", num_pages=64, max_seq_len=128)


@pytest.mark.timeout(300)
@pytest.mark.parametrize("family", ["qwen3.5-moe", "minimax-m2"])
def test_disaggregated_tensor_parallel_serving_of_a_library_checkpoint(family, tmp_path):
    """The same checkpoints behind the HTTP server as four CPU processes: one attention lane of two tensor-parallel
    ranks (head shards of the gated attention and of the gated DeltaNet, the cross-head q/k norm with its
    all-reduce) and two expert-parallel ranks, each reading only its part of the directory."""
    import requests

    from fastafd_b200.server.args import parse_args
    from fastafd_b200.server.launch import local_endpoint
    from fastafd_b200.server.supervisor import LocalSupervisor

    cls_name, cfg_name, extra = FAMILIES[family]
    if not (hasattr(transformers, cls_name) and hasattr(transformers, cfg_name)):
        pytest.skip(f"transformers {transformers.__version__} has no {cls_name}")
    torch.manual_seed(0)
    kw = dict(COMMON)
    kw.update(extra)
    model = getattr(transformers, cls_name)(getattr(transformers, cfg_name)(**kw)).float().eval()
    with torch.no_grad():
        for _name, p in model.named_parameters():
            if p.dim() == 1:
                p.add_(0.1 * torch.randn_like(p))
    path = str(tmp_path / family)
    model.save_pretrained(path, safe_serialization=True)
    g = torch.Generator().manual_seed(1)
    prompts = [torch.randint(0, 256, (n,), generator=g).tolist() for n in (5, 11, 3)]
    want = [_library_greedy(model, p, 6) for p in prompts]
    args = parse_args(["--mode", "afd-serve", "--model-path", path, "--device", "cpu", "--afd-num-mb", "2", "--afd-attn-dp-size", "1",
                       "--afd-attn-tp-size", "2", "--afd-mlp-ep-size", "2", "--num-pages", "64", "--max-seq-len-override", "128",
                       "--afd-max-running-requests", "8", "--cuda-graph-max-bs", "8"])
    sup = LocalSupervisor(args)
    got = []
    with local_endpoint(args, sup) as url:
        for p in prompts:
            r = requests.post(url + "/v1/chat/completions", json={"input_ids": p, "max_tokens": 6, "temperature": 0, "ignore_eos": True,
                                                                  "return_token_ids": True, "stream": False}, timeout=200).json()
            got.append(r["choices"][0]["token_ids"])
        assert sup.get_failures() == []
    assert got == want


def test_extra_layers_behind_the_last_one_are_not_read(tmp_path):
    """GLM-4.5 checkpoints carry a next-token-prediction block as decoder layer `num_hidden_layers` (its own
    experts included). It is not served; its tensors are skipped whatever their shapes."""
    import glob

    from safetensors.torch import load_file, save_file

    cls_name, cfg_name, extra = FAMILIES["glm4-moe"]
    torch.manual_seed(0)
    kw = dict(COMMON)
    kw.update(extra)
    model = getattr(transformers, cls_name)(getattr(transformers, cfg_name)(**kw)).float().eval()
    path = str(tmp_path / "glm")
    model.save_pretrained(path, safe_serialization=True)
    f = glob.glob(path + "/*.safetensors")[0]
    sd = {k: v.clone() for k, v in load_file(f).items()}
    n = kw["num_hidden_layers"]
    sd[f"model.layers.{n}.eh_proj.weight"] = torch.randn(7, 3)
    sd[f"model.layers.{n}.mlp.experts.0.gate_proj.weight"] = torch.randn(5, 5)
    sd[f"model.layers.{n}.self_attn.q_proj.weight"] = torch.randn(2, 2)
    save_file(sd, f, metadata={"format": "pt"})
    prompts = [[5, 9, 2, 44, 17], [8, 3]]
    want = [_library_greedy(model, p, 4) for p in prompts]
    llm = LLM(path, device="cpu", num_pages=64, max_seq_len=128)
    try:
        got = [o["token_ids"] for o in llm.generate(prompts, SamplingParams(max_tokens=4, ignore_eos=True))]
    finally:
        llm.shutdown()
    assert got == want


def test_checkpoint_key_prefixes_of_multimodal_wrappers():
    """Text models inside multimodal wrappers: every nesting of `language_model.` in front of the text model's keys
    maps to the plain key; vision towers and next-token-prediction heads are not read."""
    from fastafd_b200.models.loader import normalize_key as n

    cases = {"model.language_model.layers.3.self_attn.q_proj.weight": "model.layers.3.self_attn.q_proj.weight",
             "model.language_model.embed_tokens.weight": "model.embed_tokens.weight",
             "language_model.model.layers.0.input_layernorm.weight": "model.layers.0.input_layernorm.weight",
             "language_model.lm_head.weight": "lm_head.weight",
             "model.language_model.language_model.norm.weight": "model.norm.weight",
             "model.layers.0.mlp.gate.weight": "model.layers.0.mlp.gate.weight", "lm_head.weight": "lm_head.weight",
             "model.layers.0.block_sparse_moe.gate.weight": "model.layers.0.mlp.gate.weight",
             "model.layers.0.mlp.shared_experts.up_proj.weight": "model.layers.0.mlp.shared_expert.up_proj.weight",
             "model.visual.blocks.0.attn.qkv.weight": None, "model.language_model.visual.merger.norm.weight": None,
             "mtp.layers.0.self_attn.q_proj.weight": None, "model.layers.0.self_attn.rotary_emb.inv_freq": None}
    for key, want in cases.items():
        assert n(key) == want, (key, n(key), want)


def test_qwen35_inside_its_multimodal_wrapper(tmp_path):
    """Qwen3.5 as published: `Qwen3_5MoeForConditionalGeneration` with the text model under `text_config` and a
    vision tower beside it. Text-only requests give the library's tokens; the tower is never read."""
    T = transformers
    if not all(hasattr(T, n) for n in ("Qwen3_5MoeForConditionalGeneration", "Qwen3_5MoeConfig", "Qwen3_5MoeTextConfig")):
        pytest.skip("no Qwen3.5 multimodal classes in this transformers")
    kw = dict(COMMON)
    kw.update(GDN)
    vision = dict(depth=1, hidden_size=32, intermediate_size=64, num_heads=2, out_hidden_size=64, patch_size=2, spatial_merge_size=1,
                  temporal_patch_size=1, in_channels=3, num_position_embeddings=16)
    torch.manual_seed(0)
    model = T.Qwen3_5MoeForConditionalGeneration(T.Qwen3_5MoeConfig(text_config=T.Qwen3_5MoeTextConfig(**kw).to_dict(),
                                                                   vision_config=vision)).float().eval()
    path = str(tmp_path / "wrapped")
    model.save_pretrained(path, safe_serialization=True)
    prompts = [[5, 9, 2, 44, 17, 3, 200], [8, 3, 99]]
    want = []
    for p in prompts:
        ids = list(p)
        with torch.no_grad():
            for _ in range(5):
                ids.append(int(model(input_ids=torch.tensor([ids])).logits[0, -1].argmax()))
        want.append(ids[len(p):])
    llm = LLM(path, device="cpu", num_pages=64, max_seq_len=128)
    try:
        got = [o["token_ids"] for o in llm.generate(prompts, SamplingParams(max_tokens=5, ignore_eos=True))]
    finally:
        llm.shutdown()
    assert got == want


def test_alignment_tool_against_the_library(tmp_path, capsys):
    """`python -m fastafd_b200.validate --model-path DIR --against transformers`: the alignment report (identical
    share, first divergence, rank gate) with the library's implementation as the other side; and with the package's
    own whole-sequence forward of the same directory."""
    import json

    from fastafd_b200 import validate

    cls_name, cfg_name, extra = FAMILIES["minimax-m2"]
    torch.manual_seed(0)
    kw = dict(COMMON)
    kw.update(extra)
    path = str(tmp_path / "m")
    getattr(transformers, cls_name)(getattr(transformers, cfg_name)(**kw)).float().save_pretrained(path, safe_serialization=True)
    common = ["--model-path", path, "--device", "cpu", "--prompts", "2", "--prompt-len", "9", "--decode", "4"]
    assert validate.main(common + ["--against", "transformers"]) == 0
    rep = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert rep["against"] == "transformers" and rep["verdict"] == "pass" and rep["match"] == 1.0
    assert rep["rank_gate"]["worst_rank"] == 0 and rep["first_divergence"] == [4, 4]
    assert validate.main(common) == 0
    assert json.loads(capsys.readouterr().out.strip().splitlines()[-1])["against"] == "oracle"


def test_core_attention_disaggregation_on_a_library_checkpoint(tmp_path, monkeypatch):
    """MiniMax-M2 (the model the reference runs this mode on) saved by the library, served with the attention core on
    two attention ranks and everything else on a model rank (one process, CPU): the library's tokens."""
    cls_name, cfg_name, extra = FAMILIES["minimax-m2"]
    if not (hasattr(transformers, cls_name) and hasattr(transformers, cfg_name)):
        pytest.skip(f"transformers {transformers.__version__} has no {cls_name}")
    torch.manual_seed(0)
    kw = dict(COMMON)
    kw.update(extra)
    model = getattr(transformers, cls_name)(getattr(transformers, cfg_name)(**kw)).float().eval()
    with torch.no_grad():
        for _name, p in model.named_parameters():
            if p.dim() == 1:
                p.add_(0.1 * torch.randn_like(p))
    path = str(tmp_path / "m2")
    model.save_pretrained(path, safe_serialization=True)
    g = torch.Generator().manual_seed(1)
    prompts = [torch.randint(0, 256, (n,), generator=g).tolist() for n in (5, 11, 3, 20)]
    want = [_library_greedy(model, p, 6) for p in prompts]
    monkeypatch.setenv("MINISGL_AFD_MODE", "cad")
    monkeypatch.setenv("FASTAFD_CAD_ATTN_PER_MODEL", "2")
    llm = LLM(path, device="cpu", num_pages=64, max_seq_len=128, num_mb=2)
    try:
        assert type(llm.coordinator).__name__ == "CadCoordinator"
        got = [o["token_ids"] for o in llm.generate(prompts, SamplingParams(max_tokens=6, ignore_eos=True))]
    finally:
        llm.shutdown()
    assert got == want


def test_hybrid_model_under_queueing_slot_reuse_and_chunked_prefill(tmp_path):
    """Ten requests through three request slots, prompts up to 40 tokens prefilled 16 tokens at a time, two
    micro-batches: every request slot (and with it a recurrent-state slot and conv taps) is reused several times
    and prompts are split over steps; each request still gets the library's tokens."""
    cls_name, cfg_name, extra = FAMILIES["qwen3.5-moe"]
    if not (hasattr(transformers, cls_name) and hasattr(transformers, cfg_name)):
        pytest.skip(f"transformers {transformers.__version__} has no {cls_name}")
    torch.manual_seed(0)
    kw = dict(COMMON)
    kw.update(extra)
    model = getattr(transformers, cls_name)(getattr(transformers, cfg_name)(**kw)).float().eval()
    with torch.no_grad():
        for _name, p in model.named_parameters():
            if p.dim() == 1:
                p.add_(0.1 * torch.randn_like(p))
    path = str(tmp_path / "hybrid")
    model.save_pretrained(path, safe_serialization=True)
    g = torch.Generator().manual_seed(3)
    prompts = [torch.randint(0, 256, (n,), generator=g).tolist() for n in (7, 33, 12, 5, 40, 9, 21, 3, 18, 26)]
    max_tokens = [3, 6, 2, 7, 4, 5, 1, 6, 3, 4]
    want = [_library_greedy(model, p, n) for p, n in zip(prompts, max_tokens)]
    llm = LLM(path, device="cpu", num_pages=64, max_seq_len=128, max_running_requests=3, cuda_graph_max_bs=4, num_mb=2,
              max_batched_tokens=16)
    try:
        got = [o["token_ids"] for o in llm.generate(prompts, [SamplingParams(max_tokens=n, ignore_eos=True) for n in max_tokens])]
    finally:
        llm.shutdown()
    assert got == want
