"""Model, quantisation and runtime configuration.

``ModelConfig.from_hf`` reads a Hugging Face ``config.json`` dict (Qwen3-MoE, Qwen3.5-MoE
hybrid, MiniMax-M2, GLM-4-MoE, and the dense Llama / Qwen2 / Qwen3 / Mistral families);
``PRESETS`` holds the benchmark shapes so that synthetic random-init runs need no files.

Reference: python/minisgl/models/config.py (ModelConfig.from_hf, QuantConfig, layer_types),
python/minisgl/engine/config.py, python/minisgl/scheduler/config.py.
"""
from __future__ import annotations

import json
from dataclasses import dataclass, replace
from pathlib import Path
from typing import Any, Dict, Optional, Tuple


@dataclass(frozen=True)
class QuantConfig:
    """``fp8``: e4m3 weights with 128x128 ``weight_scale_inv`` blocks and dynamic 1x128
    activation scales. ``fp8_channel``: per-output-channel weight scales (requantised to
    blocks at load)."""
    method: str = "none"            # none | fp8 | fp8_channel
    block: Tuple[int, int] = (128, 128)
    ignored_modules: Tuple[str, ...] = ()

    @property
    def is_fp8(self) -> bool:
        return self.method in ("fp8", "fp8_channel")

    def applies_to(self, module_name: str) -> bool:
        return self.is_fp8 and not any(module_name.endswith(m) or m in module_name for m in self.ignored_modules)


@dataclass(frozen=True)
class RopeConfig:
    theta: float = 1e6
    rotary_dim: int = 0             # 0 -> head_dim
    scaling: Optional[Dict[str, Any]] = None   # llama3 / yarn parameters


SUPPORTED_ARCHITECTURES = ("LlamaForCausalLM", "MistralForCausalLM", "Qwen2ForCausalLM", "Qwen3ForCausalLM",
                           "Qwen3MoeForCausalLM", "Glm4MoeForCausalLM", "MiniMaxM2ForCausalLM", "Qwen3_5MoeForCausalLM",
                           "Qwen3_5MoeForConditionalGeneration", "Qwen3NextForCausalLM")


@dataclass(frozen=True)
class ModelConfig:
    architecture: str = "Qwen3MoeForCausalLM"
    num_layers: int = 4
    hidden_size: int = 256
    num_q_heads: int = 4
    num_kv_heads: int = 2
    head_dim: int = 64
    vocab_size: int = 1024
    rms_eps: float = 1e-6
    rope: RopeConfig = RopeConfig()
    max_position: int = 40960
    tie_embeddings: bool = False
    qk_norm: str = "head"           # none | head (per-head RMSNorm) | cross_head (MiniMax)
    attention_bias: bool = False
    # dense MLP (dense models, GLM first-k dense layers, shared experts)
    intermediate_size: int = 0
    # MoE
    num_experts: int = 8
    num_experts_per_tok: int = 2
    moe_intermediate_size: int = 512
    norm_topk_prob: bool = True
    scoring: str = "softmax"        # softmax | sigmoid
    router_bias: bool = False       # e_score_correction_bias (MiniMax, GLM)
    router_fp32: bool = False       # keep the gate weight in fp32 (MiniMax)
    routed_scaling_factor: float = 1.0
    n_group: int = 1
    topk_group: int = 1
    num_shared_experts: int = 0
    shared_expert_intermediate_size: int = 0
    shared_expert_gate: bool = False      # Qwen3.5: sigmoid gate on the shared expert
    first_k_dense: int = 0          # GLM: leading dense layers
    # hybrid (Qwen3.5): per-layer type "full" | "linear"
    layer_types: Tuple[str, ...] = ()
    gdn_num_k_heads: int = 0
    gdn_num_v_heads: int = 0
    gdn_head_k_dim: int = 0
    gdn_head_v_dim: int = 0
    gdn_conv_kernel: int = 4
    attn_output_gate: bool = False  # Qwen3.5 full attention: q||gate, sigmoid output gate
    norm_offset1: bool = False      # RMSNorm weights stored as (w - 1)
    quant: QuantConfig = QuantConfig()
    dtype: str = "bfloat16"
    eos_token_ids: Tuple[int, ...] = ()

    # ------------------------------------------------------------------ derived
    @property
    def is_moe(self) -> bool:
        return self.num_experts > 0

    @property
    def rotary_dim(self) -> int:
        return self.rope.rotary_dim or self.head_dim

    @property
    def q_size(self) -> int:
        return self.num_q_heads * self.head_dim

    @property
    def kv_size(self) -> int:
        return self.num_kv_heads * self.head_dim

    def layer_type(self, layer: int) -> str:
        return self.layer_types[layer] if self.layer_types else "full"

    def is_moe_layer(self, layer: int) -> bool:
        return self.is_moe and layer >= self.first_k_dense

    @property
    def num_full_attn_layers(self) -> int:
        return sum(1 for i in range(self.num_layers) if self.layer_type(i) == "full")

    @property
    def num_linear_layers(self) -> int:
        return self.num_layers - self.num_full_attn_layers

    def kv_bytes_per_token(self, tp: int = 1, elem: int = 2) -> int:
        kv_heads = max(1, self.num_kv_heads // tp)
        return 2 * self.num_full_attn_layers * kv_heads * self.head_dim * elem

    def with_layers(self, n: int) -> "ModelConfig":
        lt = self.layer_types[:n] if self.layer_types else ()
        return replace(self, num_layers=n, layer_types=lt)

    # ------------------------------------------------------------------ HF
    @staticmethod
    def from_hf(cfg: Dict[str, Any]) -> "ModelConfig":
        if "text_config" in cfg and "architectures" in cfg:   # Qwen3.5 wraps the text model
            inner = dict(cfg["text_config"])
            inner.setdefault("architectures", cfg["architectures"])
            if "quantization_config" in cfg:
                inner.setdefault("quantization_config", cfg["quantization_config"])
            cfg = inner
        arch = (cfg.get("architectures") or ["LlamaForCausalLM"])[0]

        if arch not in SUPPORTED_ARCHITECTURES:
            raise ValueError(f"architecture {arch!r} is not served; supported: {', '.join(SUPPORTED_ARCHITECTURES)}")

        def experts() -> int:
            """Routed experts: the key differs by family and by the library version that wrote the file."""
            for k in ("num_experts", "num_local_experts", "n_routed_experts"):
                if cfg.get(k):
                    return int(cfg[k])
            raise KeyError(f"{arch}: config.json names no expert count (num_experts / num_local_experts / n_routed_experts)")

        hidden = cfg["hidden_size"]
        heads = cfg["num_attention_heads"]
        head_dim = cfg.get("head_dim") or hidden // heads
        rope_scaling = cfg.get("rope_scaling") or cfg.get("rope_parameters")
        theta = cfg.get("rope_theta") or (rope_scaling or {}).get("rope_theta", 10000.0)
        partial = cfg.get("partial_rotary_factor") or (rope_scaling or {}).get("partial_rotary_factor") or 1.0
        rotary_dim = cfg.get("rotary_dim") or int(head_dim * partial)
        q = cfg.get("quantization_config") or {}
        quant = QuantConfig()
        if q.get("quant_method") == "fp8":
            blk = tuple(q.get("weight_block_size") or (128, 128))
            method = "fp8" if q.get("weight_block_size") else "fp8_channel"
            ignored = tuple(q.get("modules_to_not_convert") or q.get("ignored_layers") or ())
            quant = QuantConfig(method, blk, ignored)
        eos = cfg.get("eos_token_id")
        eos_ids = tuple(eos) if isinstance(eos, (list, tuple)) else ((eos,) if eos is not None else ())
        kw: Dict[str, Any] = dict(
            architecture=arch, num_layers=cfg["num_hidden_layers"], hidden_size=hidden,
            num_q_heads=heads, num_kv_heads=cfg.get("num_key_value_heads", heads), head_dim=head_dim,
            vocab_size=cfg["vocab_size"], rms_eps=cfg.get("rms_norm_eps", 1e-6),
            rope=RopeConfig(float(theta), rotary_dim if rotary_dim != head_dim else 0,
                            rope_scaling if rope_scaling and rope_scaling.get("rope_type", rope_scaling.get("type")) not in (None, "default") else None),
            max_position=cfg.get("max_position_embeddings", 32768),
            tie_embeddings=bool(cfg.get("tie_word_embeddings", False)),
            attention_bias=bool(cfg.get("attention_bias", False)),
            intermediate_size=cfg.get("intermediate_size", 0) or 0,
            quant=quant, eos_token_ids=eos_ids, num_experts=0, qk_norm="none",
        )
        if arch in ("Qwen3ForCausalLM",):
            kw.update(qk_norm="head")
        if arch in ("Qwen2ForCausalLM",):
            kw.update(attention_bias=True)
        if cfg.get("mlp_bias"):
            raise ValueError(f"{arch}: MLP projections with a bias (mlp_bias) are not supported")
        if cfg.get("hidden_act", "silu") not in ("silu", "swish"):
            raise ValueError(f"{arch}: activation {cfg.get('hidden_act')!r} is not supported (SwiGLU with SiLU only)")
        # Attention over a sliding window is not implemented; within the window it equals full attention, so a model
        # that uses one is served up to its window length.
        window = cfg.get("sliding_window")
        if window and cfg.get("use_sliding_window", arch.startswith("Mistral")) and int(window) < kw["max_position"]:
            kw["max_position"] = int(window)
        if arch in ("Qwen3MoeForCausalLM", "Qwen3_5MoeForCausalLM", "Qwen3_5MoeForConditionalGeneration", "Qwen3NextForCausalLM"):
            if cfg.get("mlp_only_layers") or int(cfg.get("decoder_sparse_step", 1) or 1) != 1:
                raise ValueError(f"{arch}: dense layers among the MoE layers (mlp_only_layers / decoder_sparse_step) are not supported")
        if arch == "Qwen3MoeForCausalLM":
            kw.update(qk_norm="head", num_experts=experts(), num_experts_per_tok=cfg["num_experts_per_tok"],
                      moe_intermediate_size=cfg["moe_intermediate_size"],
                      norm_topk_prob=bool(cfg.get("norm_topk_prob", True)))
        elif arch == "MiniMaxM2ForCausalLM":
            kw.update(qk_norm="cross_head" if cfg.get("use_qk_norm", True) else "none",
                      num_experts=experts(), num_experts_per_tok=cfg["num_experts_per_tok"],
                      moe_intermediate_size=cfg["intermediate_size"], scoring="sigmoid", router_bias=True,
                      router_fp32=True, norm_topk_prob=True)
        elif arch == "Glm4MoeForCausalLM":
            kw.update(qk_norm="head" if cfg.get("use_qk_norm", False) else "none",
                      num_experts=experts(), num_experts_per_tok=cfg["num_experts_per_tok"],
                      moe_intermediate_size=cfg["moe_intermediate_size"], scoring="sigmoid", router_bias=True,
                      norm_topk_prob=bool(cfg.get("norm_topk_prob", True)),
                      routed_scaling_factor=float(cfg.get("routed_scaling_factor", 1.0)),
                      n_group=cfg.get("n_group", 1), topk_group=cfg.get("topk_group", 1),
                      num_shared_experts=cfg.get("n_shared_experts", 0),
                      shared_expert_intermediate_size=cfg.get("n_shared_experts", 0) * cfg["moe_intermediate_size"],
                      first_k_dense=cfg.get("first_k_dense_replace", 0))
        elif arch in ("Qwen3_5MoeForCausalLM", "Qwen3_5MoeForConditionalGeneration", "Qwen3NextForCausalLM"):
            n = cfg["num_hidden_layers"]
            lt = cfg.get("layer_types")
            if lt is None:
                interval = cfg.get("full_attention_interval", 4)
                lt = ["full_attention" if (i + 1) % interval == 0 else "linear_attention" for i in range(n)]
            kw.update(qk_norm="head", num_experts=experts(), num_experts_per_tok=cfg["num_experts_per_tok"],
                      moe_intermediate_size=cfg["moe_intermediate_size"],
                      norm_topk_prob=bool(cfg.get("norm_topk_prob", True)), num_shared_experts=1,
                      shared_expert_intermediate_size=cfg.get("shared_expert_intermediate_size", 0),
                      shared_expert_gate=True,
                      layer_types=tuple("full" if t.startswith("full") else "linear" for t in lt),
                      gdn_num_k_heads=cfg.get("linear_num_key_heads", 16),
                      gdn_num_v_heads=cfg.get("linear_num_value_heads", 64),
                      gdn_head_k_dim=cfg.get("linear_key_head_dim", 128),
                      gdn_head_v_dim=cfg.get("linear_value_head_dim", 128),
                      gdn_conv_kernel=cfg.get("linear_conv_kernel_dim", 4),
                      attn_output_gate=True, norm_offset1=True)
        return ModelConfig(**kw)

    def to_hf(self) -> Dict[str, Any]:
        """The ``config.json`` dict that :meth:`from_hf` reads back into this configuration
        (used when a synthetic checkpoint is written for tests or offline conversion)."""
        out: Dict[str, Any] = dict(
            architectures=[self.architecture], hidden_size=self.hidden_size, num_hidden_layers=self.num_layers,
            num_attention_heads=self.num_q_heads, num_key_value_heads=self.num_kv_heads, head_dim=self.head_dim,
            vocab_size=self.vocab_size, rms_norm_eps=self.rms_eps, rope_theta=self.rope.theta,
            max_position_embeddings=self.max_position, tie_word_embeddings=self.tie_embeddings,
            attention_bias=self.attention_bias, intermediate_size=self.intermediate_size, torch_dtype=self.dtype)
        if self.rope.rotary_dim:
            out["rotary_dim"] = self.rope.rotary_dim
        if self.rope.scaling:
            out["rope_scaling"] = dict(self.rope.scaling)
        if self.eos_token_ids:
            out["eos_token_id"] = list(self.eos_token_ids)
        if self.quant.is_fp8:
            out["quantization_config"] = {"quant_method": "fp8", "modules_to_not_convert": list(self.quant.ignored_modules)}
            if self.quant.method == "fp8":
                out["quantization_config"]["weight_block_size"] = list(self.quant.block)
        a = self.architecture
        if a == "Qwen3MoeForCausalLM":
            out.update(num_experts=self.num_experts, num_experts_per_tok=self.num_experts_per_tok,
                       moe_intermediate_size=self.moe_intermediate_size, norm_topk_prob=self.norm_topk_prob)
        elif a == "MiniMaxM2ForCausalLM":
            out.update(use_qk_norm=self.qk_norm == "cross_head", num_local_experts=self.num_experts,
                       num_experts_per_tok=self.num_experts_per_tok, intermediate_size=self.moe_intermediate_size)
        elif a == "Glm4MoeForCausalLM":
            out.update(use_qk_norm=self.qk_norm == "head", n_routed_experts=self.num_experts,
                       num_experts_per_tok=self.num_experts_per_tok, moe_intermediate_size=self.moe_intermediate_size,
                       norm_topk_prob=self.norm_topk_prob, routed_scaling_factor=self.routed_scaling_factor,
                       n_group=self.n_group, topk_group=self.topk_group, n_shared_experts=self.num_shared_experts,
                       first_k_dense_replace=self.first_k_dense)
        elif a in ("Qwen3_5MoeForCausalLM", "Qwen3_5MoeForConditionalGeneration", "Qwen3NextForCausalLM"):
            out.update(num_experts=self.num_experts, num_experts_per_tok=self.num_experts_per_tok,
                       moe_intermediate_size=self.moe_intermediate_size, norm_topk_prob=self.norm_topk_prob,
                       shared_expert_intermediate_size=self.shared_expert_intermediate_size,
                       layer_types=["full_attention" if t == "full" else "linear_attention" for t in self.layer_types],
                       linear_num_key_heads=self.gdn_num_k_heads, linear_num_value_heads=self.gdn_num_v_heads,
                       linear_key_head_dim=self.gdn_head_k_dim, linear_value_head_dim=self.gdn_head_v_dim,
                       linear_conv_kernel_dim=self.gdn_conv_kernel)
        return out

    @staticmethod
    def from_path(path: str) -> "ModelConfig":
        """A checkpoint directory's ``config.json``; the stop tokens are those of ``config.json`` together with those
        of ``generation_config.json`` when the directory has one (chat models list their end-of-turn token there)."""
        cfg = ModelConfig.from_hf(json.loads((Path(path) / "config.json").read_text()))
        gen = Path(path) / "generation_config.json"
        if gen.exists():
            try:
                eos = json.loads(gen.read_text()).get("eos_token_id")
            except (OSError, ValueError):
                eos = None
            more = tuple(eos) if isinstance(eos, (list, tuple)) else ((eos,) if eos is not None else ())
            ids = tuple(dict.fromkeys(int(t) for t in cfg.eos_token_ids + more))
            cfg = replace(cfg, eos_token_ids=ids)
        return cfg


def _hybrid_types(n: int, interval: int = 4) -> Tuple[str, ...]:
    return tuple("full" if (i + 1) % interval == 0 else "linear" for i in range(n))


_FP8 = QuantConfig("fp8")

PRESETS: Dict[str, ModelConfig] = {
    # plumbing model for the CPU/gloo slice
    "tiny-qwen3-moe": ModelConfig(),
    "qwen3-30b-a3b": ModelConfig(
        num_layers=48, hidden_size=2048, num_q_heads=32, num_kv_heads=4, head_dim=128, vocab_size=151936,
        num_experts=128, num_experts_per_tok=8, moe_intermediate_size=768, eos_token_ids=(151645,)),
    "qwen3-235b-a22b-fp8": ModelConfig(
        num_layers=94, hidden_size=4096, num_q_heads=64, num_kv_heads=4, head_dim=128, vocab_size=151936,
        num_experts=128, num_experts_per_tok=8, moe_intermediate_size=1536, quant=_FP8, eos_token_ids=(151645,)),
    "minimax-m2.5-fp8": ModelConfig(
        architecture="MiniMaxM2ForCausalLM", num_layers=62, hidden_size=3072, num_q_heads=48, num_kv_heads=8,
        head_dim=128, vocab_size=200064, rope=RopeConfig(5e6, 64), qk_norm="cross_head", num_experts=256,
        num_experts_per_tok=8, moe_intermediate_size=1536, scoring="sigmoid", router_bias=True, router_fp32=True,
        quant=_FP8),
    "qwen3.5-397b-a17b-fp8": ModelConfig(
        architecture="Qwen3_5MoeForCausalLM", num_layers=60, hidden_size=4096, num_q_heads=32, num_kv_heads=2,
        head_dim=256, vocab_size=248320, rope=RopeConfig(1e7, 64), num_experts=512, num_experts_per_tok=10,
        moe_intermediate_size=1024, num_shared_experts=1, shared_expert_intermediate_size=1024,
        shared_expert_gate=True, layer_types=_hybrid_types(60), gdn_num_k_heads=16, gdn_num_v_heads=64,
        gdn_head_k_dim=128, gdn_head_v_dim=128, gdn_conv_kernel=4, attn_output_gate=True, norm_offset1=True,
        quant=_FP8),
    "glm-4.5-air": ModelConfig(
        architecture="Glm4MoeForCausalLM", num_layers=46, hidden_size=4096, num_q_heads=96, num_kv_heads=8,
        head_dim=128, vocab_size=151552, rope=RopeConfig(1e6, 64), qk_norm="none", attention_bias=True,
        intermediate_size=10944, num_experts=128, num_experts_per_tok=8, moe_intermediate_size=1408,
        scoring="sigmoid", router_bias=True, routed_scaling_factor=1.0, n_group=1, topk_group=1,
        num_shared_experts=1, shared_expert_intermediate_size=1408, first_k_dense=1),
}


def get_model_config(name_or_path: str) -> ModelConfig:
    if name_or_path in PRESETS:
        return PRESETS[name_or_path]
    p = Path(name_or_path)
    if (p / "config.json").exists():
        return ModelConfig.from_path(name_or_path)
    raise ValueError(f"unknown model '{name_or_path}': not a preset ({', '.join(PRESETS)}) nor a directory with config.json")


@dataclass
class RuntimeConfig:
    """Serving-time knobs shared by coordinator and workers (one typed object instead of
    the reference's ~130 environment variables; python/minisgl/ray_env_keys.py)."""
    model_path: str = "tiny-qwen3-moe"
    attn_dp: int = 1
    attn_tp: int = 1
    mlp_dp: int = 1
    mlp_tp: int = 1
    mlp_ep: int = 1
    num_mb: int = 2
    async_pending_steps: int = 3
    disable_overlap: bool = False
    page_size: int = 16
    num_pages: int = 0                      # 0 -> sized from free memory
    memory_ratio: float = 0.9
    max_running_requests: int = 256
    max_batched_tokens: int = 8192          # prefill token budget per lane per step
    max_seq_len: int = 0                    # 0 -> model max_position
    max_new_tokens: int = 1024
    decode_graph_bs: Tuple[int, ...] = ()   # explicit bucket list; () -> default ladder
    cuda_graph_max_bs: int = 256
    cache_type: str = "naive"               # naive | radix
    use_cuda_graph: bool = True
    moe_block_tok: int = 32
    flag_timeout_s: float = 20.0
    spec_block: int = 0                     # 0 = off; else verified tokens per step (drafts + 1)
    spec_draft_path: str = ""
    seed: int = 0
    dummy_weights: bool = False             # a checkpoint directory is served with random-init weights instead of its own
    dtype: str = "bfloat16"
    device: str = "cuda"
