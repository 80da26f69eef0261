"""EAGLE-3 style draft head: a one-layer Llama-like decoder that proposes `block - 1`
tokens per request from the target model's own hidden states.

* ``fc``: concatenation of the target's hidden states at three depths (low / middle / high
  layer) -> hidden size.
* one decoder layer whose attention input is ``concat(norm(embed(next token)), norm(feature))``
  (2H wide), followed by a SwiGLU MLP, a final norm and an LM head over a reduced draft
  vocabulary with a ``d2t`` map back to target token ids.
* draft position p holds K/V made from (token p+1, feature p); its output predicts token p+2.
* its own one-layer paged KV cache shares the target's page table (same slots).

Reference: python/minisgl/models/eagle3.py (fc over aux states, write_context :264-283,
propose chain :312-366, d2t map), python/minisgl/spec/attn_side.py:228-244,361-371.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, List, Optional, Tuple

import torch
import torch.nn.functional as F

from .. import ops
from ..config import ModelConfig
from ..models.transformer import AttnMeta, seeded_normal
from ..reference import ops_ref as ref


@dataclass(frozen=True)
class Eagle3Config:
    hidden_size: int
    num_q_heads: int
    num_kv_heads: int
    head_dim: int
    intermediate_size: int
    draft_vocab: int
    target_vocab: int
    target_layers: Tuple[int, int, int]
    rms_eps: float = 1e-6
    rope_theta: float = 1e6

    @staticmethod
    def for_target(cfg: ModelConfig, draft_vocab: int = 0) -> "Eagle3Config":
        L = cfg.num_layers
        layers = (min(2, L - 1), L // 2, max(L - 3, 0))
        return Eagle3Config(cfg.hidden_size, cfg.num_q_heads, cfg.num_kv_heads, cfg.head_dim,
                            max(cfg.moe_intermediate_size * 2, cfg.intermediate_size, 256),
                            draft_vocab or min(cfg.vocab_size, 32000), cfg.vocab_size, layers, cfg.rms_eps, cfg.rope.theta)


    @staticmethod
    def from_dir(path: str, target: ModelConfig) -> "Eagle3Config":
        """The draft head's own ``config.json`` (a one-layer Llama-style decoder): sizes, heads, draft vocabulary
        (``draft_vocab_size``, else the target's), rotary base, and the target layers whose outputs feed ``fc``
        (``eagle_config.eagle_aux_hidden_state_layer_ids``, read as layer outputs; default: layers 1, L/2 - 1 and
        L - 4; ``FASTAFD_SPEC_EAGLE3_LAYERS=a,b,c`` overrides). Variants this build does not run are refused.
        Reference: python/minisgl/models/eagle3.py:110-144."""
        import json
        import os

        raw = json.loads(open(os.path.join(path, "config.json")).read())
        if int(raw.get("num_hidden_layers", 1)) != 1:
            raise ValueError(f"EAGLE-3 draft with {raw.get('num_hidden_layers')} layers is not supported")
        eagle = raw.get("eagle_config") or {}
        if eagle.get("use_aux_hidden_state") is False:
            raise ValueError("EAGLE-3 draft without auxiliary hidden states is not supported")
        H = int(raw["hidden_size"])
        if H != target.hidden_size:
            raise ValueError(f"EAGLE-3 draft hidden size {H} != target hidden size {target.hidden_size}")
        scaling = raw.get("rope_scaling") or {}
        params = raw.get("rope_parameters") or {}
        kind = scaling.get("rope_type", scaling.get("type")) or params.get("rope_type")
        if kind not in (None, "default"):
            raise ValueError(f"EAGLE-3 draft rotary scaling {kind!r} is not supported")
        override = (os.environ.get("FASTAFD_SPEC_EAGLE3_LAYERS") or os.environ.get("MINISGL_AFD_SPEC_EAGLE3_LAYERS") or "").strip()
        ids = [int(x) for x in override.split(",")] if override else eagle.get("eagle_aux_hidden_state_layer_ids")
        L = target.num_layers
        if not ids:
            ids = [1, L // 2 - 1, L - 4]
        if len(ids) != 3 or not all(0 <= int(i) < L for i in ids):
            raise ValueError(f"EAGLE-3 auxiliary layers {ids} do not name three layers of a {L}-layer target")
        heads = int(raw["num_attention_heads"])
        return Eagle3Config(H, heads, int(raw.get("num_key_value_heads", heads)), int(raw.get("head_dim") or H // heads),
                            int(raw["intermediate_size"]), int(raw.get("draft_vocab_size") or raw.get("vocab_size") or target.vocab_size),
                            target.vocab_size, tuple(int(i) for i in ids), float(raw.get("rms_norm_eps", 1e-6)),
                            float(raw.get("rope_theta") or params.get("rope_theta") or 10000.0))


class Eagle3Draft:
    def __init__(self, cfg: Eagle3Config, device, dtype, num_slots: int):
        self.cfg, self.device, self.dtype = cfg, torch.device(device), dtype
        self.w: Dict[str, torch.Tensor] = {}
        self.k_cache = torch.zeros(num_slots, cfg.num_kv_heads, cfg.head_dim, dtype=dtype, device=device)
        self.v_cache = torch.zeros_like(self.k_cache)
        self.cos_sin = ref.build_cos_sin_cache(1 << 16, cfg.head_dim, cfg.rope_theta, device)
        self.d2t: Optional[torch.Tensor] = None

    def shapes(self) -> Dict[str, Tuple[int, ...]]:
        c = self.cfg
        H, D = c.hidden_size, c.head_dim
        return {
            "fc.weight": (H, 3 * H), "embed_tokens.weight": (c.target_vocab, H),
            "input_layernorm.weight": (H,), "hidden_norm.weight": (H,),
            "self_attn.qkv_proj.weight": ((c.num_q_heads + 2 * c.num_kv_heads) * D, 2 * H),
            "self_attn.o_proj.weight": (H, c.num_q_heads * D),
            "post_attention_layernorm.weight": (H,),
            "mlp.gate_up_proj.weight": (2 * c.intermediate_size, H), "mlp.down_proj.weight": (H, c.intermediate_size),
            "norm.weight": (H,), "lm_head.weight": (c.draft_vocab, H),
        }

    def init_random(self, seed: int = 0, share_embedding: Optional[torch.Tensor] = None) -> "Eagle3Draft":
        for name, shape in self.shapes().items():
            if name == "embed_tokens.weight" and share_embedding is not None:
                self.w[name] = share_embedding
            elif name.endswith("norm.weight") or name.endswith("layernorm.weight"):
                self.w[name] = torch.ones(shape, dtype=self.dtype, device=self.device)
            else:
                self.w[name] = seeded_normal("eagle3." + name, shape, 0.02, seed, self.device, self.dtype)
        c = self.cfg
        # draft id -> target id; identity on the first draft_vocab ids for synthetic heads
        self.d2t = torch.arange(c.draft_vocab, dtype=torch.int32, device=self.device)
        return self

    def load(self, path: str, share_embedding: Optional[torch.Tensor] = None,
             share_lm_head: Optional[torch.Tensor] = None) -> "Eagle3Draft":
        """Load a draft checkpoint (safetensors; q/k/v and gate/up stored separately or merged;
        ``d2t`` stored as offsets relative to the draft index, as published EAGLE-3 heads do). A head that
        ships no embedding uses the target's (`share_embedding`); one without its own LM head uses the target's
        (`share_lm_head`, full vocabulary, identity map)."""
        from safetensors.torch import load_file
        import glob
        import os

        raw: Dict[str, torch.Tensor] = {}
        for f in sorted(glob.glob(os.path.join(path, "*.safetensors"))):
            raw.update(load_file(f))
        raw = {k.replace("midlayer.", "").replace("model.", ""): v for k, v in raw.items()}
        if "self_attn.q_proj.weight" in raw:
            raw["self_attn.qkv_proj.weight"] = torch.cat([raw.pop(f"self_attn.{n}_proj.weight") for n in "qkv"], 0)
        if "mlp.gate_proj.weight" in raw:
            raw["mlp.gate_up_proj.weight"] = torch.cat([raw.pop("mlp.gate_proj.weight"), raw.pop("mlp.up_proj.weight")], 0)
        if "embed_tokens.weight" not in raw and share_embedding is not None:
            raw["embed_tokens.weight"] = share_embedding
        if "lm_head.weight" not in raw and share_lm_head is not None:
            if self.cfg.draft_vocab != share_lm_head.shape[0]:
                raise ValueError(f"draft without an LM head but draft vocabulary {self.cfg.draft_vocab} != target's {share_lm_head.shape[0]}")
            raw["lm_head.weight"] = share_lm_head
            raw.pop("d2t", None)
        for name, shape in self.shapes().items():
            if name not in raw:
                raise KeyError(f"draft checkpoint lacks {name}")
            if tuple(raw[name].shape) != tuple(shape):
                raise ValueError(f"{name}: {tuple(raw[name].shape)} != {shape}")
            self.w[name] = raw[name].to(self.device, self.dtype)
        if "d2t" in raw:
            off = raw["d2t"].to(torch.int64)
            if off.numel() != self.cfg.draft_vocab:
                raise ValueError(f"d2t has {off.numel()} entries, the draft LM head {self.cfg.draft_vocab} rows")
            self.d2t = (torch.arange(off.numel()) + off).to(torch.int32).to(self.device)
        else:
            self.d2t = torch.arange(self.cfg.draft_vocab, dtype=torch.int32, device=self.device)
        return self

    # ------------------------------------------------------------------ forward
    def fuse_features(self, aux: List[torch.Tensor]) -> torch.Tensor:
        """Three captured target hidden states [T,H] each -> draft feature [T,H]."""
        return F.linear(torch.cat(aux, dim=-1), self.w["fc.weight"])

    def layer(self, next_tokens: torch.Tensor, feature: torch.Tensor, meta: AttnMeta, page_size: int) -> torch.Tensor:
        """One pass of the draft layer over T positions: K/V are stored at meta.out_loc, the
        queries attend to the draft cache; returns the hidden output [T,H] (pre final norm)."""
        c, w = self.cfg, self.w
        D, Hq, Hkv = c.head_dim, c.num_q_heads, c.num_kv_heads
        e = ops.embedding(next_tokens, w["embed_tokens.weight"])
        x = torch.cat([ops.rmsnorm(e, w["input_layernorm.weight"], c.rms_eps),
                       ops.rmsnorm(feature, w["hidden_norm.weight"], c.rms_eps)], dim=-1)
        qkv = F.linear(x, w["self_attn.qkv_proj.weight"]).contiguous()
        ops.qk_norm_rope_store(qkv, None, None, self.cos_sin, meta.positions, meta.out_loc, self.k_cache, self.v_cache,
                               Hq, Hkv, D, D, c.rms_eps, status=meta.status)
        T = qkv.shape[0]
        q = qkv.view(T, Hq + 2 * Hkv, D)[:, :Hq]
        o = ops.decode_attention(q, self.k_cache, self.v_cache, meta.page_table, meta.seq_lens, Hq, Hkv, D, meta.q_len,
                                 page_size, ref.softmax_scale(D), splits=1, status=meta.status)
        h = feature + F.linear(o.reshape(T, Hq * D), w["self_attn.o_proj.weight"])
        m = ops.silu_mul(F.linear(ops.rmsnorm(h, w["post_attention_layernorm.weight"], c.rms_eps), w["mlp.gate_up_proj.weight"]))
        return h + F.linear(m, w["mlp.down_proj.weight"])

    def logits_to_tokens(self, h: torch.Tensor) -> torch.Tensor:
        logits = F.linear(ops.rmsnorm(h, self.w["norm.weight"], self.cfg.rms_eps), self.w["lm_head.weight"])
        return self.d2t[ops.argmax(logits).long()]
