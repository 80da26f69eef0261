"""Hugging Face safetensors checkpoint loading, split by serving role.

* streaming: tensors are read file by file with ``safe_open`` and placed straight into the
  stage that needs them; nothing else is kept.
* role split: an attention rank skips every routed-expert tensor, an expert rank skips
  everything else.
* merging: ``q_proj | k_proj | v_proj`` -> ``qkv_proj`` and ``gate_proj | up_proj`` ->
  ``gate_up_proj`` (each shard merged after tensor-parallel slicing, with GQA kv-head
  replication when there are fewer kv heads than TP ranks).
* expert parallelism: rank r owns experts [r*ceil(E/ep), (r+1)*ceil(E/ep)); missing experts
  on the last rank are zero padding. Per-expert tensors are stacked to [E_local, ...].
* block FP8: ``weight`` in e4m3 with ``weight_scale_inv`` per 128x128 block (scales always
  handled in fp32, even if stored in bf16). Expert weights stay FP8 with their exact block
  scales; dense attention-side projections are dequantised to the compute dtype at load
  (they run as plain library GEMMs). Static KV-cache scales in the checkpoint are ignored
  (the KV cache is bf16).

Reference: python/minisgl/models/weight.py (key normalisation :76-99, TP shard rules
:142-185, scale sharding :274-312, merges :24-41,585-594, expert stacking :394-402,596-620,
role split :506-513, dtype casting :123-139).
"""
from __future__ import annotations

import glob
import os
import re
from dataclasses import replace
from typing import Dict, Iterator, List, Optional, Tuple

import torch

from ..config import ModelConfig
from ..reference import ops_ref as ref
from .transformer import AttentionStage, ExpertStage, shard_attention_param

_EXPERT_RE = re.compile(r"\.(?:mlp|block_sparse_moe)\.experts\.(\d+)\.(gate_proj|up_proj|down_proj|w1|w2|w3)\.(weight|weight_scale_inv)$")
_EXPERT_ALIAS = {"w1": "gate_proj", "w3": "up_proj", "w2": "down_proj"}


_WRAPPER_RE = re.compile(r"^(?:model\.)?(?:language_model\.)+")


def normalize_key(name: str) -> Optional[str]:
    """Checkpoint key -> internal key, or None for tensors this build does not use."""
    if ".visual." in name or name.startswith("visual.") or "mtp." in name:
        return None
    # multimodal wrappers nest the text model: model.language_model.layers..., language_model.model.layers...
    m = _WRAPPER_RE.match(name)
    if m and m.group(0):
        rest = name[m.end():]
        name = rest if rest.startswith(("model.", "lm_head.")) else "model." + rest
    if name.endswith((".k_scale", ".v_scale", ".kv_scale", "rotary_emb.inv_freq")):
        return None
    name = name.replace(".block_sparse_moe.gate.", ".mlp.gate.")
    name = name.replace(".block_sparse_moe.e_score_correction_bias", ".mlp.gate.e_score_correction_bias")
    name = name.replace(".mlp.shared_experts.", ".mlp.shared_expert.")
    return name


def iter_checkpoint(path: str, want=None) -> Iterator[Tuple[str, torch.Tensor]]:
    """(key, tensor) of every tensor in the directory's safetensors files; with `want`, only
    keys for which it returns True are read from disk (an attention rank never touches the
    bytes of the routed experts and the other way round)."""
    from safetensors import safe_open

    files = sorted(glob.glob(os.path.join(path, "*.safetensors")))
    if not files:
        raise FileNotFoundError(f"no .safetensors files in {path}")
    for f in files:
        with safe_open(f, framework="pt", device="cpu") as sf:
            for k in sf.keys():
                if want is None or want(k):
                    yield k, sf.get_tensor(k)


_LAYER_RE = re.compile(r"(?:^|\.)layers\.(\d+)\.")


def _beyond_last_layer(key: str, num_layers: int) -> bool:
    """Checkpoints of models with next-token-prediction heads store those as extra decoder layers behind the last
    one (GLM-4.5: layer `num_hidden_layers`); they are not served and need not be read."""
    m = _LAYER_RE.search(key)
    return m is not None and int(m.group(1)) >= num_layers


def _dequant_if_fp8(w: torch.Tensor, scale: Optional[torch.Tensor]) -> torch.Tensor:
    if w.dtype == torch.float8_e4m3fn:
        if scale is None:
            raise ValueError("FP8 weight without weight_scale_inv")
        return ref.block_dequant_fp8(w, scale.float())
    return w


def split_q_gate_rows(t: torch.Tensor, heads: int, head_dim: int) -> torch.Tensor:
    """Gated attention (Qwen3.5): the checkpoint's q_proj has 2 x head_dim rows per head, the head's query rows
    and then its gate rows. Returns the rows as [query rows of all heads | gate rows of all heads].
    Reference: python/minisgl/models/qwen35_moe.py:299-303 (split_query_gate on the projection's output)."""
    per_head = t.reshape(heads, 2, head_dim, *t.shape[1:])
    return torch.cat([per_head[:, 0].reshape(heads * head_dim, *t.shape[1:]),
                      per_head[:, 1].reshape(heads * head_dim, *t.shape[1:])], 0).contiguous()


def split_qwen3_next_projections(cfg, raw: Dict[str, torch.Tensor]) -> None:
    """Qwen3-Next stores the gated-DeltaNet input projections as two matrices whose rows are grouped by key head:
    ``in_proj_qkvz`` = per key head [q (dk) | k (dk) | v of its value heads | z of its value heads] and
    ``in_proj_ba`` = per key head [b of its value heads | a of its value heads]. Qwen3.5 stores the four
    projections on their own (q of all heads, k of all heads, v; z; b; a). Rewrites the former into the latter,
    in place."""
    hk, hv, dk, dv = cfg.gdn_num_k_heads, cfg.gdn_num_v_heads, cfg.gdn_head_k_dim, cfg.gdn_head_v_dim
    per = hv // hk
    for key in [k for k in raw if k.endswith("linear_attn.in_proj_qkvz.weight")]:
        base = key[:-len("in_proj_qkvz.weight")]
        w = raw.pop(key)
        g = w.reshape(hk, 2 * dk + 2 * per * dv, w.shape[1])
        q, k_, v, z = g[:, :dk], g[:, dk:2 * dk], g[:, 2 * dk:2 * dk + per * dv], g[:, 2 * dk + per * dv:]
        raw[base + "in_proj_qkv.weight"] = torch.cat([q.reshape(hk * dk, -1), k_.reshape(hk * dk, -1), v.reshape(hv * dv, -1)], 0).contiguous()
        raw[base + "in_proj_z.weight"] = z.reshape(hv * dv, -1).contiguous()
        ba = raw.pop(base + "in_proj_ba.weight").reshape(hk, 2 * per, w.shape[1])
        raw[base + "in_proj_b.weight"] = ba[:, :per].reshape(hv, -1).contiguous()
        raw[base + "in_proj_a.weight"] = ba[:, per:].reshape(hv, -1).contiguous()


def merge_q_gate_rows(t: torch.Tensor, heads: int, head_dim: int) -> torch.Tensor:
    """Inverse of `split_q_gate_rows`: [queries | gates] back to the checkpoint's per-head [q | gate] rows."""
    q, g = t[:heads * head_dim], t[heads * head_dim:]
    both = torch.stack([q.reshape(heads, head_dim, *t.shape[1:]), g.reshape(heads, head_dim, *t.shape[1:])], 1)
    return both.reshape(2 * heads * head_dim, *t.shape[1:]).contiguous()


def load_attention_stage(stage: AttentionStage, path: str) -> None:
    """Fill an AttentionStage from a checkpoint directory (TP-sharded, merged, role-filtered)."""
    cfg = stage.cfg
    need = stage.param_shapes()
    raw: Dict[str, torch.Tensor] = {}
    scales: Dict[str, torch.Tensor] = {}
    def wanted(key: str) -> bool:                     # skip_expert_weights
        k = normalize_key(key)
        return k is not None and not _EXPERT_RE.search(k) and not _beyond_last_layer(k, cfg.num_layers)

    for key, t in iter_checkpoint(path, wanted):
        k = normalize_key(key)
        if k.endswith(".weight_scale_inv"):
            scales[k[:-len("_scale_inv")]] = t
        else:
            raw[k] = t
    for k in list(raw):
        # a depthwise Conv1d stores its taps as [channels, 1, kernel]; the stage keeps [channels, kernel]
        if k.endswith("linear_attn.conv1d.weight") and raw[k].dim() == 3 and raw[k].shape[1] == 1:
            raw[k] = raw[k].squeeze(1)
    was_fp8 = set()
    for k in list(raw):
        if k in scales or raw[k].dtype == torch.float8_e4m3fn:
            raw[k] = _dequant_if_fp8(raw[k], scales.get(k))       # exact in fp32: code x block scale
            was_fp8.add(k)
    if cfg.num_linear_layers:                   # after the dequantisation: the values are exact in fp32, rows can move
        for k in [k for k in raw if k.endswith(("in_proj_qkvz.weight", "in_proj_ba.weight")) and k in was_fp8]:
            base = k.rsplit("in_proj_", 1)[0]
            was_fp8.update(base + n for n in (("in_proj_qkv.weight", "in_proj_z.weight") if k.endswith("qkvz.weight")
                                              else ("in_proj_b.weight", "in_proj_a.weight")))
        split_qwen3_next_projections(cfg, raw)
    full: Dict[str, torch.Tensor] = {}
    for i in range(cfg.num_layers):
        p = f"model.layers.{i}."
        a = p + "self_attn."
        if a + "q_proj.weight" in raw:
            if cfg.attn_output_gate:          # checkpoint rows: per head [q | gate]; the stage keeps [q of all heads | gates]
                for suf in (".weight", ".bias"):
                    if a + "q_proj" + suf in raw:
                        raw[a + "q_proj" + suf] = split_q_gate_rows(raw[a + "q_proj" + suf], cfg.num_q_heads, cfg.head_dim)
            if a + "q_proj.weight" in was_fp8:
                was_fp8.add(a + "qkv_proj.weight")
            full[a + "qkv_proj.weight"] = torch.cat([raw.pop(a + n + ".weight") for n in ("q_proj", "k_proj", "v_proj")], 0)
            if a + "q_proj.bias" in raw:
                full[a + "qkv_proj.bias"] = torch.cat([raw.pop(a + n + ".bias") for n in ("q_proj", "k_proj", "v_proj")], 0)
        for m in (p + "mlp.", p + "mlp.shared_expert."):
            if m + "gate_proj.weight" in raw:
                if m + "gate_proj.weight" in was_fp8:
                    was_fp8.add(m + "gate_up_proj.weight")
                full[m + "gate_up_proj.weight"] = torch.cat([raw.pop(m + "gate_proj.weight"), raw.pop(m + "up_proj.weight")], 0)
    full.update(raw)
    if cfg.tie_embeddings:
        full.pop("lm_head.weight", None)
    state = {}
    fp8_src = {}
    for name, (shape, kind) in need.items():
        if name not in full:
            raise KeyError(f"checkpoint lacks {name}")
        t = shard_attention_param(cfg, name, full[name], stage.tp_rank, stage.tp_size)
        if tuple(t.shape) != tuple(shape):
            raise ValueError(f"{name}: checkpoint shape {tuple(t.shape)} != expected {shape}")
        state[name] = t
        if name in was_fp8:
            # The dense projection was block-FP8 in the checkpoint. Its fp32 values (code x scale) go to the
            # stage beside the bf16 copy: re-quantising a 128x128-aligned shard of them gives back the
            # checkpoint's codes and scales (the block maximum is +-448 x scale by construction), so the
            # GPU keeps the checkpoint's own e4m3 weights instead of a bf16 rounding of them.
            fp8_src[name] = t.float()
    stage._fp8_src = fp8_src
    stage.load_state(state)
    stage._fp8_src = {}


def load_expert_stage(stage: ExpertStage, path: str) -> None:
    """Fill an ExpertStage: only routed-expert tensors of this rank's expert range are read."""
    cfg, E = stage.cfg, stage.experts_local
    lo, hi = stage.expert_base, min(stage.expert_base + E, cfg.num_experts)
    I, H = cfg.moe_intermediate_size, cfg.hidden_size
    parts: Dict[int, Dict[Tuple[int, str, str], torch.Tensor]] = {}
    def wanted(key: str) -> bool:                     # skip_non_expert_weights, other ranks' experts
        k = normalize_key(key)
        m = _EXPERT_RE.search(k) if k is not None else None
        return m is not None and lo <= int(m.group(1)) < hi and not _beyond_last_layer(k, cfg.num_layers)

    for key, t in iter_checkpoint(path, wanted):
        k = normalize_key(key)
        m = _EXPERT_RE.search(k)
        e = int(m.group(1))
        layer = int(re.search(r"layers\.(\d+)\.", k).group(1))
        proj = _EXPERT_ALIAS.get(m.group(2), m.group(2))
        parts.setdefault(layer, {})[(e - lo, proj, m.group(3))] = t
    for layer in stage.moe_layers:
        got = parts.get(layer, {})
        fp8 = any(t.dtype == torch.float8_e4m3fn for t in got.values())
        wdt = torch.float8_e4m3fn if fp8 else stage.dtype
        gu = torch.zeros(E, 2 * I, H, dtype=wdt)
        dn = torch.zeros(E, H, I, dtype=wdt)
        gus = torch.ones(E, (2 * I + 127) // 128, (H + 127) // 128, dtype=torch.float32) if fp8 else None
        dns = torch.ones(E, (H + 127) // 128, (I + 127) // 128, dtype=torch.float32) if fp8 else None
        for e in range(hi - lo):
            try:
                gu[e, :I], gu[e, I:], dn[e] = got[(e, "gate_proj", "weight")], got[(e, "up_proj", "weight")], got[(e, "down_proj", "weight")]
            except KeyError as err:
                raise KeyError(f"checkpoint lacks expert {lo + e} of layer {layer}: {err}") from None
            if fp8:
                if I % 128:
                    # gate rows and up rows are merged into one matrix; with an intermediate size that is not a
                    # multiple of the 128-row scale block, the last gate rows and the first up rows would share a block
                    raise ValueError(f"block-FP8 experts need moe_intermediate_size to be a multiple of 128, got {I}")
                gb = (I + 127) // 128
                gus[e, :gb] = got[(e, "gate_proj", "weight_scale_inv")].float()
                gus[e, gb:] = got[(e, "up_proj", "weight_scale_inv")].float()
                dns[e] = got[(e, "down_proj", "weight_scale_inv")].float()
        dev = stage.device
        stage.set_layer(layer, gu.to(dev), dn.to(dev), None if gus is None else gus.to(dev), None if dns is None else dns.to(dev))


def save_checkpoint(cfg: ModelConfig, attn: AttentionStage, experts: List[ExpertStage], path: str,
                    fp8_experts: bool = False, shard_mb: int = 64) -> None:
    """Write single-rank stages as a Hugging Face style checkpoint (separate q/k/v and gate/up
    tensors, per-expert tensors, optional block-FP8 experts). Used to build synthetic
    checkpoints for tests and for offline conversion."""
    import json

    from safetensors.torch import save_file

    os.makedirs(path, exist_ok=True)
    with open(os.path.join(path, "config.json"), "w") as f:
        from ..config import QuantConfig

        json.dump((replace(cfg, quant=QuantConfig("fp8")) if fp8_experts and not cfg.quant.is_fp8 else cfg).to_hf(), f)
    out: Dict[str, torch.Tensor] = {}
    D = cfg.head_dim
    for name, t in attn.w.items():
        t = t.detach().cpu()
        if name.endswith("qkv_proj.weight") or name.endswith("qkv_proj.bias"):
            qn = cfg.num_q_heads * D * (2 if cfg.attn_output_gate else 1)
            kn = cfg.num_kv_heads * D
            base, suf = name.rsplit("qkv_proj", 1)
            out[base + "q_proj" + suf], out[base + "k_proj" + suf], out[base + "v_proj" + suf] = \
                t[:qn].contiguous(), t[qn:qn + kn].contiguous(), t[qn + kn:].contiguous()
            if cfg.attn_output_gate:          # the checkpoint format keeps each head's query and gate rows together
                out[base + "q_proj" + suf] = merge_q_gate_rows(out[base + "q_proj" + suf], cfg.num_q_heads, D)
        elif name.endswith("gate_up_proj.weight"):
            half = t.shape[0] // 2
            base = name[:-len("gate_up_proj.weight")]
            out[base + "gate_proj.weight"], out[base + "up_proj.weight"] = t[:half].contiguous(), t[half:].contiguous()
        else:
            out[name] = t.contiguous()
    I = cfg.moe_intermediate_size
    for st in experts:
        for layer in st.moe_layers:
            gu, dn = st.gate_up[layer].cpu(), st.down[layer].cpu()
            for e in range(min(st.experts_local, cfg.num_experts - st.expert_base)):
                p = f"model.layers.{layer}.mlp.experts.{st.expert_base + e}."
                for pname, w in (("gate_proj", gu[e, :I]), ("up_proj", gu[e, I:]), ("down_proj", dn[e])):
                    if fp8_experts:
                        q, s = ref.block_quant_fp8(w.float())
                        out[p + pname + ".weight"], out[p + pname + ".weight_scale_inv"] = q.contiguous(), s.contiguous()
                    else:
                        out[p + pname + ".weight"] = w.contiguous()
    shard, size, idx = {}, 0, 0
    for k in sorted(out):
        shard[k] = out[k]
        size += out[k].numel() * out[k].element_size()
        if size > shard_mb << 20:
            save_file(shard, os.path.join(path, f"model-{idx:05d}.safetensors"))
            shard, size, idx = {}, 0, idx + 1
    if shard:
        save_file(shard, os.path.join(path, f"model-{idx:05d}.safetensors"))
