"""Stage-structured transformer models for Attention-FFN disaggregation.

A model is split into two stages that live on different GPUs:

* :class:`AttentionStage` (attention GPU): embedding, per-layer attention block
  (input norm -> qkv projection -> q/k norm + RoPE + paged KV store -> paged attention ->
  o_proj), post-attention norm, router, optional local dense MLP / shared expert, final
  norm, LM head.
* :class:`ExpertStage` (expert GPU): the routed experts of every MoE layer for one
  expert-parallel rank.

The same classes run on CPU in fp32 (oracle, CPU/gloo slice) and on CUDA in bf16 where
every op below lands in the sm_100a kernel library (`fastafd_b200.ops`); dense
projections use cuBLAS through ``torch.nn.functional.linear``.

Families covered by configuration: Qwen3-MoE, MiniMax-M2 (sigmoid + bias routing,
cross-head q/k norm, partial rotary), GLM-4-MoE (first-k dense layers, shared experts,
routed scaling), Qwen3.5 hybrid (gated DeltaNet layers, gated full attention, shared
expert with sigmoid gate), and the dense Llama / Qwen2 / Qwen3 / Mistral models.

Stage API parity with the reference: python/minisgl/models/qwen3_moe_afd.py:201-228
(embed_input_ids / forward_attention / route / finalize_hidden / forward_lm_head) and
:280-290 (run_experts); families in python/minisgl/models/{minimax_m2,glm4_moe,qwen35_moe}_afd.py.
"""
from __future__ import annotations

import hashlib
import os
from dataclasses import dataclass
from typing import Dict, List, Optional, Tuple

import torch
import torch.nn.functional as F

from .. import ops
from ..config import ModelConfig
from ..reference import ops_ref as ref

Tensor = torch.Tensor


# ------------------------------------------------------------------ deterministic init
def seeded_normal(name: str, shape, std: float, seed: int, device, dtype, fast: bool = False) -> Tensor:
    """N(0, std) values that depend only on (seed, name): every process that creates the
    tensor `name` gets the same numbers. ``fast`` draws on the target CUDA device (large
    benchmark models); otherwise on CPU (tests compare across processes and devices)."""
    h = int.from_bytes(hashlib.sha256(f"{seed}:{name}".encode()).digest()[:7], "little")
    if fast and torch.device(device).type == "cuda":
        g = torch.Generator(device=device).manual_seed(h)
        return torch.empty(shape, dtype=torch.float32 if dtype == torch.float8_e4m3fn else dtype,
                           device=device).normal_(0.0, std, generator=g)
    g = torch.Generator(device="cpu").manual_seed(h)
    return (torch.randn(shape, generator=g, dtype=torch.float32) * std).to(dtype).to(device)


@dataclass
class AttnMeta:
    """Per-micro-batch attention inputs (device tensors with graph-stable addresses)."""
    positions: Tensor          # [T] int32
    out_loc: Tensor            # [T] int32 KV slot of each token (-1 = padding, no store)
    page_table: Tensor         # [B, max_pages] int32
    seq_lens: Tensor           # [B] int32, KV length including this step's tokens
    q_len: int = 1             # tokens per request in this step (decode 1, verify block)
    is_prefill: bool = False
    prefill_lens: Optional[List[int]] = None   # tokens of each request in this prefill step
    lane: int = -1                             # micro-batch lane (per-lane buffers of fused collectives)
    state_slots: Optional[Tensor] = None       # [B] int32 GDN state slot per request
    splits: int = 1
    workspace: Optional[Tensor] = None
    status: Optional[Tensor] = None


class KVPool:
    """bf16 (or fp32 on CPU) paged KV cache: [full_layers][slots, kv_heads, head_dim] x {K, V}.
    Reference: python/minisgl/kvcache/mha_pool.py:10-66."""

    def __init__(self, cfg: ModelConfig, num_pages: int, page_size: int, kv_heads: int, device, dtype):
        self.num_pages, self.page_size = num_pages, page_size
        n = cfg.num_full_attn_layers
        self.k = torch.zeros(n, num_pages * page_size, kv_heads, cfg.head_dim, dtype=dtype, device=device)
        self.v = torch.zeros_like(self.k)

    @staticmethod
    def bytes_per_page(cfg: ModelConfig, page_size: int, kv_heads: int, elem: int = 2) -> int:
        return 2 * cfg.num_full_attn_layers * page_size * kv_heads * cfg.head_dim * elem


class GDNStatePool:
    """Per-request recurrent state of the gated-DeltaNet layers: conv taps and the fp32
    [Hv, Dv, Dk] matrix. Reference: python/minisgl/kvcache/hybrid_pool.py:20-62."""

    def __init__(self, cfg: ModelConfig, slots: int, device, dtype, tp: int = 1):
        n = cfg.num_linear_layers
        hk, hv = cfg.gdn_num_k_heads // tp, cfg.gdn_num_v_heads // tp
        conv_dim = 2 * hk * cfg.gdn_head_k_dim + hv * cfg.gdn_head_v_dim
        self.conv = torch.zeros(n, slots, cfg.gdn_conv_kernel - 1, conv_dim, dtype=dtype, device=device)
        self.rec = torch.zeros(n, slots, hv, cfg.gdn_head_v_dim, cfg.gdn_head_k_dim, dtype=torch.float32, device=device)

    def reset(self, slot_ids: Tensor) -> None:
        self.conv[:, slot_ids.long()] = 0
        self.rec[:, slot_ids.long()] = 0


def _linear(x: Tensor, w: Tensor, b: Optional[Tensor] = None) -> Tensor:
    return F.linear(x, w, b)


# Dense projections (qkv, o_proj, GDN in/out projections, dense and shared-expert MLPs, LM head) are
# plain library GEMMs by default, on bf16 weights (a block-FP8 checkpoint's dense weights are
# dequantised once at load). Measured on B200 in CUDA-graph replay:
#   bf16, split-K tcgen05 kernel of this repository against the library: 64 x 5120 x 2048 qkv 10.1 / 6.8 us,
#   64 x 2048 x 4096 o_proj 11.3 / 8.4 us;
#   block-FP8 (activation quantisation + e4m3 kernel with exact 128x128 scales, half the weight bytes)
#   against the library on the bf16 copy: 44 x 9216 x 4096 29.0 / 16.9 us, 44 x 4096 x 8192 29.3 / 17.3 us,
#   88 x 9216 x 4096 41.7 / 17.6 us - the per-K-block promotion of the accumulator through registers costs
#   more than the halved weight stream saves.
# So both own paths are opt-in: FASTAFD_OWN_DENSE=1 (bf16 and FP8 weights), FASTAFD_OWN_DENSE=fp8 (FP8 only).
_OWN_DENSE_ENV = os.environ.get("FASTAFD_OWN_DENSE", "")
_OWN_DENSE = _OWN_DENSE_ENV == "1"
_OWN_DENSE_FP8 = _OWN_DENSE_ENV in ("1", "fp8")
_OWN_DENSE_MAX_TOKENS = 128


class AttentionStage:
    """Everything of the model that runs on an attention GPU. Tensor-parallel over `tp`
    ranks (heads split; o_proj row-parallel; vocab-parallel embedding and LM head); the
    all-reduce / all-gather is delegated to `comm` (None = single rank)."""

    def __init__(self, cfg: ModelConfig, device, dtype, tp_rank: int = 0, tp_size: int = 1, comm=None):
        self.cfg, self.device, self.dtype = cfg, torch.device(device), dtype
        self.tp_rank, self.tp_size, self.comm = tp_rank, tp_size, comm
        assert cfg.num_q_heads % tp_size == 0
        self.hq = cfg.num_q_heads // tp_size
        # GQA: kv heads are replicated when there are fewer of them than TP ranks
        self.hkv = max(1, cfg.num_kv_heads // tp_size)
        self.kv_rep = max(1, tp_size // cfg.num_kv_heads)
        self.w: Dict[str, Tensor] = {}
        self.full_index = {}   # layer -> index among full-attention layers
        self.lin_index = {}
        for i in range(cfg.num_layers):
            if cfg.layer_type(i) == "full":
                self.full_index[i] = len(self.full_index)
            else:
                self.lin_index[i] = len(self.lin_index)
        self.cos_sin: Optional[Tensor] = None
        self.status: Optional[Tensor] = None      # device status word of the process (set by the worker)
        self.cad = None                           # cad.gpu.CadModelHook: the attention core runs on other GPUs
        self.w_fp8: Dict[str, Tuple[Tensor, Tensor]] = {}
        self.w_merged: Dict[str, Tensor] = {}
        self.vocab_local = (cfg.vocab_size + tp_size - 1) // tp_size
        self.vocab_start = tp_rank * self.vocab_local

    # ------------------------------------------------------------------ weights
    def param_shapes(self) -> Dict[str, Tuple[Tuple[int, ...], str]]:
        """name -> (local shape, kind) where kind in {weight, norm, fp32}."""
        c, H, D = self.cfg, self.cfg.hidden_size, self.cfg.head_dim
        out: Dict[str, Tuple[Tuple[int, ...], str]] = {}
        vl = min(self.vocab_local, c.vocab_size - self.vocab_start)
        out["model.embed_tokens.weight"] = ((vl, H), "weight")
        out["model.norm.weight"] = ((H,), "norm")
        if not c.tie_embeddings:
            out["lm_head.weight"] = ((vl, H), "weight")
        for i in range(c.num_layers):
            p = f"model.layers.{i}."
            out[p + "input_layernorm.weight"] = ((H,), "norm")
            out[p + "post_attention_layernorm.weight"] = ((H,), "norm")
            if c.layer_type(i) == "full":
                qmul = 2 if c.attn_output_gate else 1
                out[p + "self_attn.qkv_proj.weight"] = (((self.hq * qmul + 2 * self.hkv) * D, H), "weight")
                if c.attention_bias:
                    out[p + "self_attn.qkv_proj.bias"] = (((self.hq * qmul + 2 * self.hkv) * D,), "weight")
                out[p + "self_attn.o_proj.weight"] = ((H, self.hq * D), "weight")
                if c.qk_norm == "head":
                    out[p + "self_attn.q_norm.weight"] = ((D,), "norm")
                    out[p + "self_attn.k_norm.weight"] = ((D,), "norm")
                elif c.qk_norm == "cross_head":
                    out[p + "self_attn.q_norm.weight"] = ((self.hq * D,), "norm")
                    out[p + "self_attn.k_norm.weight"] = ((self.hkv * D,), "norm")
            else:
                hk, hv = c.gdn_num_k_heads // self.tp_size, c.gdn_num_v_heads // self.tp_size
                dk, dv = c.gdn_head_k_dim, c.gdn_head_v_dim
                conv_dim = 2 * hk * dk + hv * dv
                out[p + "linear_attn.in_proj_qkv.weight"] = ((conv_dim, H), "weight")
                out[p + "linear_attn.in_proj_z.weight"] = ((hv * dv, H), "weight")
                out[p + "linear_attn.in_proj_b.weight"] = ((hv, H), "weight")
                out[p + "linear_attn.in_proj_a.weight"] = ((hv, H), "weight")
                out[p + "linear_attn.conv1d.weight"] = ((conv_dim, c.gdn_conv_kernel), "weight")
                out[p + "linear_attn.A_log"] = ((hv,), "fp32")
                out[p + "linear_attn.dt_bias"] = ((hv,), "fp32")
                out[p + "linear_attn.norm.weight"] = ((dv,), "norm")
                out[p + "linear_attn.out_proj.weight"] = ((H, hv * dv), "weight")
            if c.is_moe_layer(i):
                out[p + "mlp.gate.weight"] = ((c.num_experts, H), "fp32" if c.router_fp32 else "weight")
                if c.router_bias:
                    out[p + "mlp.gate.e_score_correction_bias"] = ((c.num_experts,), "fp32")
                if c.num_shared_experts > 0:
                    si = c.shared_expert_intermediate_size // self.tp_size
                    out[p + "mlp.shared_expert.gate_up_proj.weight"] = ((2 * si, H), "weight")
                    out[p + "mlp.shared_expert.down_proj.weight"] = ((H, si), "weight")
                    if c.shared_expert_gate:
                        out[p + "mlp.shared_expert_gate.weight"] = ((1, H), "weight")
            else:
                inter = c.intermediate_size // self.tp_size
                out[p + "mlp.gate_up_proj.weight"] = ((2 * inter, H), "weight")
                out[p + "mlp.down_proj.weight"] = ((H, inter), "weight")
        return out

    def init_random(self, seed: int = 0, std: float = 0.02, fast: bool = False) -> "AttentionStage":
        """Random-init weights. TP shards take their slice of the full tensor so that a TP run
        equals the single-rank run."""
        for name, (shape, kind) in self.param_shapes().items():
            dt = torch.float32 if kind == "fp32" else self.dtype
            if kind == "norm":
                base = torch.zeros(shape) if self.cfg.norm_offset1 else torch.ones(shape)
                self.w[name] = (base + seeded_normal(name, shape, 0.02, seed, "cpu", torch.float32)).to(dt).to(self.device)
            elif name.endswith("A_log"):
                self.w[name] = seeded_normal(name, shape, 0.5, seed, self.device, dt, fast)
            elif self.tp_size == 1:
                self.w[name] = seeded_normal(name, shape, std, seed, self.device, dt, fast)
            else:
                self.w[name] = self._tp_slice(name, seed, std, dt, fast)
        self._post_load()
        return self

    def _tp_slice(self, name: str, seed: int, std: float, dt, fast: bool = False) -> Tensor:
        """Slice of the full-size random tensor that this TP rank owns. With `fast` the full
        tensor is drawn on the target GPU (every rank of the lane draws the same numbers from the
        same seed) instead of on the host."""
        if not hasattr(self, "_full_shapes"):
            self._full_shapes = {k: v[0] for k, v in AttentionStage(self.cfg, "cpu", torch.float32).param_shapes().items()}
        full_shape = self._full_shapes[name]
        if fast and self.device.type == "cuda":
            full = seeded_normal(name, full_shape, std, seed, self.device, dt, True)
            return shard_attention_param(self.cfg, name, full, self.tp_rank, self.tp_size).clone()
        full = seeded_normal(name, full_shape, std, seed, "cpu", torch.float32)
        return shard_attention_param(self.cfg, name, full, self.tp_rank, self.tp_size).to(dt).to(self.device)

    def load_state(self, state: Dict[str, Tensor]) -> None:
        for name, (shape, kind) in self.param_shapes().items():
            t = state[name]
            assert tuple(t.shape) == tuple(shape), f"{name}: {tuple(t.shape)} != {shape}"
            self.w[name] = t.to(self.device, torch.float32 if kind == "fp32" else self.dtype)
        self._post_load()

    def _post_load(self) -> None:
        c, D = self.cfg, self.cfg.head_dim
        self.cos_sin = ref.build_cos_sin_cache(min(c.max_position, 1 << 17), c.rotary_dim, c.rope.theta, self.device,
                                              scaling=c.rope.scaling)
        # kernel-ready forms (CUDA): per-head norm weights with the +1 offset folded in once, and for
        # gated attention the projection rows re-ordered from [q | gate | k | v] to [q | k | v | gate],
        # so that q, k, v are a contiguous prefix of every output row (norm + RoPE + store and the
        # attention kernel read them in place) and the gate is a strided view behind them.
        self.qk_w: Dict[int, Tuple[Tensor, Tensor]] = {}
        self.gate_last = False
        for i in range(c.num_layers):
            if c.layer_type(i) != "full":
                continue
            p = f"model.layers.{i}.self_attn."
            if c.qk_norm == "head":
                qw, kw = self.w[p + "q_norm.weight"], self.w[p + "k_norm.weight"]
                self.qk_w[i] = (qw + 1, kw + 1) if c.norm_offset1 else (qw, kw)
            if c.attn_output_gate and self.device.type == "cuda":
                n = self.hq * D
                src = getattr(self, "_fp8_src", {})
                for suffix in ("qkv_proj.weight", "qkv_proj.bias"):
                    w = self.w.get(p + suffix)
                    if w is not None:
                        self.w[p + suffix] = torch.cat([w[:n], w[2 * n:], w[n:2 * n]], 0).contiguous()
                    if p + suffix in src:           # the checkpoint's FP8 values follow the same row order
                        t = src[p + suffix]
                        src[p + suffix] = torch.cat([t[:n], t[2 * n:], t[n:2 * n]], 0).contiguous()
                self.gate_last = True
        self._merge_gdn_in_proj()
        self._quantize_dense_weights()

    def _merge_gdn_in_proj(self) -> None:
        """Gated DeltaNet layers on CUDA: the four input projections become two GEMMs, [qkv | z] (the wide
        pair, FP8 where the checkpoint is) and [b | a] (Hv rows each); the single tensors stay as row
        views of the merged ones, so nothing is stored twice. The decode kernels read the column
        ranges of the merged outputs in place. Reference: python/minisgl/models/qwen35_moe.py:124-151
        (in_proj_qkvz / in_proj_ba)."""
        c = self.cfg
        self.w_merged: Dict[str, Tensor] = {}
        if self.device.type != "cuda":
            return
        src = getattr(self, "_fp8_src", {})
        for i in range(c.num_layers):
            if c.layer_type(i) == "full":
                continue
            p = f"model.layers.{i}.linear_attn."
            for merged, parts in (("in_proj_qkvz.weight", ("in_proj_qkv.weight", "in_proj_z.weight")),
                                  ("in_proj_ba.weight", ("in_proj_b.weight", "in_proj_a.weight"))):
                ws = [self.w.get(p + n) for n in parts]
                if any(w is None for w in ws) or len({w.dtype for w in ws}) != 1:
                    continue
                m = torch.cat(ws, 0).contiguous()
                self.w_merged[p + merged] = m
                off = 0
                for n, w in zip(parts, ws):
                    self.w[p + n] = m[off:off + w.shape[0]]
                    off += w.shape[0]
                if all(p + n in src for n in parts):
                    src[p + merged] = torch.cat([src[p + n] for n in parts], 0)

    def _quantize_dense_weights(self) -> None:
        """Block-FP8 checkpoints keep their dense projections in e4m3 with 128x128 scales on the GPU
        (half the bytes of the decode-time weight stream); the bf16 copies serve prefill-sized GEMMs."""
        c = self.cfg
        self.w_fp8: Dict[str, Tuple[Tensor, Tensor]] = {}
        if not (c.quant.is_fp8 and self.device.type == "cuda" and _OWN_DENSE_FP8):
            return
        for name, w in list(self.w.items()) + list(self.w_merged.items()):
            if not name.endswith(("qkv_proj.weight", "o_proj.weight", "in_proj_qkv.weight", "in_proj_z.weight",
                                  "in_proj_qkvz.weight", "out_proj.weight", "gate_up_proj.weight", "down_proj.weight")):
                continue
            if name.endswith(("in_proj_qkv.weight", "in_proj_z.weight")) and \
                    name.rsplit("in_proj_", 1)[0] + "in_proj_qkvz.weight" in self.w_merged:
                continue                     # served by the merged projection
            if w.dtype != torch.bfloat16 or w.shape[0] % 128 or w.shape[1] % 128 or not c.quant.applies_to(name):
                continue
            src = getattr(self, "_fp8_src", {}).get(name)         # the checkpoint's exact values, when it was FP8
            q, sc = ref.block_quant_fp8(src.to(self.device) if src is not None else w.float())
            self.w_fp8[name] = (q.contiguous(), ops.plain_tile_scales(sc[None].float()).contiguous())

    def _proj(self, x: Tensor, name: str, bias: Optional[Tensor] = None) -> Tensor:
        """x @ w[name].T (+ bias)."""
        w = self.w[name] if name in self.w else self.w_merged[name]
        q = self.w_fp8.get(name)
        if ((_OWN_DENSE or q is not None) and x.is_cuda and x.dtype == torch.bfloat16 and w.dtype == torch.bfloat16
                and x.dim() == 2 and 0 < x.shape[0] <= _OWN_DENSE_MAX_TOKENS and w.shape[0] % 128 == 0
                and w.shape[1] % 64 == 0 and x.is_contiguous()):
            if q is not None:
                xq, xs = ops.group_quant_fp8(x, 128)
                return ops.dense_gemm(xq, q[0], x_scale=xs, w_scale=q[1], bias=bias, status=self.status)
            return ops.dense_gemm(x, w, bias=bias, status=self.status)
        return F.linear(x, w, bias)

    # ------------------------------------------------------------------ forward pieces
    def embed(self, ids: Tensor, scatter: bool = False) -> Tensor:
        """Vocab-parallel gather. Under TP the partial rows are summed over the ranks: all-reduce
        (every rank gets all T rows) or, with `scatter`, reduce-scatter (rank r keeps rows
        [r*T/tp, (r+1)*T/tp): the token-sharded residual stream of the AFD pipeline)."""
        h = ops.embedding(ids, self.w["model.embed_tokens.weight"], self.vocab_start)
        if self.tp_size > 1:
            h = self.comm.reduce_scatter(h) if scatter else self.comm.all_reduce(h)
        return h

    def input_norm(self, layer: int, x: Tensor, residual: Optional[Tensor]) -> Tuple[Tensor, Tensor]:
        """Pre-attention norm. With `residual`, adds x into it first. Returns (normed, residual)."""
        w = self.w[f"model.layers.{layer}.input_layernorm.weight"]
        if residual is None:
            return ops.rmsnorm(x, w, self.cfg.rms_eps, self.cfg.norm_offset1), x
        return ops.add_rmsnorm(x, residual, w, self.cfg.rms_eps, self.cfg.norm_offset1), residual

    def attention(self, layer: int, x: Tensor, meta: AttnMeta, kv: KVPool, gdn: Optional[GDNStatePool] = None,
                  reduce: str = "all_reduce") -> Tensor:
        """x: normed hidden [T,H] -> attention block output after o_proj. Under TP the row-parallel
        o_proj leaves partial sums: `reduce` = all_reduce ([T,H] everywhere), scatter (rank r
        keeps its T/tp rows) or none."""
        if self.cfg.layer_type(layer) == "linear":
            out = self._linear_attention(layer, x, meta, gdn)
        else:
            out = self._full_attention(layer, x, meta, kv, fuse_scatter=(self.tp_size > 1 and reduce == "scatter"))
            if isinstance(out, tuple):          # o_proj already reduce-scattered by the fused path
                return out[0]
        if self.tp_size > 1 and reduce != "none":
            out = self.comm.reduce_scatter(out) if reduce == "scatter" else self.comm.all_reduce(out)
        return out

    def _full_attention(self, layer: int, x: Tensor, meta: AttnMeta, kv: KVPool, fuse_scatter: bool = False):
        c, D = self.cfg, self.cfg.head_dim
        p = f"model.layers.{layer}.self_attn."
        qkv = self._proj(x, p + "qkv_proj.weight", self.w.get(p + "qkv_proj.bias"))
        T = x.shape[0]
        gate = None
        nqkv = (self.hq + 2 * self.hkv) * D
        if c.attn_output_gate and self.gate_last:
            gate = qkv[:, nqkv:]                       # rows are [q | k | v | gate]: nothing is copied
        elif c.attn_output_gate:
            # rows are [q(hq*D) | gate(hq*D) | k | v]
            q_part, gate, kv_part = qkv[:, :self.hq * D], qkv[:, self.hq * D:2 * self.hq * D], qkv[:, 2 * self.hq * D:]
            qkv = torch.cat([q_part, kv_part], dim=-1).contiguous()
        li = self.full_index[layer]
        kc, vc = kv.k[li], kv.v[li]
        remote = self.cad is not None and not meta.is_prefill and qkv.is_cuda
        if remote:
            kc = vc = None            # core-attention disaggregation: K/V are stored by the attention GPUs
        qw, kw = self.qk_w.get(layer, (None, None))
        if c.qk_norm == "cross_head" and qkv.is_cuda:
            # one launch: joint RMSNorm over the q heads / k heads + RoPE + paged store
            qn, kn = self.hq * D, self.hkv * D
            sq = None
            if self.tp_size > 1:
                sq = self.comm.all_reduce(ops.qk_square_sums(qkv, qn, kn))
            ops.cross_head_norm_rope_store(qkv, self.w[p + "q_norm.weight"], self.w[p + "k_norm.weight"], self.cos_sin,
                                           meta.positions, meta.out_loc, kc, vc, self.hq, self.hkv, D, c.rotary_dim,
                                           c.rms_eps, c.num_q_heads * D, max(c.num_kv_heads, self.tp_size) * D,
                                           sq=sq, status=meta.status)
        else:
            if c.qk_norm == "cross_head":
                qkv = self._cross_head_norm(qkv, self.w[p + "q_norm.weight"], self.w[p + "k_norm.weight"])
            ops.qk_norm_rope_store(qkv, qw, kw, self.cos_sin, meta.positions, meta.out_loc, kc, vc, self.hq, self.hkv,
                                   D, c.rotary_dim, c.rms_eps, status=meta.status)
        q = qkv.view(T, -1, D)[:, :self.hq]
        scale = ref.softmax_scale(D)
        if remote:
            o = self.cad.attention(layer, meta.lane, qkv[:, :nqkv] if qkv.shape[1] != nqkv else qkv)
        elif meta.is_prefill:
            o = self._prefill_attention(q, kc, vc, meta, scale, kv.page_size)
        else:
            o = ops.decode_attention(q, kc, vc, meta.page_table, meta.seq_lens, self.hq, self.hkv, D,
                                     meta.q_len, kv.page_size, scale, splits=meta.splits,
                                     workspace=meta.workspace, status=meta.status)
        o = o.reshape(T, self.hq * D)
        if gate is not None:
            o = ops.sigmoid_gate_mul(o if o.is_contiguous() else o.contiguous(), gate)
        w_o = self.w[p + "o_proj.weight"]
        if (fuse_scatter and meta.lane >= 0 and o.is_cuda and o.dtype == torch.bfloat16
                and hasattr(self.comm, "oproj_reduce_scatter") and self.comm.can_fuse_oproj(T, o.shape[1])):
            # GEMM epilogue pushes the partial rows to their owners; returns this rank's summed rows
            return (self.comm.oproj_reduce_scatter(meta.lane, o.contiguous(), w_o),)
        return self._proj(o, p + "o_proj.weight")

    def _prefill_attention(self, q: Tensor, kc: Tensor, vc: Tensor, meta: AttnMeta, scale: float, page_size: int) -> Tensor:
        """Causal attention of each request's new chunk against its paged KV (which already holds
        the chunk: K/V were stored before this call). On CUDA all requests run in one var-len launch
        of the paged kernel's multi-token mode; on CPU the oracle, request by request."""
        D = self.cfg.head_dim
        lens = list(meta.prefill_lens)
        if q.is_cuda and lens and max(lens) > 0:
            # one launch over (request, query-row tile, kv head); rows past a request's chunk leave at once
            starts = torch.zeros(len(lens) + 1, dtype=torch.int32)
            starts[1:] = torch.tensor(lens, dtype=torch.int32).cumsum(0)
            return ops.prefill_attention_varlen(q, kc, vc, meta.page_table, meta.seq_lens, starts.to(q.device), max(lens),
                                                self.hq, self.hkv, D, page_size, scale, status=meta.status)
        out = torch.zeros_like(q)
        off = 0
        for b, n in enumerate(lens):
            if n == 0:
                continue
            qb = q[off:off + n].contiguous()
            ob = ops.decode_attention(qb, kc, vc, meta.page_table[b:b + 1], meta.seq_lens[b:b + 1], self.hq, self.hkv,
                                      D, n, page_size, scale, splits=1, status=meta.status)
            out[off:off + n] = ob
            off += n
        return out

    def _cross_head_norm(self, qkv: Tensor, qw: Tensor, kw: Tensor) -> Tensor:
        """MiniMax-M2: RMSNorm over all q heads jointly (and all k heads jointly). Under TP the
        sum of squares is all-reduced. Reference: python/minisgl/layers/norm.py:110-149."""
        c, D = self.cfg, self.cfg.head_dim
        qn, kn = self.hq * D, self.hkv * D
        q, k = qkv[:, :qn].float(), qkv[:, qn:qn + kn].float()
        sq = torch.stack([q.pow(2).sum(-1), k.pow(2).sum(-1)], dim=-1)
        if self.tp_size > 1:
            sq = self.comm.all_reduce(sq)
        qd, kd = c.num_q_heads * D, max(c.num_kv_heads, self.tp_size) * D
        q = q * torch.rsqrt(sq[:, 0:1] / qd + c.rms_eps) * qw.float()
        k = k * torch.rsqrt(sq[:, 1:2] / kd + c.rms_eps) * kw.float()
        out = qkv.clone()
        out[:, :qn] = q.to(qkv.dtype)
        out[:, qn:qn + kn] = k.to(qkv.dtype)
        return out

    def _linear_attention(self, layer: int, x: Tensor, meta: AttnMeta, gdn: GDNStatePool) -> Tensor:
        """Gated DeltaNet block: in-proj -> causal conv (k taps) + SiLU -> gated delta rule ->
        per-head gated RMSNorm -> out-proj. Reference: python/minisgl/models/qwen35_moe.py:58-247."""
        from ..ops import gdn as gdn_ops

        c = self.cfg
        p = f"model.layers.{layer}.linear_attn."
        li = self.lin_index[layer]
        hk, hv = c.gdn_num_k_heads // self.tp_size, c.gdn_num_v_heads // self.tp_size
        dk, dv = c.gdn_head_k_dim, c.gdn_head_v_dim
        if p + "in_proj_qkvz.weight" in self.w_merged and p + "in_proj_ba.weight" in self.w_merged:
            C = 2 * hk * dk + hv * dv
            qkvz = self._proj(x, p + "in_proj_qkvz.weight")
            ba = _linear(x, self.w_merged[p + "in_proj_ba.weight"])
            mixed, z, b, a = qkvz[:, :C], qkvz[:, C:], ba[:, :hv], ba[:, hv:]
        else:
            mixed = self._proj(x, p + "in_proj_qkv.weight")
            z = self._proj(x, p + "in_proj_z.weight")
            b = _linear(x, self.w[p + "in_proj_b.weight"])
            a = _linear(x, self.w[p + "in_proj_a.weight"])
        out = gdn_ops.gdn_block(mixed, z, a, b, self.w[p + "conv1d.weight"], self.w[p + "A_log"], self.w[p + "dt_bias"],
                                self.w[p + "norm.weight"], gdn.conv[li], gdn.rec[li], meta, hk, hv, dk, dv, c.rms_eps)
        return self._proj(out if out.is_contiguous() else out.contiguous(), p + "out_proj.weight")

    def post_attn_norm(self, layer: int, attn_out: Tensor, residual: Tensor, out: Optional[Tensor] = None) -> Tensor:
        w = self.w[f"model.layers.{layer}.post_attention_layernorm.weight"]
        return ops.add_rmsnorm(attn_out, residual, w, self.cfg.rms_eps, self.cfg.norm_offset1, out=out)

    def route(self, layer: int, x: Tensor, out_idx: Optional[Tensor] = None,
              out_w: Optional[Tensor] = None) -> Tuple[Tensor, Tensor]:
        """Router of MoE layer `layer` on normed hidden x: (topk_idx int32 [T,K], topk_w fp32 [T,K])."""
        c = self.cfg
        p = f"model.layers.{layer}.mlp.gate."
        gw = self.w[p + "weight"]
        logits = _linear(x.float() if gw.dtype == torch.float32 else x, gw)
        if not logits.is_cuda:
            logits = logits.float()
        bias = self.w.get(p + "e_score_correction_bias")
        if c.n_group > 1:
            return ops.grouped_topk_route(logits, bias, c.num_experts_per_tok, c.n_group, c.topk_group,
                                          c.norm_topk_prob, 1.0, out_idx=out_idx, out_w=out_w)
        return ops.topk_route(logits, bias, c.num_experts_per_tok, c.scoring, c.norm_topk_prob, 1.0,
                              out_idx=out_idx, out_w=out_w)

    def local_mlp(self, layer: int, x: Tensor, reduce: str = "all_reduce") -> Optional[Tensor]:
        """Work that stays on the attention GPU: the dense MLP of non-MoE layers, or the shared
        expert of an MoE layer (None when the layer has neither)."""
        c = self.cfg
        p = f"model.layers.{layer}.mlp."
        if not c.is_moe_layer(layer):
            h = ops.silu_mul(self._proj(x, p + "gate_up_proj.weight"))
            out = self._proj(h, p + "down_proj.weight")
        elif c.num_shared_experts > 0:
            h = ops.silu_mul(self._proj(x, p + "shared_expert.gate_up_proj.weight"))
            out = self._proj(h, p + "shared_expert.down_proj.weight")
            if c.shared_expert_gate:
                out = ops.shared_gate_mul(x, self.w[p + "shared_expert_gate.weight"], out)
        else:
            return None
        if self.tp_size > 1 and reduce != "none":
            out = self.comm.reduce_scatter(out) if reduce == "scatter" else self.comm.all_reduce(out)
        return out

    def final_norm(self, x: Tensor, residual: Tensor) -> Tensor:
        return ops.add_rmsnorm(x, residual, self.w["model.norm.weight"], self.cfg.rms_eps, self.cfg.norm_offset1)

    def lm_head(self, x: Tensor) -> Tensor:
        logits = self._proj(x, "model.embed_tokens.weight" if self.cfg.tie_embeddings else "lm_head.weight")
        if self.tp_size > 1:
            logits = self.comm.all_gather_last_dim(logits)[:, :self.cfg.vocab_size]
        return logits


def shard_attention_param(cfg: ModelConfig, name: str, full: Tensor, rank: int, tp: int) -> Tensor:
    """TP shard of an attention-stage tensor given at full size (merged-qkv aware, GQA
    replication when kv_heads < tp). Reference: python/minisgl/models/weight.py:142-185."""
    if tp == 1:
        return full
    D = cfg.head_dim
    hq = cfg.num_q_heads // tp
    hkv = max(1, cfg.num_kv_heads // tp)
    kv_rank = rank * cfg.num_kv_heads // tp if cfg.num_kv_heads < tp else rank

    def rows(t, n):  # even split of dim 0
        return t[rank * n:(rank + 1) * n]

    if name.endswith("qkv_proj.weight") or name.endswith("qkv_proj.bias"):
        qmul = 2 if cfg.attn_output_gate else 1
        qn = cfg.num_q_heads * D * qmul
        q, k, v = full[:qn], full[qn:qn + cfg.num_kv_heads * D], full[qn + cfg.num_kv_heads * D:]
        if qmul == 2:
            qq, gg = q[:qn // 2], q[qn // 2:]
            qs = torch.cat([rows(qq, hq * D), rows(gg, hq * D)], 0)
        else:
            qs = rows(q, hq * D)
        ks = k[kv_rank * hkv * D:(kv_rank + 1) * hkv * D]
        vs = v[kv_rank * hkv * D:(kv_rank + 1) * hkv * D]
        return torch.cat([qs, ks, vs], 0).contiguous()
    if name.endswith("o_proj.weight") or name.endswith("out_proj.weight") or name.endswith("down_proj.weight"):
        n = full.shape[1] // tp
        return full[:, rank * n:(rank + 1) * n].contiguous()
    if name.endswith("gate_up_proj.weight"):
        I = full.shape[0] // 2
        n = I // tp
        return torch.cat([full[rank * n:(rank + 1) * n], full[I + rank * n:I + (rank + 1) * n]], 0).contiguous()
    if name.endswith("embed_tokens.weight") or name.endswith("lm_head.weight"):
        vl = (cfg.vocab_size + tp - 1) // tp
        return full[rank * vl:(rank + 1) * vl].contiguous()
    if name.endswith("self_attn.q_norm.weight") and cfg.qk_norm == "cross_head":
        return rows(full, hq * D).contiguous()
    if name.endswith("self_attn.k_norm.weight") and cfg.qk_norm == "cross_head":
        return full[kv_rank * hkv * D:(kv_rank + 1) * hkv * D].contiguous()
    if ".linear_attn." in name:
        hk, hv = cfg.gdn_num_k_heads // tp, cfg.gdn_num_v_heads // tp
        dk, dv = cfg.gdn_head_k_dim, cfg.gdn_head_v_dim
        if name.endswith("in_proj_qkv.weight") or name.endswith("conv1d.weight"):
            kq = cfg.gdn_num_k_heads * dk
            q, k, v = full[:kq], full[kq:2 * kq], full[2 * kq:]
            return torch.cat([rows(q, hk * dk), rows(k, hk * dk), rows(v, hv * dv)], 0).contiguous()
        if name.endswith("in_proj_z.weight"):
            return rows(full, hv * dv).contiguous()
        if name.endswith(("in_proj_a.weight", "in_proj_b.weight", "A_log", "dt_bias")):
            return rows(full, hv).contiguous()
    return full


class ExpertStage:
    """The routed experts owned by expert-parallel rank `ep_rank` of `ep_size`, every MoE layer.

    Weights per layer: gate_up [E_local, 2I, H] (gate rows then up rows) and down
    [E_local, H, I]; experts beyond the global count on the last rank are zero padding.
    On CUDA the gate/up rows are re-laid out for the SWIGLU epilogue of the grouped GEMM, and
    with block-FP8 weights the scales are turned into per-tile scale tables."""

    def __init__(self, cfg: ModelConfig, device, dtype, ep_rank: int = 0, ep_size: int = 1,
                 tp_rank: int = 0, tp_size: int = 1):
        self.cfg, self.device, self.dtype = cfg, torch.device(device), dtype
        self.ep_rank, self.ep_size = ep_rank, ep_size
        # MLP tensor parallelism: every rank of the TP group holds all of its experts with 1/tp of
        # the intermediate dimension (gate / up rows and down columns) and returns partial rows
        # that the attention side sums (on GPUs: one combine slot per (TP rank, k), see
        # worker/moe_client.py:FabricMoeClient).
        self.tp_rank, self.tp_size = tp_rank, tp_size
        if tp_size > 1:
            unit = 128 if self.device.type == "cuda" else 1
            if cfg.moe_intermediate_size % (tp_size * unit) != 0:
                raise ValueError(f"moe_intermediate_size must be a multiple of {unit} x the MLP TP size")
        self.experts_local = (cfg.num_experts + ep_size - 1) // ep_size
        self.expert_base = ep_rank * self.experts_local
        self.moe_layers = [i for i in range(cfg.num_layers) if cfg.is_moe_layer(i)]
        self.gate_up: Dict[int, Tensor] = {}
        self.down: Dict[int, Tensor] = {}
        self.gate_up_scale: Dict[int, Tensor] = {}
        self.down_scale: Dict[int, Tensor] = {}
        # kernel-ready forms (CUDA)
        self.w13: Dict[int, Tensor] = {}
        self.w2: Dict[int, Tensor] = {}
        self.w13_scale: Dict[int, Optional[Tensor]] = {}
        self.w2_scale: Dict[int, Optional[Tensor]] = {}

    @property
    def fp8(self) -> bool:
        return self.cfg.quant.is_fp8 and self.device.type == "cuda"

    def init_random(self, seed: int = 0, std: float = 0.02, fast: bool = False) -> "ExpertStage":
        c, E = self.cfg, self.experts_local
        valid = max(0, min(E, c.num_experts - self.expert_base))
        for i in self.moe_layers:
            gu = torch.zeros(E, 2 * c.moe_intermediate_size, c.hidden_size, dtype=self.dtype, device=self.device)
            dn = torch.zeros(E, c.hidden_size, c.moe_intermediate_size, dtype=self.dtype, device=self.device)
            if fast and self.device.type == "cuda":
                name = f"model.layers.{i}.mlp.experts.rank{self.ep_rank}of{self.ep_size}"
                gu[:valid] = seeded_normal(name + ".gate_up", gu[:valid].shape, std, seed, self.device, self.dtype, True)
                dn[:valid] = seeded_normal(name + ".down", dn[:valid].shape, std, seed, self.device, self.dtype, True)
            else:
                for e in range(valid):
                    ge = self.expert_base + e
                    name = f"model.layers.{i}.mlp.experts.{ge}."
                    gu[e] = seeded_normal(name + "gate_up_proj.weight", gu[e].shape, std, seed, self.device, self.dtype)
                    dn[e] = seeded_normal(name + "down_proj.weight", dn[e].shape, std, seed, self.device, self.dtype)
            self.set_layer(i, gu, dn)
        return self

    def set_layer(self, layer: int, gate_up: Tensor, down: Tensor, gate_up_scale: Optional[Tensor] = None,
                  down_scale: Optional[Tensor] = None) -> None:
        """Install one layer's expert weights. bf16/fp32 tensors, or e4m3 tensors with their
        128x128 block scales ([E, 2I/128, H/128] and [E, H/128, I/128])."""
        c = self.cfg
        if self.device.type != "cuda":
            if gate_up.dtype == torch.float8_e4m3fn:
                gate_up = torch.stack([ref.block_dequant_fp8(gate_up[e], gate_up_scale[e]) for e in range(gate_up.shape[0])])
                down = torch.stack([ref.block_dequant_fp8(down[e], down_scale[e]) for e in range(down.shape[0])])
            if self.tp_size > 1:
                I = c.moe_intermediate_size
                lo, hi = self.tp_rank * (I // self.tp_size), (self.tp_rank + 1) * (I // self.tp_size)
                gate_up = torch.cat([gate_up[:, lo:hi], gate_up[:, I + lo:I + hi]], dim=1)
                down = down[:, :, lo:hi]
            self.gate_up[layer], self.down[layer] = gate_up.to(self.dtype).contiguous(), down.to(self.dtype).contiguous()
            return
        I = c.moe_intermediate_size
        if self.tp_size > 1:            # this rank's slice of the intermediate dimension (whole 128-blocks)
            lo, hi = self.tp_rank * (I // self.tp_size), (self.tp_rank + 1) * (I // self.tp_size)
            if gate_up_scale is not None:
                gate_up_scale = torch.cat([gate_up_scale[:, lo // 128:hi // 128], gate_up_scale[:, (I + lo) // 128:(I + hi) // 128]], dim=1)
                down_scale = down_scale[:, :, lo // 128:hi // 128]
            gate_up = torch.cat([gate_up[:, lo:hi], gate_up[:, I + lo:I + hi]], dim=1)
            down = down[:, :, lo:hi]
            I = hi - lo
        if c.quant.is_fp8:
            if gate_up.dtype != torch.float8_e4m3fn:
                gate_up, gate_up_scale = _block_quant_experts(gate_up)
                down, down_scale = _block_quant_experts(down)
            self.w13[layer] = ops.interleave_gate_up(gate_up.view(torch.uint8)).view(torch.float8_e4m3fn)
            self.w13_scale[layer] = ops.interleave_gate_up_scales(gate_up_scale.float(), I)
            self.w2[layer] = down.contiguous()
            self.w2_scale[layer] = ops.plain_tile_scales(down_scale.float())
        else:
            self.w13[layer] = ops.interleave_gate_up(gate_up.to(self.dtype))
            self.w2[layer] = down.to(self.dtype).contiguous()
            self.w13_scale[layer] = self.w2_scale[layer] = None

    def run_experts_dense(self, layer: int, x: Tensor, topk_idx: Tensor) -> Tensor:
        """CPU path: per-(k, token) expert output rows [K, T, H] for experts on this rank, zeros
        elsewhere (the combine buffer contents that the CUDA epilogue would write)."""
        K = topk_idx.shape[1]
        T, H = x.shape
        rows = torch.zeros(K, T, H, dtype=x.dtype, device=x.device)
        gu_all, dn_all = self.gate_up[layer], self.down[layer]
        for e in range(self.experts_local):
            sel = (topk_idx == e + self.expert_base)
            if not sel.any():
                continue
            tok, k = sel.nonzero(as_tuple=True)
            gu = _linear(x[tok], gu_all[e])
            h = ref.silu_mul(gu)
            rows[k, tok] = _linear(h, dn_all[e])
        return rows


def _block_quant_experts(w: Tensor):
    qs, ss = [], []
    for e in range(w.shape[0]):
        q, s = ref.block_quant_fp8(w[e])
        qs.append(q)
        ss.append(s)
    return torch.stack(qs), torch.stack(ss)


def combine_rows(rows: Tensor, topk_w: Tensor, topk_idx: Optional[Tensor] = None, scale: float = 1.0) -> Tensor:
    """y[t] = scale * sum_k w[t,k] * rows[k,t] in fp32, k ascending: the attention-side M2N
    reduction (same order as the CUDA combine kernel)."""
    K, T, H = rows.shape
    acc = torch.zeros(T, H, dtype=torch.float32, device=rows.device)
    for k in range(K):
        w = topk_w[:, k].float()
        if topk_idx is not None:
            w = torch.where(topk_idx[:, k] >= 0, w, torch.zeros_like(w))
        acc = torch.addcmul(acc, rows[k].float(), w[:, None])
    return (acc * scale).to(rows.dtype)
