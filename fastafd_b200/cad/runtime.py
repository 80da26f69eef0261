"""CAD decode step over a shared window.

Transport = one *window* per attention GPU: slots for the q|k|v rows a model GPU puts there,
slots in the model GPU's window for the attention output rows, epoch-stamped flags, and one
``err`` word. Every wait is bounded; a wait that runs out sets ``err``; later waits see it and
return at once; the step ends as :class:`CadStepAborted` and the worker keeps serving.

``CadWindow.local`` takes caller-owned buffers, so several "ranks" can be plain objects that
share tensors in one process: that is how the protocol is exercised on CPU (the reference's
design for tests, python/minisgl/cad/window.py:63-68). The tasks of the model side and the
attention side run under a cooperative scheduler that advances whichever side's next task has
its flags satisfied, so flag order, epochs and time-outs behave as between real GPUs.

Reference: python/minisgl/cad/{layout,window,model_side,attn_side,runtime}.py,
python/minisgl/kernel/cad_hop.py:42-204 (wait / copy / flag / epoch semantics).
"""
from __future__ import annotations

import time
from dataclasses import dataclass
from typing import List, Optional, Tuple

import torch
import torch.nn.functional as F

from .. import ops
from ..config import ModelConfig
from ..models.transformer import AttentionStage, ExpertStage, combine_rows
from ..reference import ops_ref as ref
from .config import CadConfig
from .program import attention_program, check_balanced, model_program


class CadStepAborted(RuntimeError):
    """A wait timed out (or found the window's err word set); the step's result is discarded."""


@dataclass
class CadLayout:
    """Sizes of one window. Rows are segment-major: all q rows, then all k rows, then all v rows."""
    num_layers: int
    num_mb: int
    max_tokens: int
    q_size: int
    kv_size: int

    @property
    def qkv_row(self) -> int:
        return self.q_size + 2 * self.kv_size


class CadWindow:
    """Buffers + flags of one attention rank (qkv in) and its slice of the model rank (o out)."""

    def __init__(self, layout: CadLayout, qkv: torch.Tensor, o: torch.Tensor, flags: torch.Tensor, err: torch.Tensor):
        self.layout, self.qkv, self.o, self.flags, self.err = layout, qkv, o, flags, err
        self.epoch = 0

    @staticmethod
    def local(layout: CadLayout, dtype=torch.float32, device="cpu") -> "CadWindow":
        L = layout
        return CadWindow(L, torch.zeros(L.num_mb, L.max_tokens, L.qkv_row, dtype=dtype, device=device),
                         torch.zeros(L.num_mb, L.max_tokens, L.q_size, dtype=dtype, device=device),
                         torch.zeros(2, L.num_layers, L.num_mb, dtype=torch.int64, device=device),
                         torch.zeros(1, dtype=torch.int64, device=device))

    # flags[0] = qkv ready, flags[1] = o ready; value epoch + 1 marks "released in this step"
    def release(self, kind: int, layer: int, mb: int) -> None:
        self.flags[kind, layer, mb] = self.epoch + 1

    def ready(self, kind: int, layer: int, mb: int) -> bool:
        return int(self.flags[kind, layer, mb]) == self.epoch + 1

    def begin_step(self, bucket: int) -> None:
        """Rows per peer and micro-batch of the step that starts (a transport that moves rows needs the size)."""
        self.bucket = bucket

    def end_step(self) -> None:
        """Called by each side after its last task of a step."""

    def set_err(self, code: int = 1) -> None:
        self.err[0] = code

    def bump_epoch(self) -> None:
        self.epoch += 1


@dataclass
class _MbState:
    ids: torch.Tensor
    positions: torch.Tensor
    owner: torch.Tensor            # attention rank owning each request
    residual: Optional[torch.Tensor] = None
    normed: Optional[torch.Tensor] = None
    qkv: Optional[torch.Tensor] = None
    logits: Optional[torch.Tensor] = None


class CadAttentionRank:
    """KV cache + decode attention for the requests it owns."""

    def __init__(self, cfg: ModelConfig, window: CadWindow, num_slots: int, dtype, device):
        self.cfg, self.win = cfg, window
        n = cfg.num_full_attn_layers
        self.k = torch.zeros(n, num_slots, cfg.num_kv_heads, cfg.head_dim, dtype=dtype, device=device)
        self.v = torch.zeros_like(self.k)

    def attn(self, layer: int, mb: int, sel: torch.Tensor, slots: torch.Tensor, page_table: torch.Tensor,
             seq_lens: torch.Tensor, page_size: int) -> None:
        c = self.cfg
        D, Hq, Hkv = c.head_dim, c.num_q_heads, c.num_kv_heads
        rows = self.win.qkv[mb][:sel.shape[0]][sel]
        q = rows[:, :Hq * D].reshape(-1, Hq, D)
        k = rows[:, Hq * D:(Hq + Hkv) * D].reshape(-1, Hkv, D)
        v = rows[:, (Hq + Hkv) * D:].reshape(-1, Hkv, D)
        self.k[layer][slots.long()] = k.to(self.k.dtype)
        self.v[layer][slots.long()] = v.to(self.v.dtype)
        o = ops.decode_attention(q.contiguous(), self.k[layer], self.v[layer], page_table, seq_lens, Hq, Hkv, D, 1,
                                 page_size, ref.softmax_scale(D))
        self.win.o[mb][:sel.shape[0]][sel] = o.reshape(-1, Hq * D).to(self.win.o.dtype)   # straight into the model rank's window


class CadModelMath:
    """Model-side layer math of a CAD decode step over `self.windows` (one per peer): a micro-batch's row `k`
    belongs to peer `st.owner[k]` and travels at index `k` of that peer's window. Needs `self.cfg`,
    `self.stage` (AttentionStage), `self.experts` (ExpertStage) and `self.windows`."""

    def embed_mb(self, ids: torch.Tensor, positions: torch.Tensor, owner: torch.Tensor) -> "_MbState":
        c, m = self.cfg, self.stage
        h = m.embed(ids)
        st = _MbState(ids, positions, owner, residual=h.clone())
        st.normed = ops.rmsnorm(h, m.w["model.layers.0.input_layernorm.weight"], c.rms_eps, c.norm_offset1)
        return st

    def sample_mb(self, st: "_MbState") -> torch.Tensor:
        st.logits = self.stage.lm_head(st.normed)
        return ops.argmax(st.logits)

    def _hqkv(self, layer: int, mb: int, st: _MbState, slots, page_table, seq_lens) -> None:
        c, m = self.cfg, self.stage
        p = f"model.layers.{layer}.self_attn."
        qkv = F.linear(st.normed, m.w[p + "qkv_proj.weight"], m.w.get(p + "qkv_proj.bias"))
        qw = kw = None
        if c.qk_norm == "head":
            qw, kw = m.w[p + "q_norm.weight"], m.w[p + "k_norm.weight"]
        elif c.qk_norm == "cross_head":
            qkv = m._cross_head_norm(qkv, m.w[p + "q_norm.weight"], m.w[p + "k_norm.weight"])
        ops.qk_norm_rope_store(qkv, qw, kw, m.cos_sin, st.positions, None, None, None, c.num_q_heads, c.num_kv_heads,
                               c.head_dim, c.rotary_dim, c.rms_eps)
        for a, w in enumerate(self.windows):                    # put rows + release flag = epoch + 1
            sel = st.owner == a
            w.qkv[mb][:sel.shape[0]][sel] = qkv[sel].to(w.qkv.dtype)
            w.release(0, layer, mb)

    def _hpost_ffn(self, layer: int, mb: int, st: _MbState) -> None:
        c, m = self.cfg, self.stage
        o = torch.zeros(st.ids.shape[0], c.q_size, dtype=st.residual.dtype, device=st.residual.device)
        for a, w in enumerate(self.windows):
            sel = st.owner == a
            o[sel] = w.o[mb][:sel.shape[0]][sel].to(o.dtype)
        attn_out = F.linear(o, m.w[f"model.layers.{layer}.self_attn.o_proj.weight"])
        x = m.post_attn_norm(layer, attn_out, st.residual)
        if c.is_moe_layer(layer):
            idx, wts = m.route(layer, x)
            y = combine_rows(self.expert_rows(layer, x, idx), wts, idx, c.routed_scaling_factor)
            extra = m.local_mlp(layer, x)
            if extra is not None:
                y = (y.float() + extra.float()).to(y.dtype)
        else:
            y = m.local_mlp(layer, x)
        nw = (m.w[f"model.layers.{layer + 1}.input_layernorm.weight"] if layer + 1 < c.num_layers else m.w["model.norm.weight"])
        st.normed = ops.add_rmsnorm(y, st.residual, nw, c.rms_eps, c.norm_offset1)

    def expert_rows(self, layer: int, x: torch.Tensor, idx: torch.Tensor) -> torch.Tensor:
        """Expert outputs [K, T, H] of the routed rows. Here: every expert is local; a model rank that holds a
        slice of the experts overrides this with the exchange among the model ranks."""
        return self.experts.run_experts_dense(layer, x, idx)


class CadRuntime(CadModelMath):
    """One model rank with `r` attention ranks, experts local to the model rank."""

    def __init__(self, cfg: ModelConfig, stage: AttentionStage, experts: ExpertStage, ccfg: CadConfig, *, num_mb: int,
                 max_tokens: int, page_size: int, num_pages: int, wait_timeout_s: float = 5.0):
        if any(cfg.layer_type(i) != "full" for i in range(cfg.num_layers)):
            raise ValueError("CAD serves full-attention layers only")
        self.cfg, self.stage, self.experts, self.ccfg = cfg, stage, experts, ccfg
        self.num_mb, self.page_size, self.wait_timeout_s = num_mb, page_size, wait_timeout_s
        self.r = ccfg.attn_per_model
        check_balanced(cfg.num_layers, num_mb, self.r)
        lay = CadLayout(cfg.num_layers, num_mb, max_tokens, cfg.q_size, cfg.kv_size)
        dt, dev = stage.dtype, stage.device
        self.windows = [CadWindow.local(lay, dt, dev) for _ in range(self.r)]
        self.attn = [CadAttentionRank(cfg, w, num_pages * page_size, dt, dev) for w in self.windows]

    # ------------------------------------------------------------------ one decode step
    def decode_step(self, mbs: List[Tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]],
                    drop: Optional[Tuple[str, int, int]] = None) -> List[torch.Tensor]:
        """mbs[m] = (ids [B], positions [B], page_table [B,P], owner [B]). Returns next tokens per
        micro-batch. `drop` = (kind, layer, mb) names a flag release to withhold (host-side fault
        injection: the peer's wait must time out and the step must abort cleanly)."""
        c, m = self.cfg, self.stage
        if any(int(w.err[0]) for w in self.windows):
            raise CadStepAborted("window err word is set; reset it before serving again")
        L, nmb = c.num_layers, self.num_mb
        states = []
        for ids, pos, pt, owner in mbs:
            states.append(self.embed_mb(ids, pos, owner))
        ps = self.page_size
        seq_lens = [pos + 1 for _, pos, _, _ in mbs]
        slots = [torch.gather(pt, 1, (pos // ps).long()[:, None])[:, 0] * ps + pos % ps for _, pos, pt, _ in mbs]
        model_prog = [t for t in model_program(L, nmb) if t.kind in ("hqkv", "hpost", "ffn")]
        attn_prog = {a: attention_program(L, nmb) for a in range(self.r)}
        mi, ai = 0, {a: 0 for a in range(self.r)}
        deadline = time.monotonic() + self.wait_timeout_s
        while mi < len(model_prog) or any(ai[a] < len(attn_prog[a]) for a in range(self.r)):
            progressed = False
            if mi < len(model_prog):
                t = model_prog[mi]
                if t.kind == "hqkv":
                    self._hqkv(t.layer, t.mb, states[t.mb], slots[t.mb], mbs[t.mb][2], seq_lens[t.mb])
                    if drop == ("qkv", t.layer, t.mb):
                        for w in self.windows:
                            w.flags[0, t.layer, t.mb] = 0
                    mi, progressed = mi + 1, True
                elif t.kind == "hpost":
                    if all(w.ready(1, t.layer, t.mb) for w in self.windows):
                        self._hpost_ffn(t.layer, t.mb, states[t.mb])
                        mi, progressed = mi + 1, True
                else:                                             # ffn is folded into hpost above
                    mi, progressed = mi + 1, True
            for a, w in enumerate(self.windows):
                if ai[a] >= len(attn_prog[a]):
                    continue
                t = attn_prog[a][ai[a]]
                if t.kind == "pre":
                    if w.ready(0, t.layer, t.mb):
                        ai[a], progressed = ai[a] + 1, True
                else:
                    st = states[t.mb]
                    sel = st.owner == a
                    li = m.full_index[t.layer]
                    self.attn[a].attn(li, t.mb, sel, slots[t.mb][sel], mbs[t.mb][2][sel], seq_lens[t.mb][sel].to(torch.int32), ps)
                    if drop != ("o", t.layer, t.mb):
                        w.release(1, t.layer, t.mb)
                    ai[a], progressed = ai[a] + 1, True
            if not progressed:
                if time.monotonic() > deadline:
                    for w in self.windows:
                        w.set_err(1)
                    raise CadStepAborted("a CAD wait timed out; err word set, step discarded")
                time.sleep(0.001)
        out = []
        for st in states:
            out.append(self.sample_mb(st))
        for w in self.windows:                                    # epoch bump is the last action of a step
            w.bump_epoch()
        return out

    def reset_error(self) -> None:
        """After an aborted step: clear err and move every window to a fresh epoch so that stale
        flags of the aborted step can never satisfy a wait."""
        for w in self.windows:
            w.err.zero_()
            w.bump_epoch()
