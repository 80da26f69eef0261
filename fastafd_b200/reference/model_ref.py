"""Whole-sequence reference forward: no paging, no KV cache, no micro-batches, no stages.

Given the weights held by an :class:`AttentionStage` and the :class:`ExpertStage` objects
(single rank each), it recomputes the full causal forward over a token sequence with plain
tensor algebra. It is the oracle for everything the serving path adds (paged KV, chunked
prefill, ping-pong pipeline, dispatch/combine, graphs): greedy tokens must be identical.
"""
from __future__ import annotations

from typing import List, Sequence

import torch
import torch.nn.functional as F

from ..config import ModelConfig
from . import ops_ref as ref


def _w(stage, name):
    return stage.w[name].float()


def _moe(cfg: ModelConfig, layer: int, x: torch.Tensor, attn_stage, expert_stages) -> torch.Tensor:
    p = f"model.layers.{layer}.mlp."
    gw = attn_stage.w[p + "gate.weight"].float()
    logits = x.float() @ gw.t()
    bias = attn_stage.w.get(p + "gate.e_score_correction_bias")
    if cfg.n_group > 1:
        idx, w = ref.grouped_topk_route(logits, bias, cfg.num_experts_per_tok, cfg.n_group, cfg.topk_group,
                                        cfg.norm_topk_prob)
    else:
        idx, w = ref.topk_route(logits, bias, cfg.num_experts_per_tok, cfg.scoring, cfg.norm_topk_prob)
    out = torch.zeros_like(x, dtype=torch.float32)
    for k in range(idx.shape[1]):
        for t in range(x.shape[0]):
            e = int(idx[t, k])
            st = expert_stages[e // expert_stages[0].experts_local]
            el = e - st.expert_base
            gu = x[t].float() @ st.gate_up[layer][el].float().t()
            h = ref.silu_mul(gu[None])[0]
            out[t] += w[t, k] * (h @ st.down[layer][el].float().t())
    out = out * cfg.routed_scaling_factor
    return out


def _dense_or_shared(cfg: ModelConfig, layer: int, x: torch.Tensor, stage):
    p = f"model.layers.{layer}.mlp."
    if not cfg.is_moe_layer(layer):
        h = ref.silu_mul(x.float() @ _w(stage, p + "gate_up_proj.weight").t())
        return h @ _w(stage, p + "down_proj.weight").t()
    if cfg.num_shared_experts > 0:
        h = ref.silu_mul(x.float() @ _w(stage, p + "shared_expert.gate_up_proj.weight").t())
        out = h @ _w(stage, p + "shared_expert.down_proj.weight").t()
        if cfg.shared_expert_gate:
            out = out * torch.sigmoid(x.float() @ _w(stage, p + "shared_expert_gate.weight").t())
        return out
    return None


def _full_attention(cfg: ModelConfig, layer: int, x: torch.Tensor, stage, positions) -> torch.Tensor:
    p = f"model.layers.{layer}.self_attn."
    D, Hq, Hkv = cfg.head_dim, cfg.num_q_heads, cfg.num_kv_heads
    L = x.shape[0]
    qkv = x.float() @ _w(stage, p + "qkv_proj.weight").t()
    if p + "qkv_proj.bias" in stage.w:
        qkv = qkv + _w(stage, p + "qkv_proj.bias")
    gate = None
    if cfg.attn_output_gate:
        q, gate, rest = qkv[:, :Hq * D], qkv[:, Hq * D:2 * Hq * D], qkv[:, 2 * Hq * D:]
    else:
        q, rest = qkv[:, :Hq * D], qkv[:, Hq * D:]
    k, v = rest[:, :Hkv * D], rest[:, Hkv * D:]
    if cfg.qk_norm == "head":
        off = 1.0 if cfg.norm_offset1 else 0.0
        q = ref.rmsnorm(q.view(L, Hq, D), _w(stage, p + "q_norm.weight") + off, cfg.rms_eps)
        k = ref.rmsnorm(k.view(L, Hkv, D), _w(stage, p + "k_norm.weight") + off, cfg.rms_eps)
    elif cfg.qk_norm == "cross_head":
        q = ref.rmsnorm(q, _w(stage, p + "q_norm.weight"), cfg.rms_eps).view(L, Hq, D)
        k = ref.rmsnorm(k, _w(stage, p + "k_norm.weight"), cfg.rms_eps).view(L, Hkv, D)
    else:
        q, k = q.view(L, Hq, D), k.view(L, Hkv, D)
    q = ref.apply_rope_neox(q, stage.cos_sin.float(), positions, cfg.rotary_dim)
    k = ref.apply_rope_neox(k, stage.cos_sin.float(), positions, cfg.rotary_dim)
    o = ref.prefill_attention(q, k, v.reshape(L, Hkv, D), Hq, Hkv, D, ref.softmax_scale(D)).reshape(L, Hq * D)
    if gate is not None:
        o = o * torch.sigmoid(gate)
    return o @ _w(stage, p + "o_proj.weight").t()


def _linear_attention(cfg: ModelConfig, layer: int, x: torch.Tensor, stage) -> torch.Tensor:
    p = f"model.layers.{layer}.linear_attn."
    hk, hv, dk, dv = cfg.gdn_num_k_heads, cfg.gdn_num_v_heads, cfg.gdn_head_k_dim, cfg.gdn_head_v_dim
    L = x.shape[0]
    xf = x.float()
    mixed = xf @ _w(stage, p + "in_proj_qkv.weight").t()
    z = xf @ _w(stage, p + "in_proj_z.weight").t()
    b = xf @ _w(stage, p + "in_proj_b.weight").t()
    a = xf @ _w(stage, p + "in_proj_a.weight").t()
    cw = _w(stage, p + "conv1d.weight")                      # [C, W]
    W = cw.shape[1]
    padded = torch.cat([torch.zeros(W - 1, mixed.shape[1]), mixed], 0)
    y = torch.stack([(padded[t:t + W] * cw.t()).sum(0) for t in range(L)], 0)
    y = F.silu(y)
    q = y[:, :hk * dk].reshape(L, hk, dk)
    k = y[:, hk * dk:2 * hk * dk].reshape(L, hk, dk)
    v = y[:, 2 * hk * dk:].reshape(L, hv, dv)
    state = torch.zeros(hv, dv, dk)
    o = ref.gdn_prefill(q, k, v, a, b, _w(stage, p + "A_log"), _w(stage, p + "dt_bias"), state)
    o = ref.gated_rmsnorm(o, z.view(L, hv, dv), _w(stage, p + "norm.weight"), cfg.rms_eps).reshape(L, hv * dv)
    return o @ _w(stage, p + "out_proj.weight").t()


def forward_logits(cfg: ModelConfig, stage, expert_stages, ids: Sequence[int]) -> torch.Tensor:
    """Logits of the last position for the token sequence `ids` (fp32)."""
    t = torch.tensor(ids, dtype=torch.long)
    pos = torch.arange(len(ids))
    off = cfg.norm_offset1
    h = _w(stage, "model.embed_tokens.weight")[t]
    for i in range(cfg.num_layers):
        p = f"model.layers.{i}."
        x = ref.rmsnorm(h, _w(stage, p + "input_layernorm.weight"), cfg.rms_eps, off)
        if cfg.layer_type(i) == "full":
            a = _full_attention(cfg, i, x, stage, pos)
        else:
            a = _linear_attention(cfg, i, x, stage)
        h = h + a
        x = ref.rmsnorm(h, _w(stage, p + "post_attention_layernorm.weight"), cfg.rms_eps, off)
        m = torch.zeros_like(h)
        if cfg.is_moe_layer(i):
            m = m + _moe(cfg, i, x, stage, expert_stages)
        extra = _dense_or_shared(cfg, i, x, stage)
        if extra is not None:
            m = m + extra
        h = h + m
    x = ref.rmsnorm(h[-1:], _w(stage, "model.norm.weight"), cfg.rms_eps, off)
    head = _w(stage, "model.embed_tokens.weight") if cfg.tie_embeddings else _w(stage, "lm_head.weight")
    return (x @ head.t())[0]


def greedy_generate_reference(cfg: ModelConfig, stage, expert_stages, prompts: List[List[int]], n: int) -> List[List[int]]:
    outs = []
    for prompt in prompts:
        ids = list(prompt)
        new = []
        for _ in range(n):
            tok = int(ref.argmax_lowest(forward_logits(cfg, stage, expert_stages, ids)[None])[0])
            ids.append(tok)
            new.append(tok)
        outs.append(new)
    return outs


def score_continuations(cfg: ModelConfig, stage, expert_stages, prompts: List[List[int]], outputs: List[List[int]]) -> dict:
    """Teacher-forced scoring of sampled continuations: for every emitted token, its rank in this
    reference forward's logits at that position (0 = the reference's own greedy choice). The rates
    say how close a serving engine stays to the reference even after a near-tie flipped one token
    (after which a token-for-token comparison is meaningless).
    Reference: scripts/validate/compare_minisgl_vllm.py + check_alignment_report.py (rank hit rates of
    the engine's greedy continuations under another engine's logprobs)."""
    ranks: List[List[int]] = []
    for prompt, out in zip(prompts, outputs):
        r = []
        for j, tok in enumerate(out):
            lg = forward_logits(cfg, stage, expert_stages, list(prompt) + list(out[:j]))
            r.append(int((lg > lg[tok]).sum()))
        ranks.append(r)
    flat = [x for r in ranks for x in r]
    n = max(len(flat), 1)
    return {"ranks": ranks, "tokens": len(flat),
            "top1_agreement_rate": sum(x == 0 for x in flat) / n,
            "top10_hit_rate": sum(x < 10 for x in flat) / n,
            "top100_hit_rate": sum(x < 100 for x in flat) / n}


def logit_check(cfg: ModelConfig, stage, expert_stages, prompts: List[List[int]], outputs: List[List[int]], taps,
                rel_tol: float = 0.05, min_within: float = 0.75) -> dict:
    """Compare the logits a serving engine produced with this reference forward, teacher-forced on
    the engine's own tokens.

    `taps` are the engine's (table rows, kv lengths, logits) records (AttentionWorker.logit_tap);
    prompts must have distinct lengths (a row is matched to its request by the length of its first
    record). For every record the reference recomputes the whole sequence (prompt + the tokens the
    engine emitted so far) in fp32 from `stage` / `expert_stages` (give it the weight values the
    engine computes with, e.g. bf16-rounded). A position is *within tolerance* when every logit is
    within `rel_tol` x the standard deviation of the reference logits of that position. Rounding can
    flip a router near-tie, which changes a token's experts and with them the logits by more than
    any rounding tolerance, so the criterion is: at least `min_within` of the positions are within
    tolerance, and on those the engine's argmax equals the reference's whenever the reference's
    top-2 gap exceeds twice the tolerance (one exception allowed per 20 positions).
    Returns the statistics; raises AssertionError when the criterion fails."""
    by_len = {len(p): i for i, p in enumerate(prompts)}
    assert len(by_len) == len(prompts), "prompts must have distinct lengths"
    row_req = {}
    ratios, n_arg, n_arg_ok = [], 0, 0
    for rows, lens, logits in taps:
        for row, L, lg in zip(rows.tolist(), lens.tolist(), logits):
            if row not in row_req:
                if L not in by_len:
                    continue                      # a padding row
                row_req[row] = by_len[L]
            r = row_req[row]
            j = L - len(prompts[r])
            if j < 0 or j >= len(outputs[r]):
                continue
            want = forward_logits(cfg, stage, expert_stages, list(prompts[r]) + list(outputs[r][:j]))
            tol = rel_tol * float(want.std())
            err = float((lg[:cfg.vocab_size] - want).abs().max())
            ratios.append(err / tol)
            top2 = want.topk(2).values
            if err <= tol and float(top2[0] - top2[1]) > 2 * tol:
                n_arg += 1
                n_arg_ok += int(int(lg[:cfg.vocab_size].argmax()) == int(want.argmax()))
    ratios.sort()
    within = sum(1 for x in ratios if x <= 1.0)
    stats = {"positions": len(ratios), "within_tolerance": within,
             "median_err_over_tol": round(ratios[len(ratios) // 2], 3) if ratios else None,
             "max_err_over_tol": round(ratios[-1], 3) if ratios else None, "argmax_checked": n_arg, "argmax_equal": n_arg_ok}
    assert ratios, "no logits were recorded"
    assert within >= min_within * len(ratios), f"too few positions within tolerance: {stats}"
    assert n_arg_ok >= n_arg - max(1, n_arg // 20) and n_arg > 0, f"argmax differs on confident positions: {stats}"
    return stats


def bf16_rounded_copy(stage):
    """A CPU fp32 copy of a stage whose weights hold the values a bf16 engine built from the same
    seed computes with: everything the engine keeps in bf16 is rounded to bf16, tensors it keeps in
    fp32 (router gate of fp32-routed models, selection bias, A_log, dt_bias) are left as they are."""
    import copy

    c = copy.copy(stage)
    if hasattr(stage, "param_shapes"):
        kinds = {k: kind for k, (_, kind) in stage.param_shapes().items()}
        c.w = {k: (v if kinds.get(k) == "fp32" else v.to(torch.bfloat16).float()) for k, v in stage.w.items()}
    else:
        c.gate_up = {k: v.to(torch.bfloat16).float() for k, v in stage.gate_up.items()}
        c.down = {k: v.to(torch.bfloat16).float() for k, v in stage.down.items()}
    return c
