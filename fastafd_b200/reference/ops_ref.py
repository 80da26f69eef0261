"""Plain PyTorch implementations of every op (CPU-capable, any float dtype).

They are the oracle that the CUDA kernels are tested against, and the compute path
of CPU/gloo runs. Each mirrors the contract of one kernel in ``csrc/``; maths is
done in fp32 and rounded to the input dtype at the same points as the kernels.
"""
from __future__ import annotations

import math

import torch

FP8_MAX = 448.0


# ----------------------------------------------------------------------------- norms
def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float, offset1: bool = False) -> torch.Tensor:
    xf = x.float()
    inv = torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    g = w.float() + (1.0 if offset1 else 0.0)
    return (xf * inv * g).to(x.dtype)


def add_rmsnorm(x, residual, w, eps, offset1: bool = False):
    """residual <- x + residual (rounded to dtype); returns rmsnorm(residual)."""
    r = (x.float() + residual.float()).to(x.dtype)
    residual.copy_(r)
    return rmsnorm(r, w, eps, offset1)


# ------------------------------------------------------------------------------ rope
def scale_inv_freq(inv_freq: torch.Tensor, rot_dim: int, theta: float, scaling) -> torch.Tensor:
    """Long-context frequency scaling of the RoPE table.

    ``llama3``: wavelengths longer than orig/low_freq_factor are slowed by ``factor``, shorter
    than orig/high_freq_factor are kept, with a linear blend in between. ``yarn``: frequencies
    are divided by ``factor`` along a linear ramp between the dimensions that make beta_fast and
    beta_slow rotations over the original window (no magnitude correction of cos/sin).
    Reference: python/minisgl/layers/rotary.py:72-116."""
    if not scaling:
        return inv_freq
    kind = scaling.get("rope_type", scaling.get("type", "default"))
    if kind in ("default", "linear") and "factor" not in scaling:
        return inv_freq
    if kind == "linear":
        return inv_freq / float(scaling["factor"])
    if kind == "llama3":
        f = float(scaling["factor"])
        lo, hi = float(scaling["low_freq_factor"]), float(scaling["high_freq_factor"])
        orig = float(scaling["original_max_position_embeddings"])
        wave = 2 * math.pi / inv_freq
        if lo == hi:
            return torch.where(wave < orig / hi, inv_freq, inv_freq / f)
        blend = ((orig / wave - lo) / (hi - lo)).clamp(0, 1)
        return inv_freq * ((1 - blend) / f + blend)
    if kind == "yarn":
        f = float(scaling["factor"])
        orig = float(scaling["original_max_position_embeddings"])
        half = rot_dim // 2

        def dim_of(rotations: float) -> float:
            return rot_dim * math.log(orig / (rotations * 2 * math.pi)) / (2 * math.log(theta))

        first = max(math.floor(dim_of(float(scaling.get("beta_fast", 32.0)))), 0)
        last = min(math.ceil(dim_of(float(scaling.get("beta_slow", 1.0)))), half - 1)
        ramp = ((torch.arange(half, dtype=torch.float32) - first) / max(last - first, 1)).clamp(0, 1)
        return inv_freq / f * ramp + inv_freq * (1 - ramp)
    if kind == "default":
        return inv_freq
    raise ValueError(f"unsupported rope scaling {scaling!r}")


def build_cos_sin_cache(max_pos: int, rot_dim: int, theta: float, device=None, scaling=None) -> torch.Tensor:
    """[max_pos, rot_dim] fp32: first half cos, second half sin (NeoX pairing)."""
    inv_freq = 1.0 / (theta ** (torch.arange(0, rot_dim, 2, dtype=torch.float32) / rot_dim))
    inv_freq = scale_inv_freq(inv_freq, rot_dim, theta, scaling)
    t = torch.arange(max_pos, dtype=torch.float32)
    freqs = torch.outer(t, inv_freq)
    return torch.cat([freqs.cos(), freqs.sin()], dim=-1).to(device)


def apply_rope_neox(x: torch.Tensor, cos_sin: torch.Tensor, positions: torch.Tensor, rot_dim: int):
    """x: [T, heads, D]; rotates the first rot_dim dims with pairs (i, i + rot_dim/2)."""
    half = rot_dim // 2
    cs = cos_sin[positions.long()]  # [T, rot_dim]
    cos, sin = cs[:, None, :half], cs[:, None, half:]
    xf = x.float()
    a, b = xf[..., :half], xf[..., half:rot_dim]
    out = xf.clone()
    out[..., :half] = a * cos - b * sin
    out[..., half:rot_dim] = b * cos + a * sin
    return out.to(x.dtype)


def qk_norm_rope_store(qkv, qw, kw, cos_sin, positions, out_loc, k_cache, v_cache, Hq, Hkv, D,
                       rot_dim, eps):
    """In place on qkv [T, (Hq+2Hkv)*D]; stores K (roped) and V at slots out_loc (-1 = skip)."""
    T = qkv.shape[0]
    v3 = qkv.view(T, Hq + 2 * Hkv, D)
    q, k, v = v3[:, :Hq], v3[:, Hq:Hq + Hkv], v3[:, Hq + Hkv:]
    if qw is not None:
        q = rmsnorm(q, qw, eps)
    if kw is not None:
        k = rmsnorm(k, kw, eps)
    q = apply_rope_neox(q, cos_sin, positions, rot_dim)
    k = apply_rope_neox(k, cos_sin, positions, rot_dim)
    v3[:, :Hq] = q
    v3[:, Hq:Hq + Hkv] = k
    if k_cache is not None:
        ok = out_loc >= 0
        loc = out_loc[ok].long()
        k_cache[loc] = k[ok].to(k_cache.dtype)
        v_cache[loc] = v[ok].to(v_cache.dtype)
    return qkv


# ------------------------------------------------------------------------- attention
def decode_attention(q, k_cache, v_cache, page_table, seq_lens, Hq, Hkv, D, q_len, page_size,
                     sm_scale):
    """q: [B*q_len, Hq, D]; caches [slots, Hkv, D]; returns [B*q_len, Hq, D]."""
    B = seq_lens.shape[0]
    G = Hq // Hkv
    out = torch.zeros_like(q)
    for b in range(B):
        L = int(seq_lens[b])
        if L <= 0:
            continue
        t = torch.arange(L, device=q.device)
        slots = page_table[b, (t // page_size).long()].long() * page_size + (t % page_size)
        k = k_cache[slots].float()  # [L, Hkv, D]
        v = v_cache[slots].float()
        for j in range(q_len):
            lim = L - q_len + 1 + j
            if lim <= 0:
                continue
            qj = q[b * q_len + j].float().view(Hkv, G, D)
            s = torch.einsum("hgd,lhd->hgl", qj, k[:lim]) * sm_scale
            p = torch.softmax(s, dim=-1)
            o = torch.einsum("hgl,lhd->hgd", p, v[:lim])
            out[b * q_len + j] = o.reshape(Hq, D).to(q.dtype)
    return out


def prefill_attention(q, k, v, Hq, Hkv, D, sm_scale, prefix_k=None, prefix_v=None):
    """Causal attention of one sequence chunk. q/k/v: [L, H*, D]; prefix_*: cached [P, Hkv, D]."""
    L = q.shape[0]
    G = Hq // Hkv
    if prefix_k is not None and prefix_k.shape[0] > 0:
        k = torch.cat([prefix_k.to(k.dtype), k], 0)
        v = torch.cat([prefix_v.to(v.dtype), v], 0)
    P = k.shape[0] - L
    qf = q.float().view(L, Hkv, G, D)
    s = torch.einsum("lhgd,mhd->hglm", qf, k.float()) * sm_scale
    mask = torch.arange(k.shape[0], device=q.device)[None, :] <= (torch.arange(L, device=q.device)[:, None] + P)
    s = s.masked_fill(~mask[None, None], float("-inf"))
    p = torch.softmax(s, dim=-1)
    o = torch.einsum("hglm,mhd->lhgd", p, v.float())
    return o.reshape(L, Hq, D).to(q.dtype)


# ---------------------------------------------------------------------------- router
def topk_route(logits, bias, K: int, scoring: str = "softmax", renorm: bool = True, scale: float = 1.0):
    """Returns (idx int32 [T,K], weights fp32 [T,K]). Ties go to the lower expert id."""
    lf = logits.float()
    if scoring == "softmax":
        scores = torch.softmax(lf, dim=-1)
        sel = scores
    elif scoring == "sigmoid":
        scores = torch.sigmoid(lf)
        sel = scores + (bias.float() if bias is not None else 0.0)
    else:
        raise ValueError(scoring)
    # stable sort descending => equal values keep ascending index order
    order = torch.sort(sel, dim=-1, descending=True, stable=True).indices[:, :K]
    w = torch.gather(scores, 1, order)
    if renorm:
        w = w / w.sum(-1, keepdim=True).clamp_min(1e-20)
    return order.to(torch.int32), (w * scale).float()


def grouped_topk_route(logits, bias, K, n_group, topk_group, renorm=True, scale=1.0):
    """GLM-4 / DeepSeek style: sigmoid scores, pick topk_group groups by the sum of each
    group's top-2 biased scores, then top-K inside the chosen groups."""
    T, E = logits.shape
    scores = torch.sigmoid(logits.float())
    sel = scores + (bias.float() if bias is not None else 0.0)
    g = sel.view(T, n_group, E // n_group)
    gscore = g.topk(2, dim=-1).values.sum(-1)
    gidx = gscore.topk(topk_group, dim=-1).indices
    gmask = torch.zeros(T, n_group, dtype=torch.bool, device=logits.device).scatter_(1, gidx, True)
    masked = sel.masked_fill(~gmask[:, :, None].expand_as(g).reshape(T, E), float("-inf"))
    order = torch.sort(masked, dim=-1, descending=True, stable=True).indices[:, :K]
    w = torch.gather(scores, 1, order)
    if renorm:
        w = w / w.sum(-1, keepdim=True).clamp_min(1e-20)
    return order.to(torch.int32), (w * scale).float()


# ------------------------------------------------------------------------------- mlp
def silu_mul(gate_up: torch.Tensor) -> torch.Tensor:
    I = gate_up.shape[-1] // 2
    g, u = gate_up[..., :I].float(), gate_up[..., I:].float()
    return (torch.nn.functional.silu(g) * u).to(gate_up.dtype)


def moe_experts(x, topk_idx, topk_w, w_gate_up, w_down, expert_base: int = 0, scale: float = 1.0):
    """Dense-loop MoE: x [T,H]; w_gate_up [E,2I,H] (gate rows then up rows); w_down [E,H,I].
    Experts outside [expert_base, expert_base+E) contribute nothing. Per-(token,k)
    expert outputs are rounded to x.dtype before the weighted fp32 sum, as the
    combine buffers hold them in that dtype."""
    T, H = x.shape
    E = w_gate_up.shape[0]
    out = torch.zeros(T, H, dtype=torch.float32, device=x.device)
    for e in range(E):
        sel = (topk_idx == e + expert_base)
        if not sel.any():
            continue
        tok, k = sel.nonzero(as_tuple=True)
        xe = x[tok].float()
        gu = (xe @ w_gate_up[e].float().t()).to(x.dtype)
        h = silu_mul(gu)
        ye = (h.float() @ w_down[e].float().t()).to(x.dtype)
        out.index_add_(0, tok, ye.float() * topk_w[tok, k].float()[:, None])
    return (out * scale).to(x.dtype)


# ----------------------------------------------------------------------------- fp8
def _to_e4m3(x: torch.Tensor) -> torch.Tensor:
    return x.clamp(-FP8_MAX, FP8_MAX).to(torch.float8_e4m3fn)


def group_quant_fp8(x: torch.Tensor, group: int = 128, pow2: bool = False):
    """Per-row, per-`group` e4m3 quantisation: scale = max(amax, 1e-10)/448 (optionally
    rounded up to a power of two). Returns (q e4m3 [rows,H], scales fp32 [rows,H/group])."""
    rows, H = x.shape
    xf = x.float().view(rows, H // group, group)
    amax = xf.abs().amax(-1).clamp_min(1e-10)
    scale = amax / FP8_MAX
    if pow2:
        scale = torch.exp2(torch.ceil(torch.log2(scale)))
    q = _to_e4m3(xf / scale[..., None]).view(rows, H)
    return q, scale


def group_dequant_fp8(q: torch.Tensor, scale: torch.Tensor, group: int = 128) -> torch.Tensor:
    rows, H = q.shape
    return (q.float().view(rows, H // group, group) * scale[..., None]).view(rows, H)


def block_quant_fp8(w: torch.Tensor, block: int = 128):
    """128x128 block quantisation of a weight [N,K]: returns (e4m3 [N,K], scale fp32
    [ceil(N/b), ceil(K/b)]) with w ~= q * scale (the checkpoint's weight_scale_inv)."""
    N, K = w.shape
    nb, kb = (N + block - 1) // block, (K + block - 1) // block
    wp = torch.zeros(nb * block, kb * block, dtype=torch.float32, device=w.device)
    wp[:N, :K] = w.float()
    blk = wp.view(nb, block, kb, block)
    amax = blk.abs().amax(dim=(1, 3)).clamp_min(1e-10)
    scale = amax / FP8_MAX
    q = _to_e4m3(blk / scale[:, None, :, None]).view(nb * block, kb * block)[:N, :K].contiguous()
    return q, scale


def block_dequant_fp8(q: torch.Tensor, scale: torch.Tensor, block: int = 128) -> torch.Tensor:
    N, K = q.shape
    s = scale.repeat_interleave(block, 0)[:N].repeat_interleave(block, 1)[:, :K]
    return q.float() * s


def fp8_gemm_nt(xq, xs, wq, ws, out_dtype=torch.bfloat16, block: int = 128):
    """out[m,n] = sum_kb (xq[m,kb] . wq[n,kb]) * xs[m,kb] * ws[n/128,kb]: the exact
    block-scaled contract (fp32 accumulation per 128-deep K block)."""
    M, K = xq.shape
    N = wq.shape[0]
    out = torch.zeros(M, N, dtype=torch.float32, device=xq.device)
    xf, wf = xq.float(), wq.float()
    wsr = ws.repeat_interleave(block, 0)[:N]
    for kb in range(K // block):
        part = xf[:, kb * block:(kb + 1) * block] @ wf[:, kb * block:(kb + 1) * block].t()
        out += part * xs[:, kb:kb + 1] * wsr[:, kb][None, :]
    return out.to(out_dtype)


# ---------------------------------------------------------------------- sampling
def argmax_lowest(logits: torch.Tensor) -> torch.Tensor:
    """Arg-max with ties to the lowest index."""
    mx = logits.max(dim=-1, keepdim=True).values
    idx = torch.arange(logits.shape[-1], device=logits.device).expand_as(logits)
    return torch.where(logits == mx, idx, logits.shape[-1]).min(dim=-1).values.to(torch.int32)


def sample(logits: torch.Tensor, temperatures, top_ks, top_ps, generator=None) -> torch.Tensor:
    """Greedy rows (temperature <= 0) take the arg-max; others temperature-softmax then
    top-k / top-p filtering and a multinomial draw."""
    T, V = logits.shape
    out = argmax_lowest(logits)
    for i in range(T):
        temp = float(temperatures[i])
        if temp <= 0:
            continue
        p = torch.softmax(logits[i].float() / temp, -1)
        k = int(top_ks[i])
        if 0 < k < V:
            kth = p.topk(k).values[-1]
            p = torch.where(p < kth, torch.zeros_like(p), p)
        tp = float(top_ps[i])
        if tp < 1.0:
            sp, si = p.sort(descending=True)
            cum = sp.cumsum(0)
            cut = (cum - sp) > tp
            sp = torch.where(cut, torch.zeros_like(sp), sp)
            p = torch.zeros_like(p).scatter_(0, si, sp)
        p = p / p.sum()
        out[i] = torch.multinomial(p, 1, generator=generator).to(torch.int32)[0]
    return out


def greedy_accept(draft: torch.Tensor, target: torch.Tensor):
    """draft: [B, block-1] proposed tokens; target: [B, block] arg-max of the target model at
    each verified position. Accept the longest prefix of the draft equal to the target,
    then emit the target's token. Returns (n_emitted [B], emitted [B, block])."""
    B, blk = target.shape
    match = (draft == target[:, :blk - 1]).int()
    acc = match.cumprod(dim=1).sum(dim=1)  # accepted draft tokens
    n = acc + 1
    pos = torch.arange(blk, device=target.device)[None, :]
    emitted = torch.where(pos < n[:, None], target, torch.full_like(target, -1))
    return n.to(torch.int32), emitted


# ----------------------------------------------------------------- gated DeltaNet
def l2norm(x, eps=1e-6):
    return x * torch.rsqrt((x * x).sum(-1, keepdim=True) + eps)


def gdn_recurrent_step(q, k, v, a, b, A_log, dt_bias, state):
    """One token of the gated delta rule per request.
    q,k: [B,Hk,Dk]; v: [B,Hv,Dv]; a,b: [B,Hv]; state: [B,Hv,Dv,Dk] fp32 (updated in place).
    Hv is a multiple of Hk (query/key heads are repeated). Returns out [B,Hv,Dv]."""
    B, Hk, Dk = q.shape
    Hv = v.shape[1]
    rep = Hv // Hk
    qf = l2norm(q.float()).repeat_interleave(rep, 1) * (Dk ** -0.5)
    kf = l2norm(k.float()).repeat_interleave(rep, 1)
    g = -torch.exp(A_log.float())[None] * torch.nn.functional.softplus(a.float() + dt_bias.float()[None])
    beta = torch.sigmoid(b.float())
    state.mul_(torch.exp(g)[..., None, None])
    kv = torch.einsum("bhvk,bhk->bhv", state, kf)
    delta = (v.float() - kv) * beta[..., None]
    state.add_(torch.einsum("bhv,bhk->bhvk", delta, kf))
    out = torch.einsum("bhvk,bhk->bhv", state, qf)
    return out.to(v.dtype)


def gdn_prefill(q, k, v, a, b, A_log, dt_bias, state):
    """Token-serial reference over one sequence. q,k: [L,Hk,Dk]; v: [L,Hv,Dv]; a,b: [L,Hv];
    state [Hv,Dv,Dk] fp32 updated in place. Returns [L,Hv,Dv]."""
    outs = []
    st = state.unsqueeze(0)
    for t in range(q.shape[0]):
        outs.append(gdn_recurrent_step(q[t:t + 1], k[t:t + 1], v[t:t + 1], a[t:t + 1], b[t:t + 1],
                                       A_log, dt_bias, st)[0])
    return torch.stack(outs, 0)


def causal_conv1d_step(x, conv_state, weight, bias=None, activation=True):
    """Depthwise causal conv, one token. x: [B,C]; conv_state: [B,taps-1... stored as [B,W-1,C]]
    holds the previous W-1 inputs (oldest first) and is shifted in place; weight [C,W]."""
    W = weight.shape[1]
    full = torch.cat([conv_state.float(), x.float()[:, None, :]], dim=1)  # [B,W,C]
    y = (full * weight.float().t()[None]).sum(1)
    if bias is not None:
        y = y + bias.float()
    conv_state.copy_(full[:, 1:].to(conv_state.dtype))
    if activation:
        y = torch.nn.functional.silu(y)
    return y.to(x.dtype)


def gated_rmsnorm(x, z, w, eps):
    """Per-head RMSNorm(x) * w * silu(z). x,z: [..., D]."""
    xf = x.float()
    inv = torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return (xf * inv * w.float() * torch.nn.functional.silu(z.float())).to(x.dtype)


def softmax_scale(head_dim: int) -> float:
    return 1.0 / math.sqrt(head_dim)
