"""Operator surface. CUDA tensors go to the sm_100a kernel library; CPU tensors go to the
PyTorch oracle in :mod:`fastafd_b200.reference.ops_ref` (CPU/gloo runs and tests).

There is one CUDA implementation per op and no backend selection: a CUDA tensor on a
machine without the built library raises.
"""
from __future__ import annotations

import ctypes as C
from typing import Optional

import torch

from ..reference import ops_ref as ref
from . import _lib
from ._lib import GroupedGemmDesc, check, cur_stream, lib, ptr

EPI_STORE, EPI_SWIGLU, EPI_COMBINE = 0, 1, 2
NUM_SMS = 148


# ----------------------------------------------------------------------------- norms
def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float, offset1: bool = False,
            out: Optional[torch.Tensor] = None) -> torch.Tensor:
    if not x.is_cuda:
        return ref.rmsnorm(x, w, eps, offset1)
    x2 = x.reshape(-1, x.shape[-1])
    out = torch.empty_like(x2) if out is None else out
    check(lib().afd_rmsnorm(ptr(x2), None, ptr(w), ptr(out), x2.shape[0], x2.shape[1], eps,
                            int(offset1), cur_stream()), "rmsnorm")
    return out.view(x.shape)


def add_rmsnorm(x: torch.Tensor, residual: torch.Tensor, w: torch.Tensor, eps: float,
                offset1: bool = False, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """residual <- x + residual in place; returns rmsnorm(residual) * w."""
    if not x.is_cuda:
        r = ref.add_rmsnorm(x, residual, w, eps, offset1)
        return r if out is None else out.copy_(r)
    out = torch.empty_like(x) if out is None else out
    check(lib().afd_rmsnorm(ptr(x), ptr(residual), ptr(w), ptr(out), x.shape[0], x.shape[1], eps,
                            int(offset1), cur_stream()), "add_rmsnorm")
    return out


def qk_norm_rope_store(qkv, qw, kw, cos_sin, positions, out_loc, k_cache, v_cache, Hq, Hkv, D,
                       rot_dim, eps, status=None):
    """In place on the first (Hq+2Hkv)*D columns of qkv [T, >= (Hq+2Hkv)*D] (rows may carry more
    columns behind them, e.g. an output gate): per-head RMSNorm of q/k (when weights given), NeoX
    RoPE, and a store of k/v into the paged cache ([slots,Hkv,D]) at out_loc (-1 skips)."""
    if not qkv.is_cuda:
        n = (Hq + 2 * Hkv) * D
        if qkv.shape[1] != n:
            part = qkv[:, :n].contiguous()
            ref.qk_norm_rope_store(part, qw, kw, cos_sin, positions, out_loc, k_cache, v_cache, Hq, Hkv, D, rot_dim, eps)
            qkv[:, :n] = part
            return qkv
        return ref.qk_norm_rope_store(qkv, qw, kw, cos_sin, positions, out_loc, k_cache, v_cache,
                                      Hq, Hkv, D, rot_dim, eps)
    T = qkv.shape[0]
    assert qkv.stride(1) == 1
    slots = k_cache.shape[0] if k_cache is not None else 0
    check(lib().afd_qk_norm_rope_store(ptr(qkv), qkv.stride(0), ptr(qw), ptr(kw), ptr(cos_sin), ptr(positions),
                                       ptr(out_loc), ptr(k_cache), ptr(v_cache), T, Hq, Hkv, D,
                                       rot_dim, eps, cos_sin.shape[0], slots, ptr(status),
                                       cur_stream()), "qk_norm_rope_store")
    return qkv


def cross_head_norm_rope_store(qkv, qw, kw, cos_sin, positions, out_loc, k_cache, v_cache, Hq, Hkv, D, rot_dim, eps,
                               q_denom: int, k_denom: int, sq: Optional[torch.Tensor] = None, status=None):
    """MiniMax-M2 attention prologue in one launch, in place on qkv [T, (Hq+2Hkv)*D] bf16 (CUDA):
    RMSNorm over all q heads jointly and all k heads jointly (`q_denom` / `k_denom` = element
    counts of the full, unsharded q and k; `sq` [T,2] = all-reduced sums of squares under TP, else
    computed here), weights per element, then RoPE and the paged K/V store."""
    T = qkv.shape[0]
    assert qkv.is_cuda and qkv.stride(1) == 1
    slots = k_cache.shape[0] if k_cache is not None else 0
    check(lib().afd_cross_head_norm_rope_store(ptr(qkv), qkv.stride(0), ptr(qw), ptr(kw), ptr(sq), float(q_denom),
                                               float(k_denom), ptr(cos_sin), ptr(positions), ptr(out_loc), ptr(k_cache),
                                               ptr(v_cache), T, Hq, Hkv, D, rot_dim, eps, cos_sin.shape[0], slots,
                                               ptr(status), cur_stream()), "cross_head_norm_rope_store")
    return qkv


def qk_square_sums(qkv, q_elems: int, k_elems: int) -> torch.Tensor:
    """[T,2] fp32 sums of squares of the first q_elems and the next k_elems columns of each row."""
    out = torch.empty(qkv.shape[0], 2, dtype=torch.float32, device=qkv.device)
    check(lib().afd_qk_square_sums(ptr(qkv), qkv.stride(0), ptr(out), qkv.shape[0], q_elems, k_elems, cur_stream()),
          "qk_square_sums")
    return out


def grouped_topk_route(logits, bias, K: int, n_group: int, topk_group: int, renorm: bool = True, scale: float = 1.0,
                       out_idx=None, out_w=None):
    """GLM-4 / DeepSeek routing (sigmoid scores, group-limited top-k). logits [T,E] fp32 or bf16."""
    if not logits.is_cuda:
        idx, w = ref.grouped_topk_route(logits, bias, K, n_group, topk_group, renorm, scale)
        if out_idx is not None:
            return out_idx.copy_(idx), out_w.copy_(w)
        return idx, w
    T, E = logits.shape
    if logits.dtype not in (torch.float32, torch.bfloat16) or not logits.is_contiguous():
        logits = logits.float().contiguous()
    idx = torch.empty(T, K, dtype=torch.int32, device=logits.device) if out_idx is None else out_idx
    w = torch.empty(T, K, dtype=torch.float32, device=logits.device) if out_w is None else out_w
    check(lib().afd_grouped_topk_route(ptr(logits), ptr(bias), ptr(idx), ptr(w), T, E, K, n_group, topk_group,
                                       int(renorm), scale, int(logits.dtype == torch.bfloat16), cur_stream()),
          "grouped_topk_route")
    return idx, w


def shared_gate_mul(x, gate_w, y):
    """y[t] *= sigmoid(x[t] . gate_w) in place (Qwen3.5 shared-expert gate); gate_w [1,H] or [H]."""
    if not y.is_cuda:
        g = torch.sigmoid(torch.nn.functional.linear(x, gate_w.view(1, -1)).float())
        return y.copy_((y.float() * g).to(y.dtype))
    assert x.is_contiguous() and y.is_contiguous() and x.dtype == torch.bfloat16 and gate_w.dtype == torch.bfloat16
    check(lib().afd_shared_gate_mul(ptr(x), ptr(gate_w), ptr(y), x.shape[0], x.shape[1], cur_stream()), "shared_gate_mul")
    return y


def sigmoid_gate_mul(o, gate):
    """o *= sigmoid(gate) in place; o contiguous [T,n] bf16, gate a [T,n] view whose rows may be strided."""
    if not o.is_cuda:
        return o.copy_((o.float() * torch.sigmoid(gate.float())).to(o.dtype))
    assert o.is_contiguous() and gate.stride(1) == 1 and gate.shape == o.shape
    check(lib().afd_sigmoid_gate_mul(ptr(o), ptr(gate), gate.stride(0), o.shape[0], o.shape[1], cur_stream()),
          "sigmoid_gate_mul")
    return o


def embedding(ids: torch.Tensor, table: torch.Tensor, vocab_start: int = 0,
              out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Rows of `table` for ids in [vocab_start, vocab_start + rows); zeros elsewhere."""
    if not table.is_cuda:
        local = ids.long() - vocab_start
        ok = (local >= 0) & (local < table.shape[0])
        res = table[local.clamp(0, table.shape[0] - 1)]
        return torch.where(ok[:, None], res, torch.zeros_like(res))
    T, H = ids.shape[0], table.shape[1]
    out = torch.empty(T, H, dtype=table.dtype, device=table.device) if out is None else out
    check(lib().afd_embedding(ptr(ids), ptr(table), ptr(out), T, H, vocab_start,
                              vocab_start + table.shape[0], cur_stream()), "embedding")
    return out


def silu_mul(gate_up: torch.Tensor) -> torch.Tensor:
    if not gate_up.is_cuda:
        return ref.silu_mul(gate_up)
    rows, I2 = gate_up.shape
    out = torch.empty(rows, I2 // 2, dtype=gate_up.dtype, device=gate_up.device)
    check(lib().afd_silu_mul(ptr(gate_up), ptr(out), rows, I2 // 2, cur_stream()), "silu_mul")
    return out


def topk_route(logits: torch.Tensor, bias: Optional[torch.Tensor], K: int, scoring: str = "softmax",
               renorm: bool = True, scale: float = 1.0, out_idx=None, out_w=None):
    """Router scoring + top-k. logits fp32 [T,E]. Returns (idx int32 [T,K], w fp32 [T,K])."""
    if not logits.is_cuda:
        idx, w = ref.topk_route(logits, bias, K, scoring, renorm, scale)
        if out_idx is not None:
            return out_idx.copy_(idx), out_w.copy_(w)
        return idx, w
    T, E = logits.shape
    if logits.dtype not in (torch.float32, torch.bfloat16) or not logits.is_contiguous():
        logits = logits.float().contiguous()
    idx = torch.empty(T, K, dtype=torch.int32, device=logits.device) if out_idx is None else out_idx
    w = torch.empty(T, K, dtype=torch.float32, device=logits.device) if out_w is None else out_w
    check(lib().afd_topk_route(ptr(logits), ptr(bias), ptr(idx), ptr(w), T, E, K,
                               0 if scoring == "softmax" else 1, int(renorm), scale,
                               int(logits.dtype == torch.bfloat16), cur_stream()),
          "topk_route")
    return idx, w


def argmax(logits: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    if not logits.is_cuda:
        return ref.argmax_lowest(logits)
    T, V = logits.shape
    out = torch.empty(T, dtype=torch.int32, device=logits.device) if out is None else out
    if logits.dtype not in (torch.bfloat16, torch.float32):
        logits = logits.float()
    scratch = torch.empty(T * lib().afd_argmax_chunks(V) * 2, dtype=torch.float32, device=logits.device)
    check(lib().afd_argmax(ptr(logits), ptr(out), T, V, logits.stride(0),
                           int(logits.dtype == torch.bfloat16), ptr(scratch), cur_stream()), "argmax")
    return out


def sample(logits: torch.Tensor, temperatures: torch.Tensor, top_ks: torch.Tensor, top_ps: torch.Tensor,
           generator: Optional[torch.Generator] = None, uniform: Optional[torch.Tensor] = None,
           out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """One token per row: arg-max where temperature <= 0, else temperature softmax, top-k /
    top-p filtering and a multinomial draw (inverse CDF from `uniform`, drawn from `generator`
    when not given). CUDA rows run csrc/sampling.cu; CPU rows the oracle."""
    if not logits.is_cuda:
        return ref.sample(logits, temperatures, top_ks, top_ps, generator)
    T, V = logits.shape
    dev = logits.device
    if logits.dtype not in (torch.bfloat16, torch.float32):
        logits = logits.float()
    if logits.stride(1) != 1:
        logits = logits.contiguous()
    if uniform is None:
        uniform = torch.rand(T, device=dev, dtype=torch.float32, generator=generator)
    out = torch.empty(T, dtype=torch.int32, device=dev) if out is None else out
    t = temperatures.to(device=dev, dtype=torch.float32).contiguous()
    k = top_ks.to(device=dev, dtype=torch.int32).contiguous()
    p = top_ps.to(device=dev, dtype=torch.float32).contiguous()
    check(lib().afd_sample(ptr(logits), logits.stride(0), T, V, int(logits.dtype == torch.bfloat16), ptr(t), ptr(k),
                           ptr(p), ptr(uniform.contiguous()), ptr(out), cur_stream()), "sample")
    return out


def group_quant_fp8(x: torch.Tensor, group: int = 128, pow2: bool = False):
    if not x.is_cuda:
        return ref.group_quant_fp8(x, group, pow2)
    rows, H = x.shape
    q = torch.empty(rows, H, dtype=torch.float8_e4m3fn, device=x.device)
    s = torch.empty(rows, H // group, dtype=torch.float32, device=x.device)
    check(lib().afd_group_quant_fp8(ptr(x), ptr(q), ptr(s), rows, H, group, int(pow2), cur_stream()),
          "group_quant_fp8")
    return q, s


# ------------------------------------------------------------------------- attention
def prefill_attention_varlen(q, k_cache, v_cache, page_table, seq_lens, q_starts, max_q_len: int, Hq, Hkv, D, page_size,
                             sm_scale, out=None, status=None):
    """Causal attention of every request's new chunk against its paged KV, all requests in one launch
    (CUDA). q [sum of chunk lengths, Hq, D] bf16 (rows may be strided); q_starts int32 [B+1] = row
    offsets of the chunks; seq_lens [B] = KV length including the chunk. Returns [rows, Hq, D]."""
    B = seq_lens.shape[0]
    if q.stride(2) != 1 or q.stride(1) != D:
        q = q.contiguous()
    out = torch.zeros(q.shape, dtype=q.dtype, device=q.device) if out is None else out
    check(lib().afd_prefill_attention_varlen(ptr(q), q.stride(0), ptr(k_cache), ptr(v_cache), ptr(page_table), ptr(seq_lens),
                                             ptr(q_starts), ptr(out), B, Hq, Hkv, D, max_q_len, page_size,
                                             page_table.shape[1], k_cache.shape[0], sm_scale, ptr(status), cur_stream()),
          "prefill_attention_varlen")
    return out


def decode_attn_workspace(B, Hq, Hkv, q_len, D, splits, device) -> Optional[torch.Tensor]:
    if splits <= 1:
        return None
    n = lib().afd_decode_attn_workspace_bytes(B, Hq, Hkv, q_len, D, splits)
    return torch.zeros(n, dtype=torch.uint8, device=device)    # arrival counters start at zero


def pick_attn_splits(B: int, Hkv: int, m_tiles: int, max_kv: int, D: int = 128) -> int:
    """KV splits of the decode attention kernel for a grid of B*Hkv*m_tiles row tiles.

    Fitted to timings on B200: one CTA streams its KV range at a rate set by latency, and an
    SM runs two CTAs (head dims up to 128) about as fast as one, a third one at the cost of
    more time. So the time of a launch goes as  (1/s) * max(1, ceil(ctas*s/SMs) / 2)  plus a
    small cost per split for the merge; the grid never exceeds one wave of resident CTAs and
    a split never gets fewer than 256 tokens."""
    resident = 3 if D <= 128 else 1
    conc = 2 if D <= 128 else 1
    ctas = max(1, B * Hkv * m_tiles)
    s_max = max(1, min(max_kv // 256, (NUM_SMS * resident) // ctas, 32))
    best, best_cost = 1, None
    for s in range(1, s_max + 1):
        per_sm = -(-ctas * s // NUM_SMS)
        cost = max(1.0, per_sm / conc) / s + 0.01 * s
        if best_cost is None or cost < best_cost - 1e-9:
            best, best_cost = s, cost
    return best


def decode_attention(q, k_cache, v_cache, page_table, seq_lens, Hq, Hkv, D, q_len, page_size,
                     sm_scale, splits: int = 1, workspace=None, out=None, status=None, out_ptr: Optional[int] = None):
    """Paged GQA decode attention. q [B*q_len, Hq, D] bf16 (rows may be strided, e.g. a view
    into a merged qkv buffer); caches [slots, Hkv, D]. Returns a contiguous [B*q_len, Hq, D]."""
    if not q.is_cuda:
        return ref.decode_attention(q, k_cache, v_cache, page_table, seq_lens, Hq, Hkv, D, q_len,
                                    page_size, sm_scale)
    B = seq_lens.shape[0]
    if q.stride(2) != 1 or q.stride(1) != D:
        q = q.contiguous()
    if out_ptr is None:
        out = torch.empty(q.shape, dtype=q.dtype, device=q.device) if out is None else out
        out_ptr = ptr(out)
    # (`out_ptr`: a raw device address for the [B*q_len, Hq, D] result, e.g. a peer GPU's buffer)
    if splits > 1 and workspace is None:
        workspace = decode_attn_workspace(B, Hq, Hkv, q_len, D, splits, q.device)
    check(lib().afd_decode_attention_strided(ptr(q), q.stride(0), ptr(k_cache), ptr(v_cache), ptr(page_table),
                                     ptr(seq_lens), out_ptr, ptr(workspace), B, Hq, Hkv, D, q_len,
                                     page_size, page_table.shape[1], k_cache.shape[0], splits,
                                     sm_scale, ptr(status), cur_stream()), "decode_attention")
    return out


# ---------------------------------------------------------------------- grouped GEMM
def interleave_gate_up(w_gate_up: torch.Tensor) -> torch.Tensor:
    """[E, 2I, H] with gate rows then up rows -> rows interleaved in groups of 16
    (rows 32b..32b+15 = gate features 16b.., rows 32b+16..32b+31 = up features 16b..),
    the layout the SWIGLU epilogue of the grouped GEMM expects."""
    E, I2, H = w_gate_up.shape
    I = I2 // 2
    g = w_gate_up[:, :I].reshape(E, I // 16, 16, H)
    u = w_gate_up[:, I:].reshape(E, I // 16, 16, H)
    return torch.stack([g, u], dim=2).reshape(E, I2, H).contiguous()


def interleave_gate_up_scales(scale: torch.Tensor, I: int, block: int = 128) -> torch.Tensor:
    """Block scales [E, 2I/128, K/128] of a gate-then-up weight -> per-tile-half scales
    [E, n_tiles, 2, K/128] for the interleaved layout (half 0 = gate lanes, 1 = up lanes)."""
    E, _, KB = scale.shape
    n_tiles = 2 * I // 128
    gate_blocks = I // block
    tiles = torch.arange(n_tiles, device=scale.device)
    feat0 = tiles * 64
    gb = feat0 // block
    ub = gate_blocks + gb
    return torch.stack([scale[:, gb], scale[:, ub]], dim=2).contiguous()


def tile_major(w: torch.Tensor) -> torch.Tensor:
    """[..., N, K] weights (N % 128 == 0, K a multiple of the 128-byte k block) -> the same bytes stored
    tile by tile, [..., N/128, K/kblk, 128, kblk]: each 128-row x 128-byte tile the GEMM loads is one
    consecutive 16 KB piece of memory. Pass the result with ``w_tile_major=True``."""
    kblk = 128 // w.element_size()
    *lead, N, K = w.shape
    t = w.reshape(*lead, N // 128, 128, K // kblk, kblk)
    nd = t.dim()
    return t.permute(*range(nd - 4), nd - 4, nd - 2, nd - 3, nd - 1).contiguous()


def plain_tile_scales(scale: torch.Tensor) -> torch.Tensor:
    """[E, N/128, K/128] -> [E, n_tiles, 2, K/128] for non-interleaved weights."""
    return torch.stack([scale, scale], dim=2).contiguous()


def dense_tile_schedule(M: int, block_tok: int, device) -> tuple[torch.Tensor, torch.Tensor]:
    """tile_info / num_tok_tiles for a single-expert (dense) GEMM over M rows."""
    n = (M + block_tok - 1) // block_tok
    info = torch.zeros(max(n, 1), 4, dtype=torch.int32)
    for t in range(n):
        info[t, 0] = 0
        info[t, 1] = t * block_tok
        info[t, 2] = min(block_tok, M - t * block_tok)
    return info.to(device), torch.tensor([n], dtype=torch.int32, device=device)


def grouped_gemm(*, w, x, num_experts, n_per_expert, k, tile_info, num_tok_tiles, block_tok,
                 epilogue, out=None, out_ld=0, fp8=False, x_scale=None, w_scale=None, out_q=None,
                 out_scale=None, row_meta=None, peer_combine=(), peer_flag=(), combine_tokens=0,
                 hidden=0, epoch=None, done_counter=None, status=None, grid=NUM_SMS, trace=None,
                 k_splits=1, splitk_ws=None, splitk_cnt=None, bias=None, w_tile_major=False, l2_prefetch_bytes=0):
    """Low-level launcher of the tcgen05 grouped GEMM (see csrc/grouped_gemm.cu). `l2_prefetch_bytes`:
    while the kernel still waits for its predecessor, its CTAs pull up to this many bytes (in total) of
    the weights of their likely first work units into L2 (a hint; 0 = off)."""
    d = GroupedGemmDesc()
    d.w, d.x = ptr(w), ptr(x)
    d.num_experts, d.n_per_expert, d.k, d.pool_rows = num_experts, n_per_expert, k, x.shape[0]
    d.block_tok, d.fp8, d.epilogue, d.grid = block_tok, int(fp8), epilogue, grid
    d.tile_info, d.num_tok_tiles = ptr(tile_info), ptr(num_tok_tiles)
    d.max_tok_tiles = tile_info.shape[0]
    d.out, d.out_ld = ptr(out), out_ld
    d.x_scale, d.w_scale, d.out_q, d.out_scale = ptr(x_scale), ptr(w_scale), ptr(out_q), ptr(out_scale)
    d.row_meta = ptr(row_meta)
    for i, p in enumerate(peer_combine):
        d.peer_combine[i] = p
    for i, p in enumerate(peer_flag):
        d.peer_flag[i] = p
    d.num_peers, d.combine_tokens, d.hidden = len(peer_combine), combine_tokens, hidden
    d.epoch, d.done_counter, d.status, d.trace = ptr(epoch), ptr(done_counter), ptr(status), ptr(trace)
    d.k_splits, d.splitk_ws, d.splitk_cnt, d.bias = k_splits, ptr(splitk_ws), ptr(splitk_cnt), ptr(bias)
    d.w_tile_major = int(w_tile_major)
    d.l2_prefetch_bytes = int(l2_prefetch_bytes)
    check(lib().afd_grouped_gemm(C.byref(d), cur_stream()), "grouped_gemm")


_DENSE_SCHEDULES: dict = {}


_SPLITK_WS: dict = {}


def pick_k_splits(tok_tiles: int, n_tiles: int, k_blocks: int) -> int:
    """K splits of a dense GEMM with tok_tiles x n_tiles output tiles. Measured on B200: a split pays
    only while the launch stays within one wave of SMs and each unit keeps a long K range (the fence +
    arrival counter + partial sum of a split cost about as much as 16 K blocks of streaming), so: at
    most one unit per SM, at least 16 K blocks per unit, an exact division of K."""
    tiles = max(1, tok_tiles * n_tiles)
    best = 1
    for s in range(1, 33):
        if k_blocks % s != 0 or k_blocks // s < 16:
            continue
        if tiles * s <= NUM_SMS:
            best = s
    return best


def _splitk_buffers(tiles: int, k_splits: int, block_tok: int, device):
    """Workspace + zeroed arrival counters of the current stream (kernels on one stream run in order;
    two streams must not share them). Sized once for the largest split launch there can be
    (pick_k_splits keeps tiles x splits within two units per SM, a tile is at most 128 x 128 fp32), so
    the addresses captured in CUDA graphs never change."""
    key = (str(device), cur_stream())
    if key not in _SPLITK_WS:
        _SPLITK_WS[key] = (torch.empty(2 * NUM_SMS * 128 * 128, dtype=torch.float32, device=device),
                           torch.zeros(2 * NUM_SMS, dtype=torch.int32, device=device))
    ws, cnt = _SPLITK_WS[key]
    if tiles * k_splits * block_tok * 128 > ws.numel() or tiles > cnt.numel():
        raise ValueError("split-K launch larger than the fixed workspace; pass fewer k_splits")
    return ws, cnt


def dense_gemm(x: torch.Tensor, w: torch.Tensor, block_tok: Optional[int] = None, status=None,
               out: Optional[torch.Tensor] = None, bias: Optional[torch.Tensor] = None, k_splits: int = 0,
               x_scale: Optional[torch.Tensor] = None, w_scale: Optional[torch.Tensor] = None):
    """out = x @ w.T (+ bias) on the tcgen05 path, weights on the UMMA M side (N % 128 == 0).
    bf16: x [M,K] bf16, w [N,K] bf16, K % 64 == 0. Block-FP8: x e4m3 with `x_scale` [M, K/128] (1x128
    groups), w e4m3 with `w_scale` in the kernel's per-tile layout (ops.plain_tile_scales), K % 128 == 0.
    With few output tiles the K dimension is split over several CTAs whose fp32 partials the last one
    sums (`k_splits` 0 = choose). Tile schedules and split-K buffers are built once per shape / stream
    and kept on the device, so calls can be captured into a CUDA graph."""
    M, K = x.shape
    N = w.shape[0]
    fp8 = x.dtype == torch.float8_e4m3fn
    if block_tok is None:
        block_tok = 16 if M <= 16 else 32 if M <= 32 else 64 if (M <= 64 or fp8) else 128
    key = (M, block_tok, x.device)
    if key not in _DENSE_SCHEDULES:
        _DENSE_SCHEDULES[key] = dense_tile_schedule(M, block_tok, x.device)
    info, n = _DENSE_SCHEDULES[key]
    tok_tiles, n_tiles, k_blocks = info.shape[0], N // 128, K // (128 if fp8 else 64)
    if k_splits <= 0:
        k_splits = pick_k_splits(tok_tiles, n_tiles, k_blocks)
    ws = cnt = None
    if k_splits > 1:
        ws, cnt = _splitk_buffers(tok_tiles * n_tiles, k_splits, block_tok, x.device)
    if out is None:
        out = torch.empty(M, N, dtype=torch.bfloat16, device=x.device)
    grouped_gemm(w=w, x=x, num_experts=1, n_per_expert=N, k=K, tile_info=info, num_tok_tiles=n,
                 block_tok=block_tok, epilogue=EPI_STORE, out=out, out_ld=N, status=status, fp8=fp8,
                 x_scale=x_scale, w_scale=w_scale, k_splits=k_splits, splitk_ws=ws, splitk_cnt=cnt, bias=bias)
    return out
