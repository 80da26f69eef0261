"""Core-attention disaggregation on GPUs: hop kernels over the peer-memory fabric.

The model GPU runs the whole model except the attention core. For every full-attention layer and
micro-batch it projects q|k|v (with norm and RoPE applied), *puts* the rows of the requests each
attention GPU owns into that GPU's window and releases a flag; the attention GPU waits for the flag,
stores K/V into its paged pool, and runs decode attention with the output written straight into the
model GPU's window, then releases the o flag; the model GPU waits for the o flags of all its
attention GPUs and goes on with o_proj, the router and the experts.

Two objects:

* :class:`CadModelHook` is installed into an :class:`~fastafd_b200.models.transformer.AttentionStage`
  (``stage.cad = hook``); the stage's attention block then calls ``hook.attention(...)`` instead of
  storing K/V and running attention locally. Everything around it (the colocated MoE, CUDA graphs,
  sampling) is the ordinary engine.
* :class:`CadAttentionServer` lives on an attention GPU: KV pool, page tables, and one
  ``serve(layer, lane)`` call per (layer, micro-batch) of a step.

With ``Fabric.local`` both live in one process on one GPU and the hook calls the server inline
between its put and its wait, so every flag is already set when it is waited for (one stream; this is
how the path is tested on a single GPU). With ``Fabric.ipc`` they are separate processes and the
server runs its fixed program ``for layer: for lane: serve`` for every step.

Every wait is bounded and reports into the window's err word; a set err word makes later waits return
at once, the step's result is discarded and :meth:`check` raises :class:`CadStepAborted`.

Reference: python/minisgl/cad/{window,layout,model_side,attn_side}.py, python/minisgl/kernel/cad_hop.py.
"""
from __future__ import annotations

import ctypes as C
from typing import List, Optional

import torch

from .. import ops
from ..config import ModelConfig
from ..ops._lib import check, cur_stream, lib, ptr
from ..parallel.fabric import Fabric, Layout
from ..reference import ops_ref as ref
from .runtime import CadStepAborted

VP = C.c_void_p


def _bind():
    L = lib()
    if getattr(L, "_cad_bound", False):
        return L
    L.afd_cad_put_rows.restype = C.c_int
    L.afd_cad_put_rows.argtypes = [VP, C.c_long, VP, C.c_int, C.c_int, VP, VP, VP, VP, VP]
    L.afd_cad_wait_store.restype = C.c_int
    L.afd_cad_wait_store.argtypes = [VP, VP, VP, VP, VP, VP, C.c_int, C.c_int, C.c_int, C.c_int, C.c_long, C.c_ulonglong, VP, VP]
    L.afd_cad_wait.restype = C.c_int
    L.afd_cad_wait.argtypes = [VP, C.c_long, C.c_int, VP, C.c_ulonglong, VP, VP]
    L.afd_cad_flag.restype = C.c_int
    L.afd_cad_flag.argtypes = [VP, VP, VP]
    L.afd_cad_epoch.restype = C.c_int
    L.afd_cad_epoch.argtypes = [VP, VP]
    L._cad_bound = True
    return L


def attention_window_layout(cfg: ModelConfig, num_lanes: int, max_tokens: int) -> Layout:
    """Heap of an attention GPU: the q|k|v rows it is sent, one flag per (layer, lane), epoch, err."""
    lay = Layout()
    row = (cfg.num_q_heads + 2 * cfg.num_kv_heads) * cfg.head_dim
    for l in range(num_lanes):
        lay.add(f"qkv{l}", max_tokens * row * 2)
    lay.add("qkv_flag", cfg.num_layers * num_lanes * 4)
    lay.add("words", 64)          # [0] epoch, [1] put counter (unused here), [4] err
    return lay


def model_window_layout(cfg: ModelConfig, num_attn: int, num_lanes: int, max_tokens: int) -> Layout:
    """Heap of the model GPU: attention output rows per (attention GPU, lane), o flags, epoch, err."""
    lay = Layout()
    for a in range(num_attn):
        for l in range(num_lanes):
            lay.add(f"o{a}_{l}", max_tokens * cfg.q_size * 2)
    lay.add("o_flag", num_attn * cfg.num_layers * num_lanes * 4)
    lay.add("words", 64)
    return lay


class CadAttentionServer:
    """Attention GPU `index`: KV pool and the per-(layer, lane) wait-store + attention + flag."""

    def __init__(self, cfg: ModelConfig, fabric: Fabric, model_rank: int, index: int, num_attn: int, num_lanes: int,
                 max_tokens: int, num_pages: int, page_size: int, timeout_ns: int = int(5e9)):
        _bind()
        self.cfg, self.fab, self.index, self.num_lanes, self.max_tokens = cfg, fabric, index, num_lanes, max_tokens
        self.page_size, self.timeout_ns = page_size, timeout_ns
        dev = fabric.heap.device
        self.lay = attention_window_layout(cfg, num_lanes, max_tokens)
        self.mlay = model_window_layout(cfg, num_attn, num_lanes, max_tokens)
        row = (cfg.num_q_heads + 2 * cfg.num_kv_heads) * cfg.head_dim
        heap = fabric.heap
        self.qkv = [heap.view(self.lay.offset(f"qkv{l}"), (max_tokens, row), torch.bfloat16) for l in range(num_lanes)]
        self.flag = heap.view(self.lay.offset("qkv_flag"), (cfg.num_layers, num_lanes), torch.int32)
        self.words = heap.view(self.lay.offset("words"), (16,), torch.int32)
        self.flag.zero_()
        self.words.zero_()
        self.epoch, self.err = self.words[0:1], self.words[4:5]
        n = cfg.num_full_attn_layers
        self.k = torch.zeros(n, num_pages * page_size, cfg.num_kv_heads, cfg.head_dim, dtype=torch.bfloat16, device=dev)
        self.v = torch.zeros_like(self.k)
        # where this GPU's output rows and flags live in the model GPU's heap
        self.peer_o = [fabric.peer_ptr(model_rank, self.mlay.offset(f"o{index}_{l}")) for l in range(num_lanes)]
        self.peer_o_flag = fabric.peer_ptr(model_rank, self.mlay.offset("o_flag")) + 4 * index * cfg.num_layers * num_lanes
        # per lane: the step's metadata for the rows this GPU owns (device tensors, graph-stable)
        z = lambda *s, d=torch.int32: torch.zeros(*s, dtype=d, device=dev)  # noqa: E731
        self.out_loc = [z(max_tokens) for _ in range(num_lanes)]
        self.seq_lens = [z(max_tokens) for _ in range(num_lanes)]
        self.page_table: List[Optional[torch.Tensor]] = [None] * num_lanes
        self.n_rows = [0] * num_lanes
        self.full_index = {}
        for i in range(cfg.num_layers):
            if cfg.layer_type(i) == "full":
                self.full_index[i] = len(self.full_index)

    def set_step(self, lane: int, out_loc: torch.Tensor, seq_lens: torch.Tensor, page_table: torch.Tensor) -> None:
        """Metadata of the rows of this lane that this GPU owns, in the order the model GPU puts them."""
        n = out_loc.shape[0]
        self.n_rows[lane] = n
        self.out_loc[lane][:n].copy_(out_loc)
        self.seq_lens[lane][:n].copy_(seq_lens)
        self.page_table[lane] = page_table

    def serve(self, layer: int, lane: int) -> None:
        c, L = self.cfg, _bind()
        n, li = self.n_rows[lane], self.full_index[layer]
        D, Hq, Hkv = c.head_dim, c.num_q_heads, c.num_kv_heads
        rows = self.qkv[lane]
        check(L.afd_cad_wait_store(ptr(self.flag[layer, lane:lane + 1]), ptr(self.epoch), ptr(rows), ptr(self.out_loc[lane]),
                                   ptr(self.k[li]), ptr(self.v[li]), n, rows.shape[1], Hq * D, Hkv * D, self.k.shape[1],
                                   C.c_ulonglong(self.timeout_ns), ptr(self.err), cur_stream()), "cad_wait_store")
        if n > 0:
            q = rows[:n].view(n, Hq + 2 * Hkv, D)[:, :Hq]
            # the output rows go straight into the model GPU's window (peer stores from the attention kernel)
            ops.decode_attention(q, self.k[li], self.v[li], self.page_table[lane], self.seq_lens[lane][:n], Hq, Hkv, D, 1,
                                 self.page_size, ref.softmax_scale(D), out_ptr=self.peer_o[lane], status=self.err)
        flag = self.peer_o_flag + 4 * (layer * self.num_lanes + lane)
        check(L.afd_cad_flag(flag, ptr(self.epoch), cur_stream()), "cad_flag")

    def end_step(self) -> None:
        check(_bind().afd_cad_epoch(ptr(self.epoch), cur_stream()), "cad_epoch")

    def check(self) -> None:
        code = int(self.err.item())
        if code:
            raise CadStepAborted(f"attention GPU {self.index}: window err word = {code}")

    def reset_error(self) -> None:
        self.err.zero_()
        self.epoch.add_(1)


class CadModelHook:
    """Model-GPU side of the hop. `owner[lane]` [T] int32 names the attention GPU of every token row;
    `servers` (loopback only) are called inline between put and wait."""

    def __init__(self, cfg: ModelConfig, fabric: Fabric, attn_ranks: List[int], num_lanes: int, max_tokens: int,
                 servers: Optional[List[CadAttentionServer]] = None, timeout_ns: int = int(5e9)):
        _bind()
        self.cfg, self.fab, self.attn_ranks, self.num_lanes, self.max_tokens = cfg, fabric, attn_ranks, num_lanes, max_tokens
        self.servers, self.timeout_ns = servers, timeout_ns
        A = len(attn_ranks)
        dev = fabric.heap.device
        self.lay = model_window_layout(cfg, A, num_lanes, max_tokens)
        self.alay = attention_window_layout(cfg, num_lanes, max_tokens)
        heap = fabric.heap
        self.o = [[heap.view(self.lay.offset(f"o{a}_{l}"), (max_tokens, cfg.q_size), torch.bfloat16) for l in range(num_lanes)]
                  for a in range(A)]
        self.o_flag = heap.view(self.lay.offset("o_flag"), (A, cfg.num_layers, num_lanes), torch.int32)
        self.words = heap.view(self.lay.offset("words"), (16,), torch.int32)
        self.o_flag.zero_()
        self.words.zero_()
        self.epoch, self.err = self.words[0:1], self.words[4:5]
        self.done = torch.zeros(A, num_lanes, dtype=torch.int32, device=dev)
        self.peer_qkv = [[fabric.peer_ptr(r, self.alay.offset(f"qkv{l}")) for l in range(num_lanes)] for r in attn_ranks]
        self.peer_flag = [fabric.peer_ptr(r, self.alay.offset("qkv_flag")) for r in attn_ranks]
        # per lane: which rows go to which attention GPU (device index lists), set per step
        self.sel: List[List[Optional[torch.Tensor]]] = [[None] * num_lanes for _ in range(A)]
        self.gather: List[Optional[torch.Tensor]] = [None] * num_lanes

    def set_step(self, lane: int, owner: torch.Tensor) -> None:
        """owner [T] int32: attention GPU of every row of this lane's micro-batch."""
        order = []
        for a in range(len(self.attn_ranks)):
            idx = torch.nonzero(owner == a, as_tuple=False).flatten().to(torch.int32)
            self.sel[a][lane] = idx
            order.append(idx)
        # row t of the micro-batch is row pos[t] of its owner's compacted block
        T = owner.shape[0]
        src_gpu = owner.long()
        pos = torch.zeros(T, dtype=torch.long, device=owner.device)
        for a, idx in enumerate(order):
            pos[idx.long()] = torch.arange(idx.numel(), device=owner.device)
        self.gather[lane] = (src_gpu, pos)

    def attention(self, layer: int, lane: int, qkv: torch.Tensor) -> torch.Tensor:
        """qkv [T, (Hq + 2 Hkv) D] with norm and RoPE applied -> attention output [T, Hq D]."""
        c, L = self.cfg, _bind()
        row = (c.num_q_heads + 2 * c.num_kv_heads) * c.head_dim
        for a in range(len(self.attn_ranks)):
            idx = self.sel[a][lane]
            flag = self.peer_flag[a] + 4 * (layer * self.num_lanes + lane)
            check(L.afd_cad_put_rows(ptr(qkv), qkv.stride(0), ptr(idx), idx.numel(), row, self.peer_qkv[a][lane], flag,
                                     ptr(self.epoch), ptr(self.done[a, lane:lane + 1]), cur_stream()), "cad_put_rows")
        if self.servers is not None:                      # loopback: the attention side runs here, in stream order
            for s in self.servers:
                s.serve(layer, lane)
        A = len(self.attn_ranks)
        check(L.afd_cad_wait(ptr(self.o_flag[:, layer, lane]), self.o_flag.stride(0), A, ptr(self.epoch),
                             C.c_ulonglong(self.timeout_ns), ptr(self.err), cur_stream()), "cad_wait")
        src_gpu, pos = self.gather[lane]
        if A == 1:
            return self.o[0][lane][:qkv.shape[0]]
        stacked = torch.stack([self.o[a][lane] for a in range(A)])       # [A, max_tokens, q_size]
        return stacked[src_gpu, pos]

    def end_step(self) -> None:
        check(_bind().afd_cad_epoch(ptr(self.epoch), cur_stream()), "cad_epoch")
        if self.servers is not None:
            for s in self.servers:
                s.end_step()

    def check(self) -> None:
        code = int(self.err.item())
        if code:
            raise CadStepAborted(f"model GPU: window err word = {code}")
        for s in self.servers or []:
            s.check()

    def reset_error(self) -> None:
        self.err.zero_()
        self.epoch.add_(1)
        for s in self.servers or []:
            s.reset_error()
