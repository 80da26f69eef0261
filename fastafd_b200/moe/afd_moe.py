"""Attention-side and expert-side endpoints of the fused N2M / M2N exchange (CUDA).

One *lane* per micro-batch. The attention endpoint pushes routed rows into the expert
GPUs' receive slots (optionally quantising to FP8 on the way) and later reduces the
top-k rows that the expert GPUs' down-projection epilogues stored into its combine
buffer. The expert endpoint waits for all attention ranks, groups rows by expert and
runs the two tcgen05 grouped GEMMs; the second one writes over NVLink.

Role parity with the reference: ``MegaMoEM2NAfdAdapter.ag_moe`` / ``eg_moe``
(python/minisgl/moe/megamoe_m2n_afd.py:336-470,755-911). Unlike the reference there is
no hidden % 512 / intermediate % 512 restriction: hidden % 128 == 0 and
intermediate % 128 == 0 (bf16: % 64) suffice.
"""
from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass
from typing import Dict, List, Optional

import torch

from ..ops import EPI_COMBINE, EPI_SWIGLU, NUM_SMS, grouped_gemm

# The gate/up GEMM is launched (programmatic dependent launch) while the kernel in front of it still
# runs or waits for the sources' flags; HBM is idle then, and the GEMM's resident CTAs use the time to
# pull this many bytes of their first weight tiles into L2 (FASTAFD_L2_PREFETCH_MB, 0 turns it off).
L2_PREFETCH_BYTES = int(float(os.environ.get("FASTAFD_L2_PREFETCH_MB", "64")) * (1 << 20))
from ..ops._lib import (CombineDesc, DirectDesc, DispatchDesc, GroupDesc, RouteDirectDesc, RouteDispatchDesc, ScheduleDesc,
                        check, cur_stream, lib, ptr)
from ..parallel.fabric import Fabric, Layout

DEFAULT_TIMEOUT_NS = int(float(os.environ.get("FASTAFD_FLAG_TIMEOUT_S", "20")) * 1e9)
TRACE_LEN = 1024      # rows of the device-side timeline ring (kTraceLen in csrc/common.cuh)


# A consumer kernel that spins on peer flags with all its CTAs resident takes SM slots, shared memory
# and issue bandwidth from whatever else runs meanwhile (the other micro-batch's attention, the
# other lane's GEMM): measured on the attention side, the lane's own chain shrank from 274 to 188 us
# (Qwen3-235B shapes) and from 65 to 58 us (Qwen3-30B shapes) once the wait ran as a single warp in
# a launch of its own in front of the consumer. FASTAFD_SPLIT_WAIT=0 puts the wait back inside.
_SPLIT_WAIT = os.environ.get("FASTAFD_SPLIT_WAIT", "1") != "0"


def _trace_enabled() -> bool:
    return os.environ.get("FASTAFD_COMM_TRACE", "0") == "1"


@dataclass(frozen=True)
class MoeCommConfig:
    num_ag: int              # attention ranks (dispatch sources)
    num_eg: int              # expert ranks
    num_lanes: int           # micro-batches in flight
    max_tokens: int          # tokens per attention rank per lane (receive capacity)
    hidden: int
    topk: int
    num_experts: int         # global routed experts (padded to a multiple of num_eg)
    intermediate: int
    fp8: bool = False
    block_tok: int = 32
    # Steps with at most this many tokens per attention rank use the direct exchange: rows are stored
    # straight into per-expert stripes of the expert GPU's pool (slot claimed with an atomic add), so
    # the expert side neither groups nor gathers. 0 switches it off (receive slots + grouping only).
    direct_tokens: int = 0

    @property
    def direct_cap(self) -> int:
        """Rows per expert stripe: every token of every source may choose the same expert."""
        n = self.num_ag * self.direct_tokens
        return (n + self.block_tok - 1) // self.block_tok * self.block_tok

    @property
    def direct_rows(self) -> int:
        return self.experts_per_eg * self.direct_cap

    def use_direct(self, tokens: int) -> bool:
        return 0 < tokens <= self.direct_tokens

    @property
    def experts_per_eg(self) -> int:
        return (self.num_experts + self.num_eg - 1) // self.num_eg

    @property
    def row_bytes(self) -> int:
        return self.hidden * (1 if self.fp8 else 2)

    @property
    def pool_rows(self) -> int:
        k_eff = min(self.topk, self.experts_per_eg)
        return self.num_ag * self.max_tokens * k_eff + self.experts_per_eg * self.block_tok

    @property
    def max_tok_tiles(self) -> int:
        k_eff = min(self.topk, self.experts_per_eg)
        return (self.num_ag * self.max_tokens * k_eff + self.block_tok - 1) // self.block_tok + self.experts_per_eg


def ag_layout(cfg: MoeCommConfig) -> Layout:
    lay = Layout()
    for lane in range(cfg.num_lanes):
        lay.add(f"combine{lane}", cfg.topk * cfg.max_tokens * cfg.hidden * 2)
        lay.add(f"m2n_flag{lane}", 4 * cfg.num_eg)
    return lay


def eg_layout(cfg: MoeCommConfig) -> Layout:
    lay = Layout()
    for lane in range(cfg.num_lanes):
        lay.add(f"recv_x{lane}", cfg.num_ag * cfg.max_tokens * cfg.row_bytes)
        lay.add(f"recv_scale{lane}", cfg.num_ag * cfg.max_tokens * (cfg.hidden // 128) * 4)
        lay.add(f"recv_idx{lane}", cfg.num_ag * cfg.max_tokens * cfg.topk * 4)
        lay.add(f"n2m_flag{lane}", 4 * cfg.num_ag)
        if cfg.direct_tokens > 0:
            lay.add(f"dpool_x{lane}", cfg.direct_rows * cfg.row_bytes)
            lay.add(f"dpool_scale{lane}", cfg.direct_rows * (cfg.hidden // 128) * 4)
            lay.add(f"dmeta{lane}", cfg.direct_rows * 4)
            lay.add(f"dcount{lane}", cfg.experts_per_eg * 4)
    return lay


def flag_report(flags: torch.Tensor, epoch_word: torch.Tensor, peer_ranks: List[int]) -> Dict[str, object]:
    """Where a lane's flag protocol stands, for the triage of a wait that ran out: the epoch this rank publishes
    or expects next, the last epoch each peer has written into this rank's flag words, and the peers that are
    behind the others (the ones a wait was waiting for). Reads device memory: call it after the failure, not
    on the hot path. Reference: python/minisgl/afd_worker_base.py:371-408 (barrier head dump)."""
    vals = [int(v) for v in flags.reshape(-1).tolist()]
    top = max(vals) if vals else 0
    return {"next_epoch": int(epoch_word.reshape(-1)[0]), "flags": {int(r): v for r, v in zip(peer_ranks, vals)},
            "behind": [int(r) for r, v in zip(peer_ranks, vals) if v < top]}


class _LaneWords:
    """Small device words a lane's kernels keep between launches."""

    def __init__(self, device):
        self.words = torch.zeros(8, dtype=torch.int32, device=device)
        self.words[0] = 1  # epoch to publish / expect next (flags start at 0)
        self.words[2] = 1  # second epoch (expert side: publish epoch)
        self.epoch = self.words[0:1]
        self.done = self.words[1:2]
        self.epoch2 = self.words[2:3]
        self.done2 = self.words[3:4]


class AgMoeEndpoint:
    """Attention rank `ag_index`: dispatch_push + combine over the fabric.

    `fabric.bases` is indexed by global rank; `eg_ranks[i]` is the global rank of expert
    GPU i."""

    def __init__(self, cfg: MoeCommConfig, fabric: Fabric, ag_index: int, eg_ranks: List[int],
                 device: torch.device, timeout_ns: int = DEFAULT_TIMEOUT_NS, status: Optional[torch.Tensor] = None):
        self.cfg, self.fabric, self.ag_index, self.eg_ranks, self.device = cfg, fabric, ag_index, eg_ranks, device
        self.timeout_ns = timeout_ns
        self.lay, self.eg_lay = ag_layout(cfg), eg_layout(cfg)
        # `status`: the process-wide device status word when the caller has one, so that a wait that
        # ran out anywhere on this GPU makes every later wait of every kernel return at once
        self.status = status if status is not None else torch.zeros(1, dtype=torch.int32, device=device)
        self.lanes = [_LaneWords(device) for _ in range(cfg.num_lanes)]
        self.trace = ([torch.zeros(TRACE_LEN, 4, dtype=torch.int64, device=device) for _ in range(cfg.num_lanes)]
                      if _trace_enabled() else None)
        heap = fabric.heap
        self.combine = [heap.view(self.lay.offset(f"combine{l}"), (cfg.topk, cfg.max_tokens, cfg.hidden),
                                  torch.bfloat16) for l in range(cfg.num_lanes)]
        self.m2n_flag = [heap.view(self.lay.offset(f"m2n_flag{l}"), (cfg.num_eg,), torch.int32)
                         for l in range(cfg.num_lanes)]
        self._dispatch_desc = [self._make_dispatch_desc(l) for l in range(cfg.num_lanes)]
        self._direct_desc = [self._make_direct_desc(l) for l in range(cfg.num_lanes)] if cfg.direct_tokens > 0 else None
        self.route_tokens_per_cta = int(os.environ.get("FASTAFD_ROUTE_TPC", "0"))
        self.route_cluster = int(os.environ.get("FASTAFD_ROUTE_CLUSTER", "0"))

    def flag_report(self) -> Dict[str, object]:
        """Per lane: the combine flags the expert ranks write here (see `flag_report`)."""
        return {f"lane{l}": flag_report(self.m2n_flag[l], self.lanes[l].epoch, self.eg_ranks) for l in range(self.cfg.num_lanes)}

    def _make_direct_desc(self, lane: int) -> DirectDesc:
        cfg, d = self.cfg, DirectDesc()
        d.num_eg, d.experts_per_eg, d.cap, d.fp8 = cfg.num_eg, cfg.experts_per_eg, cfg.direct_cap, int(cfg.fp8)
        d.H, d.K, d.src_rank = cfg.hidden, cfg.topk, self.ag_index
        for i, r in enumerate(self.eg_ranks):
            d.peer_pool[i] = self.fabric.peer_ptr(r, self.eg_lay.offset(f"dpool_x{lane}"))
            d.peer_scale[i] = self.fabric.peer_ptr(r, self.eg_lay.offset(f"dpool_scale{lane}"))
            d.peer_meta[i] = self.fabric.peer_ptr(r, self.eg_lay.offset(f"dmeta{lane}"))
            d.peer_count[i] = self.fabric.peer_ptr(r, self.eg_lay.offset(f"dcount{lane}"))
            d.peer_flag[i] = self.fabric.peer_ptr(r, self.eg_lay.offset(f"n2m_flag{lane}")) + 4 * self.ag_index
        w = self.lanes[lane]
        d.epoch, d.done_counter, d.status = ptr(w.epoch), ptr(w.done), ptr(self.status)
        d.trace = ptr(self.trace[lane]) if self.trace else None
        return d

    def _make_dispatch_desc(self, lane: int) -> DispatchDesc:
        cfg, d = self.cfg, DispatchDesc()
        d.H, d.K, d.src_rank, d.num_eg = cfg.hidden, cfg.topk, self.ag_index, cfg.num_eg
        d.experts_per_eg, d.fp8, d.recv_tokens = cfg.experts_per_eg, int(cfg.fp8), cfg.max_tokens
        for i, r in enumerate(self.eg_ranks):
            d.peer_recv_x[i] = self.fabric.peer_ptr(r, self.eg_lay.offset(f"recv_x{lane}"))
            d.peer_recv_scale[i] = self.fabric.peer_ptr(r, self.eg_lay.offset(f"recv_scale{lane}"))
            d.peer_recv_idx[i] = self.fabric.peer_ptr(r, self.eg_lay.offset(f"recv_idx{lane}"))
            d.peer_flag[i] = self.fabric.peer_ptr(r, self.eg_lay.offset(f"n2m_flag{lane}")) + 4 * self.ag_index
        w = self.lanes[lane]
        d.epoch, d.done_counter, d.status = ptr(w.epoch), ptr(w.done), ptr(self.status)
        d.trace = ptr(self.trace[lane]) if self.trace else None
        return d

    def dispatch(self, lane: int, x: torch.Tensor, topk_idx: torch.Tensor) -> None:
        """Push x [T,H] bf16 (rows of tokens routed to each expert GPU) and the top-k ids."""
        assert x.is_contiguous() and topk_idx.is_contiguous() and topk_idx.dtype == torch.int32
        if self.cfg.use_direct(x.shape[0]):
            dd = self._direct_desc[lane]
            dd.T = x.shape[0]
            check(lib().afd_dispatch_direct(ptr(x), ptr(topk_idx), C.byref(dd), cur_stream()), "dispatch_direct")
            return
        d = self._dispatch_desc[lane]
        d.x, d.topk_idx, d.T = ptr(x), ptr(topk_idx), x.shape[0]
        check(lib().afd_dispatch_push(C.byref(d), cur_stream()), "dispatch_push")

    def route_dispatch(self, lane: int, attn_out: torch.Tensor, residual: torch.Tensor, norm_w: torch.Tensor,
                       gate_w: torch.Tensor, gate_bias: Optional[torch.Tensor], x_out: torch.Tensor,
                       topk_idx: torch.Tensor, topk_w: torch.Tensor, *, scoring: str, renorm: bool, eps: float,
                       offset1: bool = False, route_scale: float = 1.0, local_schedule: Optional[ScheduleDesc] = None) -> bool:
        """One launch for: residual += attn_out; x = rmsnorm(residual); router; push to experts."""
        if self.cfg.use_direct(attn_out.shape[0]):
            r = RouteDirectDesc()
            C.memmove(C.byref(r.d), C.byref(self._direct_desc[lane]), C.sizeof(DirectDesc))
            r.d.T = attn_out.shape[0]
            r.attn_out, r.residual, r.norm_w = ptr(attn_out), ptr(residual), ptr(norm_w)
            r.gate_w, r.gate_bias = ptr(gate_w), ptr(gate_bias)
            r.x_out, r.topk_idx_out, r.topk_w_out = ptr(x_out), ptr(topk_idx), ptr(topk_w)
            r.E, r.gate_fp32 = gate_w.shape[0], int(gate_w.dtype == torch.float32)
            r.scoring, r.renorm, r.offset1 = (0 if scoring == "softmax" else 1), int(renorm), int(offset1)
            r.eps, r.route_scale = eps, route_scale
            r.tokens_per_cta, r.cluster = self.route_tokens_per_cta, self.route_cluster
            fused = local_schedule is not None and self.cfg.num_eg == 1 and self.cfg.num_ag == 1
            if fused:       # experts on this GPU, single source: the kernel's last CTA builds their tile schedule
                r.fuse_schedule = 1
                C.memmove(C.byref(r.sched), C.byref(local_schedule), C.sizeof(ScheduleDesc))
            check(lib().afd_ag_route_direct(C.byref(r), cur_stream()), "ag_route_direct")
            return fused
        r = RouteDispatchDesc()
        C.memmove(C.byref(r.d), C.byref(self._dispatch_desc[lane]), C.sizeof(DispatchDesc))
        r.d.T = attn_out.shape[0]
        r.attn_out, r.residual, r.norm_w = ptr(attn_out), ptr(residual), ptr(norm_w)
        r.gate_w, r.gate_bias = ptr(gate_w), ptr(gate_bias)
        r.x_out, r.topk_idx_out, r.topk_w_out = ptr(x_out), ptr(topk_idx), ptr(topk_w)
        r.E, r.gate_fp32 = gate_w.shape[0], int(gate_w.dtype == torch.float32)
        r.scoring, r.renorm, r.offset1 = (0 if scoring == "softmax" else 1), int(renorm), int(offset1)
        r.eps, r.route_scale = eps, route_scale
        check(lib().afd_ag_route_dispatch(C.byref(r), cur_stream()), "ag_route_dispatch")
        return False

    def combine_reduce(self, lane: int, topk_w: torch.Tensor, topk_idx: Optional[torch.Tensor], T: int,
                       scale: float = 1.0, extra: Optional[torch.Tensor] = None,
                       y: Optional[torch.Tensor] = None, residual: Optional[torch.Tensor] = None,
                       norm_w: Optional[torch.Tensor] = None, normed: Optional[torch.Tensor] = None,
                       eps: float = 1e-6, offset1: bool = False):
        """Wait for every expert GPU's M2N flag, then y[t] = scale * sum_k w[t,k] * combine[k][t]
        (+ extra). With residual/norm_w/normed also residual += y; normed = rmsnorm(residual)."""
        cfg, d = self.cfg, CombineDesc()
        w = self.lanes[lane]
        d.combine, d.topk_w, d.topk_idx = ptr(self.combine[lane]), ptr(topk_w), ptr(topk_idx)
        d.m2n_flag, d.epoch, d.done_counter = ptr(self.m2n_flag[lane]), ptr(w.epoch2), ptr(w.done2)
        d.T, d.H, d.K, d.combine_tokens, d.num_eg = T, cfg.hidden, cfg.topk, cfg.max_tokens, cfg.num_eg
        d.scale = scale
        if y is None and normed is None:
            y = torch.empty(T, cfg.hidden, dtype=torch.bfloat16, device=self.device)
        d.extra, d.y, d.residual, d.norm_w, d.normed = ptr(extra), ptr(y), ptr(residual), ptr(norm_w), ptr(normed)
        d.eps, d.offset1, d.timeout_ns, d.status = eps, int(offset1), self.timeout_ns, ptr(self.status)
        d.trace = ptr(self.trace[lane]) if self.trace else None
        if _SPLIT_WAIT and cfg.num_lanes > 1:     # with one lane nothing else runs that a resident spin could slow
            # the wait of the flags runs as one warp; the T-CTA reduction launches once they are set
            check(lib().afd_wait_flags_epoch(ptr(self.m2n_flag[lane]), cfg.num_eg, ptr(w.epoch2),
                                             C.c_ulonglong(self.timeout_ns), ptr(self.status), cur_stream()), "wait_flags")
        check(lib().afd_ag_combine(C.byref(d), cur_stream()), "ag_combine")
        return y if normed is None else normed


class EgMoeEndpoint:
    """Expert rank `eg_index`: wait + group + gather, SwiGLU grouped GEMM, down grouped GEMM
    with the M2N store epilogue."""

    def __init__(self, cfg: MoeCommConfig, fabric: Fabric, eg_index: int, ag_ranks: List[int],
                 device: torch.device, timeout_ns: int = DEFAULT_TIMEOUT_NS, grid: int = NUM_SMS,
                 status: Optional[torch.Tensor] = None):
        self.cfg, self.fabric, self.eg_index, self.ag_ranks, self.device = cfg, fabric, eg_index, ag_ranks, device
        self.timeout_ns, self.grid = timeout_ns, grid
        self.lay, self.ag_lay = eg_layout(cfg), ag_layout(cfg)
        self.status = status if status is not None else torch.zeros(1, dtype=torch.int32, device=device)
        self.lanes = [_LaneWords(device) for _ in range(cfg.num_lanes)]
        self.trace = ([torch.zeros(TRACE_LEN, 4, dtype=torch.int64, device=device) for _ in range(cfg.num_lanes)]
                      if _trace_enabled() else None)
        heap, L = fabric.heap, cfg.num_lanes
        xdt = torch.float8_e4m3fn if cfg.fp8 else torch.bfloat16
        self.recv_x = [heap.view(self.lay.offset(f"recv_x{l}"), (cfg.num_ag, cfg.max_tokens, cfg.hidden), xdt)
                       for l in range(L)]
        self.recv_scale = [heap.view(self.lay.offset(f"recv_scale{l}"),
                                     (cfg.num_ag, cfg.max_tokens, cfg.hidden // 128), torch.float32) for l in range(L)]
        self.recv_idx = [heap.view(self.lay.offset(f"recv_idx{l}"), (cfg.num_ag, cfg.max_tokens, cfg.topk),
                                   torch.int32) for l in range(L)]
        self.n2m_flag = [heap.view(self.lay.offset(f"n2m_flag{l}"), (cfg.num_ag,), torch.int32) for l in range(L)]
        R, I = cfg.pool_rows, cfg.intermediate
        # Pools are shared by the lanes: a lane's layer runs to completion on one stream.
        self.pool_x = torch.zeros(R, cfg.hidden, dtype=xdt, device=device)
        self.pool_xs = torch.ones(R, cfg.hidden // 128, dtype=torch.float32, device=device) if cfg.fp8 else None
        self.pool_h = torch.zeros(R, I, dtype=xdt, device=device)
        self.pool_hs = torch.ones(R, max(I // 128, 1), dtype=torch.float32, device=device) if cfg.fp8 else None
        self.row_meta = torch.zeros(R, dtype=torch.int32, device=device)
        self.tile_info = torch.zeros(cfg.max_tok_tiles, 4, dtype=torch.int32, device=device)
        self.counters = torch.zeros(4, dtype=torch.int32, device=device)
        self.expert_counts = torch.zeros(cfg.experts_per_eg, dtype=torch.int32, device=device)
        self.expert_base = eg_index * cfg.experts_per_eg
        self.experts_local = cfg.experts_per_eg
        if cfg.direct_tokens > 0:
            DR = cfg.direct_rows
            self.dpool_x = [heap.view(self.lay.offset(f"dpool_x{l}"), (DR, cfg.hidden), xdt) for l in range(L)]
            self.dpool_xs = [heap.view(self.lay.offset(f"dpool_scale{l}"), (DR, cfg.hidden // 128), torch.float32)
                             for l in range(L)] if cfg.fp8 else [None] * L
            self.dmeta = [heap.view(self.lay.offset(f"dmeta{l}"), (DR,), torch.int32) for l in range(L)]
            self.dcount = [heap.view(self.lay.offset(f"dcount{l}"), (cfg.experts_per_eg,), torch.int32) for l in range(L)]
            for c in self.dcount:
                c.zero_()
            self.dpool_h = torch.zeros(DR, I, dtype=xdt, device=device)
            self.dpool_hs = torch.ones(DR, max(I // 128, 1), dtype=torch.float32, device=device) if cfg.fp8 else None
            self.dtile_info = torch.zeros(cfg.experts_per_eg * (cfg.direct_cap // cfg.block_tok), 4, dtype=torch.int32, device=device)
        self.peer_combine = [[fabric.peer_ptr(r, self.ag_lay.offset(f"combine{l}")) for r in ag_ranks] for l in range(L)]
        self.peer_flag = [[fabric.peer_ptr(r, self.ag_lay.offset(f"m2n_flag{l}")) + 4 * eg_index for r in ag_ranks]
                          for l in range(L)]

    def group_gather(self, lane: int, T: int) -> None:
        cfg, d = self.cfg, GroupDesc()
        w = self.lanes[lane]
        d.recv_idx, d.n2m_flag, d.epoch = ptr(self.recv_idx[lane]), ptr(self.n2m_flag[lane]), ptr(w.epoch)
        d.A, d.T, d.K, d.recv_tokens = cfg.num_ag, T, cfg.topk, cfg.max_tokens
        d.expert_base, d.experts_local, d.block_tok = self.expert_base, self.experts_local, cfg.block_tok
        d.pool_rows, d.max_tok_tiles = cfg.pool_rows, cfg.max_tok_tiles
        d.row_meta, d.tile_info, d.counters = ptr(self.row_meta), ptr(self.tile_info), ptr(self.counters)
        d.expert_counts, d.timeout_ns, d.status = ptr(self.expert_counts), self.timeout_ns, ptr(self.status)
        d.recv_x, d.recv_scale = ptr(self.recv_x[lane]), ptr(self.recv_scale[lane]) if cfg.fp8 else None
        d.pool_x, d.pool_scale = ptr(self.pool_x), ptr(self.pool_xs)
        d.row_bytes, d.scale_per_row = cfg.row_bytes, cfg.hidden // 128
        d.trace = ptr(self.trace[lane]) if self.trace else None
        d.done_counter = ptr(w.done)
        if _SPLIT_WAIT and cfg.num_lanes > 1:
            check(lib().afd_wait_flags_epoch(ptr(self.n2m_flag[lane]), cfg.num_ag, ptr(w.epoch),
                                             C.c_ulonglong(self.timeout_ns), ptr(self.status), cur_stream()), "wait_flags")
        fused = cfg.num_ag * T * cfg.topk <= 8192 and cfg.block_tok <= 128      # one launch, else two
        check(lib().afd_eg_group_gather(C.byref(d), cur_stream()), "eg_group_gather_fused" if fused else "eg_group_gather")

    def flag_report(self) -> Dict[str, object]:
        """Per lane: the dispatch flags the attention ranks write here (see `flag_report`)."""
        return {f"lane{l}": flag_report(self.n2m_flag[l], self.lanes[l].epoch, self.ag_ranks) for l in range(self.cfg.num_lanes)}

    def run_layer(self, lane: int, T: int, w13: torch.Tensor, w2: torch.Tensor,
                  w13_scale: Optional[torch.Tensor] = None, w2_scale: Optional[torch.Tensor] = None,
                  scheduled: bool = False) -> None:
        """One MoE layer for one lane. w13: [E_local, 2I, H] gate/up interleaved (see
        ops.interleave_gate_up); w2: [E_local, H, I]. FP8 mode takes per-tile scales."""
        cfg = self.cfg
        if cfg.use_direct(T):
            return self._run_layer_direct(lane, w13, w2, w13_scale, w2_scale, scheduled)
        self.group_gather(lane, T)
        ntiles = self.counters[0:1]
        grouped_gemm(w=w13, x=self.pool_x, num_experts=self.experts_local, n_per_expert=2 * cfg.intermediate,
                     k=cfg.hidden, tile_info=self.tile_info, num_tok_tiles=ntiles, block_tok=cfg.block_tok,
                     epilogue=EPI_SWIGLU, out=None if cfg.fp8 else self.pool_h, out_ld=cfg.intermediate,
                     fp8=cfg.fp8, x_scale=self.pool_xs, w_scale=w13_scale,
                     out_q=self.pool_h if cfg.fp8 else None, out_scale=self.pool_hs,
                     status=self.status, grid=self.grid, l2_prefetch_bytes=L2_PREFETCH_BYTES)
        w = self.lanes[lane]
        grouped_gemm(w=w2, x=self.pool_h, num_experts=self.experts_local, n_per_expert=cfg.hidden,
                     k=cfg.intermediate, tile_info=self.tile_info, num_tok_tiles=ntiles,
                     block_tok=cfg.block_tok, epilogue=EPI_COMBINE, fp8=cfg.fp8, x_scale=self.pool_hs,
                     w_scale=w2_scale, row_meta=self.row_meta, peer_combine=self.peer_combine[lane],
                     peer_flag=self.peer_flag[lane], combine_tokens=cfg.max_tokens, hidden=cfg.hidden,
                     epoch=w.epoch2, done_counter=w.done2, status=self.status, grid=self.grid,
                     trace=self.trace[lane] if self.trace else None)


    def schedule_desc(self, lane: int) -> ScheduleDesc:
        cfg, w = self.cfg, self.lanes[lane]
        s = ScheduleDesc()
        s.n2m_flag, s.A, s.epoch, s.counts = ptr(self.n2m_flag[lane]), cfg.num_ag, ptr(w.epoch), ptr(self.dcount[lane])
        s.experts_local, s.cap, s.block_tok = self.experts_local, cfg.direct_cap, cfg.block_tok
        s.max_tok_tiles = self.dtile_info.shape[0]
        s.tile_info, s.counters, s.expert_counts = ptr(self.dtile_info), ptr(self.counters), ptr(self.expert_counts)
        s.timeout_ns, s.status = self.timeout_ns, ptr(self.status)
        s.trace = ptr(self.trace[lane]) if self.trace else None
        return s

    def _schedule(self, lane: int) -> None:
        """One warp: bounded wait for the sources' flags, slot counters -> tile schedule, counters reset."""
        check(lib().afd_eg_schedule(C.byref(self.schedule_desc(lane)), cur_stream()), "eg_schedule")

    def _run_layer_direct(self, lane: int, w13, w2, w13_scale, w2_scale, scheduled: bool = False) -> None:
        """The layer when the sources stored their rows straight into the expert stripes: one warp
        waits for the flags and turns the slot counters into the tile schedule, then the two GEMMs."""
        cfg, w = self.cfg, self.lanes[lane]
        if not scheduled:                       # else the (single, local) source's route kernel already did it
            self._schedule(lane)
        ntiles = self.counters[0:1]
        grouped_gemm(w=w13, x=self.dpool_x[lane], num_experts=self.experts_local, n_per_expert=2 * cfg.intermediate,
                     k=cfg.hidden, tile_info=self.dtile_info, num_tok_tiles=ntiles, block_tok=cfg.block_tok,
                     epilogue=EPI_SWIGLU, out=None if cfg.fp8 else self.dpool_h, out_ld=cfg.intermediate,
                     fp8=cfg.fp8, x_scale=self.dpool_xs[lane], w_scale=w13_scale,
                     out_q=self.dpool_h if cfg.fp8 else None, out_scale=self.dpool_hs,
                     status=self.status, grid=self.grid, l2_prefetch_bytes=L2_PREFETCH_BYTES)
        grouped_gemm(w=w2, x=self.dpool_h, num_experts=self.experts_local, n_per_expert=cfg.hidden,
                     k=cfg.intermediate, tile_info=self.dtile_info, num_tok_tiles=ntiles,
                     block_tok=cfg.block_tok, epilogue=EPI_COMBINE, fp8=cfg.fp8, x_scale=self.dpool_hs,
                     w_scale=w2_scale, row_meta=self.dmeta[lane], peer_combine=self.peer_combine[lane],
                     peer_flag=self.peer_flag[lane], combine_tokens=cfg.max_tokens, hidden=cfg.hidden,
                     epoch=w.epoch2, done_counter=w.done2, status=self.status, grid=self.grid,
                     trace=self.trace[lane] if self.trace else None)


def summarize_trace(trace: torch.Tensor, role: str, last: int = 256) -> dict:
    """Mean durations (microseconds) over the most recent `last` rounds of one lane's timeline.
    attention: wait = combine start -> flags seen (idle time waiting for the experts),
               reduce = flags seen -> combine end, round = dispatch released -> combine end,
               chain = combine end -> next dispatch released (median; the lane's own compute chain).
    expert   : wait = group start -> flags seen (idle time waiting for attention ranks),
               busy = flags seen -> down-projection flags released."""
    t = trace.cpu().numpy().astype("int64")
    rows = t[(t > 0).all(axis=1)] if role == "attention" else t[(t[:, [0, 1, 3]] > 0).all(axis=1)]
    rows = rows[rows[:, 0].argsort()][-last:]
    if len(rows) == 0:
        return {}
    us = lambda a: float(a.mean()) / 1e3  # noqa: E731
    if role == "attention":
        out = {"wait_us": us(rows[:, 2] - rows[:, 1]), "reduce_us": us(rows[:, 3] - rows[:, 2]),
               "round_trip_us": us(rows[:, 3] - rows[:, 0]), "rounds": len(rows)}
        # attention-side chain of the lane: combine end of one round -> dispatch released of the next
        # (qkv, norm + RoPE + store, attention, o_proj, route + dispatch, plus whatever the other
        # micro-batch put on the GPU in between); step boundaries (long gaps) are left out
        gaps = rows[1:, 0] - rows[:-1, 3]
        gaps = gaps[(gaps > 0) & (gaps < 5_000_000)]
        if len(gaps):
            import numpy as _np
            out["chain_us"] = float(_np.median(gaps)) / 1e3
        return out
    return {"wait_us": us(rows[:, 1] - rows[:, 0]), "busy_us": us(rows[:, 3] - rows[:, 1]), "rounds": len(rows)}


def check_status(status: torch.Tensor, what: str) -> None:
    """Raise if a kernel recorded a timeout / bounds / capacity code (host sync)."""
    code = int(status.item())
    if code != 0:
        names = {1: "mbarrier wait timed out", 2: "peer flag wait timed out",
                 3: "index out of bounds (access skipped)", 4: "capacity exceeded"}
        status.zero_()
        raise RuntimeError(f"{what}: device status {code} ({names.get(code, 'unknown')})")
