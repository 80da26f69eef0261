"""Attention tensor-parallel collectives fused with their GEMMs over the fabric.

Two operations replace the NCCL calls of the per-layer hot path of a TP lane (the rest -
embedding, LM head, cross-head norm statistics - stays on the wrapped communicator):

* ``oproj_reduce_scatter(lane, o, w)``: the row-parallel o_proj GEMM (tcgen05 kernel) stores its
  partial output rows from the epilogue straight into the peer that owns each token
  (``[tp][tokens][H]`` per lane), tile by tile while the GEMM is still running; the owner then
  sums the tp partials in fp32 after a bounded wait on the tp flags (``ag_combine_kernel``).
* ``all_gather(lane, x)``: every rank stores its token rows into all peers' gather buffers and
  releases a flag; the consumer waits for the tp flags and reads its *local* buffer, so the qkv
  GEMM that follows never touches peer memory.

Buffers are reused every layer: a rank's next reduce-scatter into a peer is ordered after that
peer's all-gather release of the same layer (which follows its read of the previous partials),
and the next all-gather after the peer's reduce-scatter release; the NCCL collectives at the
step boundary separate steps.

The default for a TP lane on CUDA; ``FASTAFD_TP_FUSED=0`` sends the same two operations through the
NCCL communicator. Measured on B200 (Qwen3-30B-A3B shapes): TP-2 + EP-2 on 4 GPUs 9.78 ms/step fused
against 10.10 ms over NCCL; TP-4 + EP-4 on 8 GPUs 7.85 ms/step fused.

Reference: python/minisgl/layers/linear.py:418-447 (o_proj + all-reduce),
python/minisgl/distributed/impl.py:28-85.
"""
from __future__ import annotations

import ctypes as C
from typing import List

import torch

from ..ops import EPI_COMBINE, dense_tile_schedule, grouped_gemm
from ..ops._lib import CombineDesc, check, cur_stream, lib, ptr
from .comm import TpComm
from .fabric import Fabric, Layout

MAX_TP = 8


class _GatherDesc(C.Structure):
    _fields_ = [("x", C.c_void_p), ("peer_buf", C.c_void_p * MAX_TP), ("peer_flag", C.c_void_p * MAX_TP),
                ("tp", C.c_int), ("my_index", C.c_int), ("T_local", C.c_int), ("H", C.c_int),
                ("epoch", C.c_void_p), ("done_counter", C.c_void_p), ("status", C.c_void_p)]


def tp_layout(tp: int, num_lanes: int, max_tokens_local: int, hidden: int) -> Layout:
    """Regions of one attention rank's heap used by the fused TP collectives."""
    lay = Layout()
    for lane in range(num_lanes):
        lay.add(f"tp_rs{lane}", tp * max_tokens_local * hidden * 2)        # partial o_proj rows per source
        lay.add(f"tp_rs_flag{lane}", 4 * tp)
        lay.add(f"tp_ag{lane}", tp * max_tokens_local * hidden * 2)        # gathered token rows
        lay.add(f"tp_ag_flag{lane}", 4 * tp)
    return lay


class TpFusedComm(TpComm):
    """`base` serves the collectives that are not fused. `ranks` are the fabric ranks of the TP
    group in TP order; `heap_base` is where `tp_layout` starts inside every rank's heap."""

    def __init__(self, base: TpComm, fabric: Fabric, ranks: List[int], my_index: int, heap_base: int,
                 num_lanes: int, max_tokens_local: int, hidden: int, device: torch.device,
                 timeout_ns: int = int(20e9), block_tok: int = 0, status=None):
        assert len(ranks) <= MAX_TP and hidden % 128 == 0
        self.base, self.fabric, self.ranks, self.rank, self.size = base, fabric, list(ranks), my_index, len(ranks)
        self.cap, self.H, self.device, self.timeout_ns = max_tokens_local, hidden, device, timeout_ns
        self.block_tok = block_tok
        self.lay = tp_layout(self.size, num_lanes, max_tokens_local, hidden)
        self.off = heap_base
        heap = fabric.heap
        self.status = status if status is not None else torch.zeros(1, dtype=torch.int32, device=device)
        tp = self.size
        self.rs_buf = [heap.view(heap_base + self.lay.offset(f"tp_rs{l}"), (tp, max_tokens_local, hidden), torch.bfloat16)
                       for l in range(num_lanes)]
        self.rs_flag = [heap.view(heap_base + self.lay.offset(f"tp_rs_flag{l}"), (tp,), torch.int32) for l in range(num_lanes)]
        self.ag_buf = [heap.view(heap_base + self.lay.offset(f"tp_ag{l}"), (tp * max_tokens_local, hidden), torch.bfloat16)
                       for l in range(num_lanes)]
        self.ag_flag = [heap.view(heap_base + self.lay.offset(f"tp_ag_flag{l}"), (tp,), torch.int32) for l in range(num_lanes)]
        # device words per lane: [rs publish epoch, rs done, rs expect epoch, rs combine done,
        #                         ag publish epoch, ag done, ag expect epoch, unused]
        self.words = []
        for _ in range(num_lanes):
            w = torch.zeros(8, dtype=torch.int32, device=device)
            w[0] = w[2] = w[4] = w[6] = 1
            self.words.append(w)
        self.ones = torch.ones(max_tokens_local, tp, dtype=torch.float32, device=device)
        self._sched = {}
        self._meta = {}

    # ---- collectives that stay on the wrapped communicator ---------------------------------
    def all_reduce(self, x):
        return self.base.all_reduce(x)

    def all_gather_last_dim(self, x):
        return self.base.all_gather_last_dim(x)

    def reduce_scatter(self, x):
        return self.base.reduce_scatter(x)

    def all_gather(self, x, lane: int = -1):
        if lane < 0 or not x.is_cuda or x.shape[0] > self.cap or x.dtype != torch.bfloat16 or x.shape[1] != self.H:
            return self.base.all_gather(x)
        return self.all_gather_rows(lane, x)

    # ---- fused paths ------------------------------------------------------------------------
    def _peer(self, r: int, name: str) -> int:
        return self.fabric.peer_ptr(self.ranks[r], self.off + self.lay.offset(name))

    def gather_push(self, lane: int, x: torch.Tensor) -> None:
        """Store x [Tl,H] into every rank's gather buffer of the lane and release the flags."""
        Tl = x.shape[0]
        w = self.words[lane]
        d = _GatherDesc()
        d.x = ptr(x.contiguous())
        for p in range(self.size):
            d.peer_buf[p] = self._peer(p, f"tp_ag{lane}")
            d.peer_flag[p] = self._peer(p, f"tp_ag_flag{lane}") + 4 * self.rank
        d.tp, d.my_index, d.T_local, d.H = self.size, self.rank, Tl, self.H
        d.epoch, d.done_counter, d.status = ptr(w[4:5]), ptr(w[5:6]), ptr(self.status)
        check(lib().afd_tp_allgather_push(C.byref(d), cur_stream()), "tp_allgather_push")

    def gather_wait(self, lane: int, Tl: int) -> torch.Tensor:
        """Bounded wait for every rank's rows; returns [tp*Tl, H], a view of this rank's gather
        buffer that stays valid until the lane's next all-gather."""
        w = self.words[lane]
        check(lib().afd_tp_allgather_wait(ptr(self.ag_flag[lane]), self.size, ptr(w[6:7]),
                                          C.c_ulonglong(self.timeout_ns), ptr(self.status), cur_stream()),
              "tp_allgather_wait")
        return self.ag_buf[lane][:self.size * Tl]

    def all_gather_rows(self, lane: int, x: torch.Tensor) -> torch.Tensor:
        self.gather_push(lane, x)
        return self.gather_wait(lane, x.shape[0])

    def can_fuse_oproj(self, T: int, k_local: int) -> bool:
        return T % self.size == 0 and T // self.size <= self.cap and k_local % 64 == 0 and T < 65536

    def oproj_push(self, lane: int, o: torch.Tensor, w_o: torch.Tensor) -> None:
        """The row-parallel GEMM o [T, K_local] @ w_o [H, K_local].T whose epilogue stores each
        partial row into the rank that owns the token (slot = this rank) and, from the last CTA,
        releases this rank's flag on every peer."""
        T, K = o.shape
        tp, Tl = self.size, T // self.size
        # token tiles of at most 64: the peer-store epilogue has been exercised with 16/32/64-token tiles only
        bt = self.block_tok or (16 if T <= 16 else 32 if T <= 32 else 64)
        key = (T, bt)
        if key not in self._sched:
            self._sched[key] = dense_tile_schedule(T, bt, self.device)
            r = torch.arange(T, dtype=torch.int64)
            meta = ((r // Tl) << 24) | (self.rank << 16) | (r % Tl)       # owner | slot of this source | row
            self._meta[key] = meta.to(torch.int32).to(self.device)
        info, n = self._sched[key]
        wd = self.words[lane]
        grouped_gemm(w=w_o, x=o, num_experts=1, n_per_expert=self.H, k=K, tile_info=info, num_tok_tiles=n,
                     block_tok=bt, epilogue=EPI_COMBINE, row_meta=self._meta[key],
                     peer_combine=[self._peer(p, f"tp_rs{lane}") for p in range(tp)],
                     peer_flag=[self._peer(p, f"tp_rs_flag{lane}") + 4 * self.rank for p in range(tp)],
                     combine_tokens=self.cap, hidden=self.H, epoch=wd[0:1], done_counter=wd[1:2], status=self.status)

    def reduce_wait(self, lane: int, Tl: int) -> torch.Tensor:
        """Bounded wait for the tp partials of this rank's rows, then their fp32 sum: [Tl, H]."""
        tp, wd = self.size, self.words[lane]
        c = CombineDesc()
        y = torch.empty(Tl, self.H, dtype=torch.bfloat16, device=self.device)
        c.combine, c.topk_w, c.topk_idx = ptr(self.rs_buf[lane]), ptr(self.ones), None
        c.m2n_flag, c.epoch, c.done_counter = ptr(self.rs_flag[lane]), ptr(wd[2:3]), ptr(wd[3:4])
        c.T, c.H, c.K, c.combine_tokens, c.num_eg = Tl, self.H, tp, self.cap, tp
        c.scale = 1.0
        c.extra, c.y, c.residual, c.norm_w, c.normed = None, ptr(y), None, None, None
        c.eps, c.offset1, c.timeout_ns, c.status, c.trace = 1e-6, 0, self.timeout_ns, ptr(self.status), None
        # one-warp wait first, so that the Tl reduction CTAs are not resident while peers still compute
        check(lib().afd_wait_flags_epoch(ptr(self.rs_flag[lane]), tp, ptr(wd[2:3]), C.c_ulonglong(self.timeout_ns),
                                         ptr(self.status), cur_stream()), "wait_flags")
        check(lib().afd_ag_combine(C.byref(c), cur_stream()), "ag_combine")
        return y

    def oproj_reduce_scatter(self, lane: int, o: torch.Tensor, w_o: torch.Tensor) -> torch.Tensor:
        """Rows of sum over ranks of o @ w_o.T that this rank owns: [T/tp, H]."""
        self.oproj_push(lane, o, w_o)
        return self.reduce_wait(lane, o.shape[0] // self.size)
