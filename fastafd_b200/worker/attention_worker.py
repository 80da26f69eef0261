"""Attention-GPU worker: request-local state, the micro-batch ping-pong pipeline, CUDA
graph capture per decode bucket, sampling and device-side token write-back.

Per step the host sends only request rows, sequence lengths and page grants (from pinned
staging buffers); input tokens of decode steps are read on the device from the token pool,
where the previous step's sampler wrote them, so consecutive decode steps need no host
round trip on the critical path.

Pipeline (2 micro-batches A, B; `main` = compute stream, one lane stream per micro-batch):

    main : compute(0,A) compute(0,B) | compute(1,A) compute(1,B) | ...
    laneA:            dispatch(0,A) ....... combine(0,A)  dispatch(1,A) ...
    laneB:                         dispatch(0,B) ....... combine(0,B) ...

compute(l) = attention block + post-attention norm + router (+ shared expert);
combine(l) waits for the expert GPUs, reduces the top-k rows and already applies the next
block's input norm. While lane A is away at the experts, `main` runs B's attention.

Reference: python/minisgl/afd_attention_worker.py:709-955 (_run_ag_pipeline_body),
:304-648 (AfdAgDecodeGraphRunner), python/minisgl/afd_attention_runtime.py:99-483
(token pool, materialize_ag_plan, page grants), python/minisgl/cuda_graph_utils.py.
"""
from __future__ import annotations

import os
import time
from contextlib import contextmanager, nullcontext
from dataclasses import dataclass, field
from typing import Dict, List, Optional

import numpy as np
import torch

from .. import ops
from ..config import ModelConfig, RuntimeConfig
from ..models.transformer import AttentionStage, AttnMeta, GDNStatePool, KVPool
from ..protocol import AgStepPlan, AgStepReply
from ..utils.trace import nvtx_range
from .moe_client import MoeClient


RING = 3   # pinned staging slots: up to two steps in flight plus the one being written


@dataclass
class _MbBuffers:
    """Static device buffers of one micro-batch (capacity = largest decode bucket)."""
    rows: torch.Tensor
    seq_lens: torch.Tensor
    positions: torch.Tensor
    out_loc: torch.Tensor
    ids: torch.Tensor
    page_table: torch.Tensor
    x_moe: torch.Tensor
    topk_idx: torch.Tensor
    topk_w: torch.Tensor
    normed: torch.Tensor
    residual: torch.Tensor
    next_tokens: torch.Tensor
    logits: Optional[torch.Tensor] = None
    host_in: Optional[torch.Tensor] = None      # pinned [RING, 2, cap] int32: rows, seq_lens
    host_out: Optional[torch.Tensor] = None     # pinned [RING, cap] int32
    workspace: Optional[torch.Tensor] = None


@dataclass
class _MbCtx:
    """View of the buffers for the token count of the current step."""
    lane: int
    T: int                      # tokens of the micro-batch (attention works on all of them)
    ids: torch.Tensor
    meta: AttnMeta
    x_moe: torch.Tensor
    topk_idx: torch.Tensor
    topk_w: torch.Tensor
    normed: torch.Tensor
    residual: torch.Tensor
    extra: Optional[torch.Tensor] = None
    pad_from: int = 0
    Tl: int = 0                 # tokens of the residual stream held by this TP rank (T / tp)
    capture: Optional[dict] = None
    keep: list = field(default_factory=list)


def determine_num_pages(cfg: ModelConfig, rt: RuntimeConfig, device: torch.device, kv_heads: int,
                        elem: int = 2) -> int:
    """Pages that fit in `memory_ratio` of the free device memory once the weights are resident,
    capped by what max_running_requests x max_seq_len can use. Explicit rt.num_pages wins.
    Reference: python/minisgl/afd_attention_worker.py:144-203."""
    if rt.num_pages > 0:
        return rt.num_pages
    want = rt.max_running_requests * (((rt.max_seq_len or cfg.max_position) + rt.page_size - 1) // rt.page_size) + 1
    if device.type != "cuda":
        return min(want, 4096)
    per_page = KVPool.bytes_per_page(cfg, rt.page_size, kv_heads, elem)
    free, _total = torch.cuda.mem_get_info(device)
    budget = int(free * rt.memory_ratio) - (2 << 30)
    return max(2, min(budget // max(per_page, 1), want))


class AttentionWorker:
    def __init__(self, cfg: ModelConfig, rt: RuntimeConfig, device, client: MoeClient, *, num_pages: int = 0,
                 tp_rank: int = 0, tp_size: int = 1, tp_comm=None, dtype=None, rank: int = 0,
                 max_bucket: Optional[int] = None, weight_init=None, status: Optional[torch.Tensor] = None,
                 dp_lane: int = 0):
        self.cfg, self.rt, self.device, self.client, self.rank = cfg, rt, torch.device(device), client, rank
        self.cuda = self.device.type == "cuda"
        self.dp_lane = dp_lane          # data-parallel lane this rank serves (all its TP ranks share it)
        self.dtype = dtype or (torch.bfloat16 if self.cuda else torch.float32)
        from ..parallel.comm import TpComm

        self.tp = tp_comm if tp_comm is not None else TpComm()
        assert self.tp.size == tp_size, "TP communicator size does not match attn_tp"
        self.model = AttentionStage(cfg, self.device, self.dtype, tp_rank, tp_size, tp_comm)
        if weight_init is not None:
            weight_init(self.model)          # weights first: the KV pool is sized from what is left
        self.num_mb, self.page_size = rt.num_mb, rt.page_size
        self.max_seq_len = rt.max_seq_len or cfg.max_position
        self.max_pages = (self.max_seq_len + self.page_size - 1) // self.page_size
        self.max_running = rt.max_running_requests
        self.dummy_row = self.max_running
        # The recurrent state of the linear-attention layers first (its size is fixed by max_running; for a large
        # hybrid model it is tens of GB), then the KV pool from what is left: a page is priced as the pool
        # allocates it, against the memory that is free once everything else is resident.
        self.gdn = GDNStatePool(cfg, self.max_running + 1, self.device, self.dtype, tp_size) if cfg.num_linear_layers else None
        self.num_pages = num_pages = num_pages or determine_num_pages(
            cfg, rt, self.device, self.model.hkv, 2 if self.cuda else 4)
        self.kv = KVPool(cfg, num_pages, self.page_size, self.model.hkv, self.device, self.dtype)
        self.token_pool = torch.zeros(self.max_running + 1, self.max_seq_len + 8, dtype=torch.int32, device=self.device)
        self.page_table_all = torch.zeros(self.max_running + 1, self.max_pages, dtype=torch.int32, device=self.device)
        self.page_table_host = np.zeros((self.max_running + 1, self.max_pages), np.int32)
        self.status = status if status is not None else torch.zeros(1, dtype=torch.int32, device=self.device)
        self.model.status = self.status if self.cuda else None
        self.cap = max_bucket or max(rt.cuda_graph_max_bs, 1)
        self.bufs = [self._make_bufs(self.cap) for _ in range(self.num_mb)]
        self.graphs: Dict[int, "torch.cuda.CUDAGraph"] = {}
        self.kernels_per_step: Dict[int, int] = {}
        self.spec = None          # SpecRunner when speculative decoding is on
        # validation hook: a list that receives (rows, kv lengths, fp32 logits) of every sampled row of
        # every eager step, so that logits can be compared with a reference forward (never set in serving)
        self.logit_tap: Optional[list] = None
        # Every micro-batch's whole chain on its own stream (FASTAFD_LANE_STREAMS=1): the attention kernel of
        # one micro-batch (HBM-bound) then overlaps the projections and the route kernel of the other
        # (latency-bound), and a late combine of one no longer holds back the other. Only for a
        # disaggregated attention rank without TP: a colocated expert stage shares its buffers between
        # the micro-batches, and TP collectives must be issued in one order on one stream.
        self.lane_parallel = (self.cuda and self.num_mb > 1 and self.tp.size == 1
                              and getattr(client, "colocated", None) is None
                              and os.environ.get("FASTAFD_LANE_STREAMS", "0") == "1")
        self._in_lane_mode = False
        if self.cuda:
            self.main_stream = torch.cuda.Stream(self.device)
            self.lane_streams = [torch.cuda.Stream(self.device) for _ in range(self.num_mb)]
            self.d2h_events = [torch.cuda.Event() for _ in range(RING)]
            self.status_host = torch.zeros(RING, 4, dtype=torch.int32).pin_memory()

    # ------------------------------------------------------------------ buffers
    def _make_bufs(self, cap: int) -> _MbBuffers:
        c, dev, dt = self.cfg, self.device, self.dtype
        K = max(c.num_experts_per_tok, 1)
        z = lambda *s, d=dt: torch.zeros(*s, dtype=d, device=dev)  # noqa: E731
        b = _MbBuffers(
            rows=z(cap, d=torch.int64), seq_lens=z(cap, d=torch.int32), positions=z(cap, d=torch.int32),
            out_loc=z(cap, d=torch.int32), ids=z(cap, d=torch.int32), page_table=z(cap, self.max_pages, d=torch.int32),
            x_moe=z(cap, c.hidden_size), topk_idx=z(cap, K, d=torch.int32), topk_w=z(cap, K, d=torch.float32),
            normed=z(cap, c.hidden_size), residual=z(cap, c.hidden_size), next_tokens=z(cap, d=torch.int32))
        b.rows.fill_(self.dummy_row)
        b.seq_lens.fill_(1)
        if self.cuda:
            b.host_in = torch.zeros(RING, 2, cap, dtype=torch.int32).pin_memory()
            b.host_out = torch.zeros(RING, cap, dtype=torch.int32).pin_memory()
        return b

    # ------------------------------------------------------------------ plan application
    def apply_grants(self, plan: AgStepPlan) -> None:
        n = len(plan.grant_rows)
        if n == 0:
            return
        self.page_table_host[plan.grant_rows, plan.grant_slots] = plan.grant_pages
        if self.cuda:
            g = torch.from_numpy(np.stack([plan.grant_rows, plan.grant_slots, plan.grant_pages]).astype(np.int64)).pin_memory()
            gd = g.to(self.device, non_blocking=True)
            self.page_table_all.index_put_((gd[0], gd[1]), gd[2].to(torch.int32))
        else:
            self.page_table_all[torch.from_numpy(plan.grant_rows).long(), torch.from_numpy(plan.grant_slots).long()] = \
                torch.from_numpy(plan.grant_pages)

    def d2h_bytes(self, plan: AgStepPlan) -> int:
        return sum(len(mb.rows) * 4 for mb in plan.mbs) + 4 * (1 + len(self.client.status_tensors()))

    def h2d_bytes(self, plan: AgStepPlan) -> int:
        n = sum(2 * len(mb.rows) * 4 for mb in plan.mbs) + 3 * 8 * len(plan.grant_rows)
        n += sum(mb.input_ids.nbytes for mb in plan.mbs if mb.input_ids is not None)
        return n

    # ------------------------------------------------------------------ pipeline
    @contextmanager
    def _on_lane(self, lane: int, after_main: bool = True):
        """Run the enclosed launches on the lane's stream, ordered after what `main` has queued
        so far; the caller orders `main` after the lane later with `_join_lane`."""
        if not self.cuda or self.num_mb == 1 or self._in_lane_mode:
            # one micro-batch: nothing to overlap with, so everything stays on the main stream and
            # consecutive kernels keep their programmatic (early-launch) dependencies. Lane mode: the
            # caller already runs the micro-batch's whole chain on its stream.
            yield
            return
        s = self.lane_streams[lane]
        if after_main:
            s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            yield

    def _join_lane(self, lane: int) -> None:
        if self.cuda and self.num_mb > 1 and not self._in_lane_mode:
            torch.cuda.current_stream().wait_stream(self.lane_streams[lane])

    def _next_norm_weight(self, layer: int) -> torch.Tensor:
        if layer + 1 < self.cfg.num_layers:
            return self.model.w[f"model.layers.{layer + 1}.input_layernorm.weight"]
        return self.model.w["model.norm.weight"]

    def _compute(self, layer: int, mb: _MbCtx) -> None:
        """Attention block + post-attention norm + router for one layer of one micro-batch; for
        MoE layers ends with the dispatch on the lane stream, for dense layers with the local MLP."""
        m, c = self.model, self.cfg
        moe = c.is_moe_layer(layer)
        fused = (moe and self.cuda and not mb.meta.is_prefill and c.n_group == 1
                 and self.client.can_fuse_route(mb.Tl, c.num_experts, c.hidden_size))
        with nvtx_range(f"AFD_AG_Attn_L{layer}_mb{mb.lane}"):
            x_in = self.tp.all_gather(mb.normed, lane=mb.lane) if self.tp.size > 1 else mb.normed
            attn_out = m.attention(layer, x_in, mb.meta, self.kv, self.gdn, reduce="scatter")
            if fused:
                p = f"model.layers.{layer}."
                self.client.route_dispatch(
                    mb.lane, layer, attn_out, mb.residual, m.w[p + "post_attention_layernorm.weight"],
                    m.w[p + "mlp.gate.weight"], m.w.get(p + "mlp.gate.e_score_correction_bias"), mb.x_moe,
                    mb.topk_idx, mb.topk_w, scoring=c.scoring, renorm=c.norm_topk_prob, eps=c.rms_eps,
                    offset1=c.norm_offset1)
                x = mb.x_moe
            else:
                x = m.post_attn_norm(layer, attn_out, mb.residual, out=mb.x_moe if moe else None)
        if moe and fused:
            mb.extra = self._local_mlp(layer, x)
            mb.keep += [attn_out, mb.extra]
            with self._on_lane(mb.lane):
                self.client.after_dispatch(mb.lane, layer, mb.Tl)
        elif moe:
            m.route(layer, x, out_idx=mb.topk_idx, out_w=mb.topk_w)
            first_pad = mb.pad_from - self.tp.rank * mb.Tl      # padding tokens are routed nowhere
            if mb.meta.is_prefill and first_pad < mb.Tl:
                mb.topk_idx[max(first_pad, 0):] = -1
            mb.extra = self._local_mlp(layer, x)
            mb.keep += [attn_out, mb.extra]
            with self._on_lane(mb.lane):
                with nvtx_range(f"AFD_AG_Dispatch_L{layer}_mb{mb.lane}"):
                    self.client.dispatch(mb.lane, layer, mb.x_moe, mb.topk_idx, mb.topk_w)
        else:
            y = self._local_mlp(layer, x)
            normed = ops.add_rmsnorm(y, mb.residual, self._next_norm_weight(layer), c.rms_eps, c.norm_offset1)
            mb.normed.copy_(normed)
            mb.keep += [attn_out, x, y, normed]

    def _local_mlp(self, layer: int, x: torch.Tensor):
        """Dense MLP / shared expert on the token shard: gather the tokens, run the TP-sharded
        MLP, scatter the partial sums back."""
        if self.tp.size == 1:
            return self.model.local_mlp(layer, x)
        c = self.cfg
        if c.is_moe_layer(layer) and c.num_shared_experts == 0:
            return None
        return self.model.local_mlp(layer, self.tp.all_gather(x), reduce="scatter")

    def _combine(self, layer: int, mb: _MbCtx) -> None:
        c = self.cfg
        if not c.is_moe_layer(layer):
            return
        with self._on_lane(mb.lane, after_main=False):
            with nvtx_range(f"AFD_AG_Combine_L{layer}_mb{mb.lane}"):
                self.client.combine(mb.lane, layer, mb.Tl, mb.topk_w, mb.topk_idx, mb.residual,
                                    self._next_norm_weight(layer), c.rms_eps, extra=mb.extra,
                                    scale=c.routed_scaling_factor, offset1=c.norm_offset1, normed_out=mb.normed)
        self._join_lane(mb.lane)

    def pipeline(self, mbs: List[_MbCtx], capture_layers=()) -> None:
        self._pipeline(mbs, capture_layers)

    def make_ctx(self, lane: int, ids: torch.Tensor, meta: AttnMeta, pad_from: Optional[int] = None) -> _MbCtx:
        """Micro-batch context with freshly allocated buffers (eager prefill / verify steps)."""
        c, dev, T = self.cfg, self.device, ids.shape[0]
        assert T % self.tp.size == 0, "token count must be a multiple of the attention TP size"
        Tl = T // self.tp.size
        K = max(c.num_experts_per_tok, 1)
        mb = _MbCtx(lane=lane, T=T, ids=ids, meta=meta,
                    x_moe=torch.zeros(Tl, c.hidden_size, dtype=self.dtype, device=dev),
                    topk_idx=torch.zeros(Tl, K, dtype=torch.int32, device=dev),
                    topk_w=torch.zeros(Tl, K, dtype=torch.float32, device=dev),
                    normed=torch.zeros(Tl, c.hidden_size, dtype=self.dtype, device=dev),
                    residual=torch.zeros(Tl, c.hidden_size, dtype=self.dtype, device=dev))
        mb.pad_from = T if pad_from is None else pad_from
        mb.Tl = Tl
        return mb

    def _pipeline(self, mbs: List[_MbCtx], capture_layers=()) -> None:
        """All layers for all micro-batches; on return mb.normed holds the final-norm output.
        `capture_layers`: hidden states (residual stream after that layer) kept in mb.capture
        for the speculative draft head."""
        m, L = self.model, self.cfg.num_layers
        lanes = self.lane_parallel and not mbs[0].meta.is_prefill and not capture_layers
        main = torch.cuda.current_stream() if lanes else None
        if lanes:
            for mb in mbs:
                self.lane_streams[mb.lane].wait_stream(main)
            self._in_lane_mode = True

        def on(mb):          # the stream that carries this micro-batch's chain
            return torch.cuda.stream(self.lane_streams[mb.lane]) if lanes else nullcontext()

        try:
            for mb in mbs:
                with on(mb):
                    h = m.embed(mb.ids, scatter=True)
                    mb.residual.copy_(h)
                    n0 = ops.rmsnorm(h, m.w["model.layers.0.input_layernorm.weight"], self.cfg.rms_eps, self.cfg.norm_offset1)
                    mb.normed.copy_(n0)
                    mb.keep += [h, n0]
                    self._compute(0, mb)
            for l in range(L):
                for mb in mbs:
                    with on(mb):
                        self._combine(l, mb)
                        if l in capture_layers:
                            mb.capture[l] = mb.residual.clone()
                        if l + 1 < L:
                            self._compute(l + 1, mb)
        finally:
            if lanes:
                self._in_lane_mode = False
                for mb in mbs:
                    main.wait_stream(self.lane_streams[mb.lane])

    # ------------------------------------------------------------------ decode
    def _decode_ctx(self, lane: int, bucket: int, q_len: int = 1) -> _MbCtx:
        b = self.bufs[lane]
        T = bucket * q_len
        meta = AttnMeta(positions=b.positions[:T], out_loc=b.out_loc[:T], page_table=b.page_table[:bucket],
                        seq_lens=b.seq_lens[:bucket], q_len=q_len, lane=lane, state_slots=b.rows[:bucket].to(torch.int32) if self.gdn else None,
                        status=self.status)
        if self.cuda:
            max_kv = self.max_seq_len
            m_tiles = (self.model.hq // self.model.hkv * q_len + 15) // 16
            meta.splits = self.decode_splits if hasattr(self, "decode_splits") else ops.pick_attn_splits(
                bucket, self.model.hkv, m_tiles, max_kv, self.cfg.head_dim)
            if meta.splits > 1:
                if b.workspace is None:
                    b.workspace = ops.decode_attn_workspace(self.cap, self.model.hq, self.model.hkv, q_len,
                                                            self.cfg.head_dim, 32, self.device)
                meta.workspace = b.workspace
        assert T % self.tp.size == 0, "decode bucket must be a multiple of the attention TP size"
        Tl = T // self.tp.size
        mb = _MbCtx(lane=lane, T=T, ids=b.ids[:T], meta=meta, x_moe=b.x_moe[:Tl], topk_idx=b.topk_idx[:Tl],
                    topk_w=b.topk_w[:Tl], normed=b.normed[:Tl], residual=b.residual[:Tl])
        mb.pad_from = T
        mb.Tl = Tl
        return mb

    def _prepare_decode_inputs(self, lane: int, bucket: int) -> None:
        """From (rows, seq_lens): gather the page-table rows, positions, KV slots and the input
        token of every request out of device state."""
        b, ps = self.bufs[lane], self.page_size
        rows, seq = b.rows[:bucket], b.seq_lens[:bucket]
        pos = seq - 1
        b.positions[:bucket].copy_(pos)
        torch.index_select(self.page_table_all, 0, rows, out=b.page_table[:bucket])
        page = torch.gather(b.page_table[:bucket], 1, (pos // ps).long()[:, None])[:, 0]
        b.out_loc[:bucket].copy_(page * ps + pos % ps)
        b.ids[:bucket].copy_(self.token_pool[rows, pos.long()])

    def _sample_and_writeback(self, lane: int, mb: _MbCtx, bucket: int) -> None:
        self._sample_from_logits(lane, self.model.lm_head(self.full_tokens(mb.normed)), bucket)

    def _sample_all(self, mbs: List[_MbCtx], bucket: int) -> None:
        """LM head and greedy sampling of every micro-batch of a decode step. The vocabulary projection
        is a weight stream (its rows outnumber the tokens by three orders of magnitude), so the
        micro-batches go through it together: one pass over the matrix instead of one per micro-batch."""
        if len(mbs) == 1:
            return self._sample_and_writeback(0, mbs[0], bucket)
        xs = [self.full_tokens(mb.normed) for mb in mbs]
        logits = self.model.lm_head(torch.cat(xs, 0))
        off = 0
        for lane, x in enumerate(xs):
            self._sample_from_logits(lane, logits[off:off + x.shape[0]], bucket)
            off += x.shape[0]

    def _sample_from_logits(self, lane: int, logits: torch.Tensor, bucket: int) -> None:
        b = self.bufs[lane]
        b.logits = logits
        if self.logit_tap is not None and not (self.cuda and torch.cuda.is_current_stream_capturing()):
            self.logit_tap.append((b.rows[:bucket].cpu().clone(), b.seq_lens[:bucket].cpu().clone(), logits[:bucket].float().cpu().clone()))
        ops.argmax(logits, out=b.next_tokens[:bucket]) if self.cuda else b.next_tokens[:bucket].copy_(ops.argmax(logits))
        self.token_pool[b.rows[:bucket], b.seq_lens[:bucket].long()] = b.next_tokens[:bucket]

    def full_tokens(self, x_local: torch.Tensor) -> torch.Tensor:
        """Token-sharded rows of this TP rank -> all rows of the micro-batch."""
        return self.tp.all_gather(x_local) if self.tp.size > 1 else x_local

    def _decode_body(self, bucket: int) -> None:
        mbs = []
        for lane in range(self.num_mb):
            self._prepare_decode_inputs(lane, bucket)
            mbs.append(self._decode_ctx(lane, bucket))
        self._pipeline(mbs)
        self._sample_all(mbs, bucket)
        if self.model.cad is not None:
            self.model.cad.end_step()          # core-attention disaggregation: the epoch bump closes the step
        self._last_mbs = mbs

    def cad_serve_step(self, plan: AgStepPlan, server) -> None:
        """Attention-GPU side of a core-attention-disaggregated decode step: this process holds the KV
        cache and the page table, takes the same plan as the model GPU, and serves every (layer,
        micro-batch) hop in program order (`server`: cad.gpu.CadAttentionServer bound to this
        worker's KV pool)."""
        bucket = plan.bucket
        with torch.cuda.stream(self.main_stream):
            self.apply_grants(plan)
            self._stage_decode(plan)
            for lane in range(self.num_mb):
                self._prepare_decode_inputs(lane, bucket)
                b = self.bufs[lane]
                server.n_rows[lane] = bucket
                server.out_loc[lane], server.seq_lens[lane], server.page_table[lane] = b.out_loc, b.seq_lens, b.page_table[:bucket]
            for layer in range(self.cfg.num_layers):
                if self.cfg.layer_type(layer) != "full":
                    continue
                for lane in range(self.num_mb):
                    server.serve(layer, lane)
            server.end_step()

    def capture_decode_graph(self, bucket: int) -> None:
        """Warm up eagerly (sets kernel attributes, primes allocators), then capture the whole
        multi-stream decode step for this bucket."""
        assert self.cuda
        for b in self.bufs:          # warm up on padding rows only: no request state is touched
            b.rows.fill_(self.dummy_row)
            b.seq_lens.fill_(1)
        with torch.cuda.stream(self.main_stream):
            self._decode_body(bucket)
        torch.cuda.synchronize(self.device)
        from ..ops._lib import LAUNCHES

        g = torch.cuda.CUDAGraph()
        c0 = LAUNCHES["count"]
        with torch.cuda.graph(g, stream=self.main_stream, capture_error_mode="thread_local"):
            self._decode_body(bucket)
        self.kernels_per_step[bucket] = LAUNCHES["count"] - c0     # library kernels in one replay
        self.graphs[bucket] = g

    def _stage_decode(self, plan: AgStepPlan) -> None:
        slot = plan.step_id % RING
        for lane, mbp in enumerate(plan.mbs):
            b, n = self.bufs[lane], len(mbp.rows)
            if self.cuda:
                b.host_in[slot, 0, :n] = torch.from_numpy(mbp.rows)
                b.host_in[slot, 1, :n] = torch.from_numpy(mbp.seq_lens)
                b.rows[:n].copy_(b.host_in[slot, 0, :n], non_blocking=True)
                b.seq_lens[:n].copy_(b.host_in[slot, 1, :n], non_blocking=True)
            else:
                b.rows[:n] = torch.from_numpy(mbp.rows).long()
                b.seq_lens[:n] = torch.from_numpy(mbp.seq_lens)

    def launch_decode(self, plan: AgStepPlan) -> None:
        """Queue one decode step (H2D of the plan, graph replay or eager body, D2H of tokens)."""
        if plan.phase == "verify":
            return self.spec.launch_verify(plan)
        bucket = plan.bucket
        ctx = torch.cuda.stream(self.main_stream) if self.cuda else nullcontext()
        with ctx:
            self.apply_grants(plan)
            self._stage_decode(plan)
            if self.cuda and self.rt.use_cuda_graph:
                if bucket not in self.graphs:
                    self.capture_decode_graph(bucket)
                    self._stage_decode(plan)
                self.graphs[bucket].replay()
            else:
                from ..ops._lib import LAUNCHES

                c0 = LAUNCHES["count"]
                self._decode_body(bucket)
                self.kernels_per_step[bucket] = LAUNCHES["count"] - c0
            if plan.temperatures is not None:
                self._resample(plan)
            if self.cuda:
                slot = plan.step_id % RING
                for lane in range(self.num_mb):
                    b = self.bufs[lane]
                    b.host_out[slot, :bucket].copy_(b.next_tokens[:bucket], non_blocking=True)
                words = [self.status] + self.client.status_tensors()
                if getattr(self.tp, "status", None) is not None:
                    words.append(self.tp.status)
                for i, st in enumerate(words[:self.status_host.shape[1]]):
                    self.status_host[slot, i:i + 1].copy_(st, non_blocking=True)
                self.d2h_events[slot].record()
            else:
                # the host path runs a step to completion here; keep its tokens per ring slot, since
                # the next step may be launched (and overwrite next_tokens) before this one is finished
                if not hasattr(self, "_host_tokens"):
                    self._host_tokens = [None] * RING
                self._host_tokens[plan.step_id % RING] = np.concatenate(
                    [self.bufs[l].next_tokens[:bucket].numpy().copy() for l in range(self.num_mb)])

    def finish_decode(self, plan: AgStepPlan) -> AgStepReply:
        if plan.phase == "verify":
            return self.spec.finish_verify(plan)
        bucket = plan.bucket
        if self.cuda:
            slot = plan.step_id % RING
            self.d2h_events[slot].synchronize()
            toks = np.concatenate([self.bufs[l].host_out[slot, :bucket].numpy().copy() for l in range(self.num_mb)])
            status = int(self.status_host[slot].max())
        else:
            toks = self._host_tokens[plan.step_id % RING]
            status = self.read_status()
        return AgStepReply(step_id=plan.step_id, rank=self.rank, next_tokens=toks.astype(np.int32), status=status)

    def sampling_generator(self, step_id: int, mb: int) -> torch.Generator:
        """Random stream of one (step, micro-batch): a function of the configured seed, the DP lane,
        the step id and the micro-batch only - the same on every tensor-parallel rank of the lane (they
        must sample the same tokens) and reproducible from `--seed`, whatever else drew random numbers."""
        g = torch.Generator(device=self.device)
        g.manual_seed((int(self.rt.seed) * 1000003 + self.dp_lane * 7919 + mb) * 2654435761 % (1 << 62) + int(step_id))
        return g

    def _resample(self, plan: AgStepPlan) -> None:
        off = 0
        for lane in range(self.num_mb):
            b, n = self.bufs[lane], plan.bucket
            t = torch.from_numpy(plan.temperatures[off:off + n]).to(self.device)
            if bool((t > 0).any()):
                toks = ops.sample(b.logits, t, torch.from_numpy(plan.top_ks[off:off + n]).to(self.device),
                                  torch.from_numpy(plan.top_ps[off:off + n]).to(self.device),
                                  generator=self.sampling_generator(plan.step_id, lane))
                b.next_tokens[:n].copy_(toks)
                self.token_pool[b.rows[:n], b.seq_lens[:n].long()] = b.next_tokens[:n]
            off += n

    # ------------------------------------------------------------------ prefill
    def run_prefill(self, plan: AgStepPlan, mb_tokens: List[int]) -> AgStepReply:
        """Eager chunked prefill. Each micro-batch is padded to mb_tokens[m] tokens per dispatch
        source (= per TP rank; the count the expert GPUs expect from every source this step);
        padding tokens are routed nowhere."""
        ctx = torch.cuda.stream(self.main_stream) if self.cuda else nullcontext()
        dev, ps = self.device, self.page_size
        with ctx:
            self.apply_grants(plan)
            mbs: List[_MbCtx] = []
            for lane, mbp in enumerate(plan.mbs):
                T_real, T = int(mbp.extend_lens.sum()) if len(mbp.extend_lens) else 0, mb_tokens[lane] * self.tp.size
                pos = np.zeros(T, np.int32)
                loc = np.full(T, -1, np.int32)
                ids = np.zeros(T, np.int32)
                off = 0
                for r, (row, n, sl) in enumerate(zip(mbp.rows, mbp.extend_lens, mbp.seq_lens)):
                    p = np.arange(sl - n, sl, dtype=np.int32)
                    pos[off:off + n] = p
                    loc[off:off + n] = self.page_table_host[row, p // ps] * ps + p % ps
                    off += n
                ids[:T_real] = mbp.input_ids
                B = len(mbp.rows)
                rows_t = torch.from_numpy(mbp.rows.astype(np.int64)).to(dev)
                meta = AttnMeta(positions=torch.from_numpy(pos).to(dev), out_loc=torch.from_numpy(loc).to(dev),
                                page_table=torch.from_numpy(self.page_table_host[mbp.rows]).to(dev) if B else
                                torch.zeros(0, self.max_pages, dtype=torch.int32, device=dev),
                                seq_lens=torch.from_numpy(mbp.seq_lens).to(dev), is_prefill=True,
                                prefill_lens=[int(n) for n in mbp.extend_lens],
                                state_slots=rows_t.to(torch.int32), status=self.status, lane=lane)
                mb = self.make_ctx(lane, torch.from_numpy(ids).to(dev), meta)
                mb.pad_from = T_real
                if self.spec is not None:
                    mb.capture = {}
                mbs.append(mb)
            self._pipeline(mbs, self.spec.capture_layers if self.spec is not None else ())
            out = []
            for lane, (mb, mbp) in enumerate(zip(mbs, plan.mbs)):
                B = len(mbp.rows)
                toks = np.full(B, -1, np.int32)
                if B and mbp.sample_rows.any():
                    last = np.cumsum(mbp.extend_lens) - 1
                    sel = torch.from_numpy(last[mbp.sample_rows]).long().to(dev)
                    logits = self.model.lm_head(self.full_tokens(mb.normed)[sel])
                    t = ops.argmax(logits)
                    if plan.temperatures is not None:
                        base = sum(len(p.rows) for p in plan.mbs[:lane])
                        mask = mbp.sample_rows
                        temps = torch.from_numpy(plan.temperatures[base:base + B][mask]).to(dev)
                        if bool((temps > 0).any()):
                            t = ops.sample(logits, temps, torch.from_numpy(plan.top_ks[base:base + B][mask]).to(dev),
                                           torch.from_numpy(plan.top_ps[base:base + B][mask]).to(dev),
                                           generator=self.sampling_generator(plan.step_id, lane))
                    rows_s = torch.from_numpy(mbp.rows[mbp.sample_rows].astype(np.int64)).to(dev)
                    lens_s = torch.from_numpy(mbp.seq_lens[mbp.sample_rows].astype(np.int64)).to(dev)
                    self.token_pool[rows_s, lens_s] = t.to(torch.int32)
                    if self.spec is not None:
                        self.spec.set_committed(rows_s, lens_s)
                    if self.logit_tap is not None:
                        self.logit_tap.append((rows_s.cpu().clone(), lens_s.cpu().clone(), logits.float().cpu().clone()))
                    toks[mbp.sample_rows] = t.cpu().numpy()
                else:
                    t = None
                if self.spec is not None and B:
                    T_real = int(mbp.extend_lens.sum())
                    self.spec.write_prefill_context(
                        torch.from_numpy(mbp.rows.astype(np.int64)).to(dev), [int(x) for x in (mbp.seq_lens - mbp.extend_lens)],
                        [int(n) for n in mbp.extend_lens], mb.ids[:T_real],
                        [mb.capture[l][:T_real] for l in self.spec.capture_layers], t, mbp.sample_rows)
                out.append(toks)
            if self.cuda:
                torch.cuda.current_stream().synchronize()
        return AgStepReply(step_id=plan.step_id, rank=self.rank,
                           next_tokens=np.concatenate(out) if out else np.zeros(0, np.int32), status=self.read_status())

    # ------------------------------------------------------------------ misc
    def run_step(self, plan: AgStepPlan, mb_tokens: Optional[List[int]] = None) -> AgStepReply:
        t0 = time.perf_counter()
        if plan.phase == "prefill":
            tp = self.tp.size
            reply = self.run_prefill(plan, mb_tokens or [(mb.num_tokens + tp - 1) // tp for mb in plan.mbs])
        elif plan.phase == "verify":
            reply = self.spec.run_verify(plan)
        else:
            self.launch_decode(plan)
            reply = self.finish_decode(plan)
        reply.step_ms = (time.perf_counter() - t0) * 1e3
        return reply

    def read_status(self) -> int:
        code = int(self.status.item()) if self.status is not None else 0
        for s in self.client.status_tensors():
            code = code or int(s.item())
        tp_status = getattr(self.tp, "status", None)       # fused TP collectives keep their own word
        if tp_status is not None:
            code = code or int(tp_status.item())
        return code
