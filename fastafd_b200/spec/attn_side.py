"""Attention-side speculative decoding (EAGLE-3 style): verify step + draft proposal.

One verify step per request processes ``block`` tokens: the last committed token followed
by ``block - 1`` draft tokens. The target model runs the normal micro-batch pipeline with
``block`` tokens per request (paged attention in multi-token mode, causal inside the block);
the LM head gives the target's own choice at each of the positions; the longest draft prefix
that equals those choices is accepted and the target's next token is appended (greedy
verification is lossless: the output equals plain greedy decoding). The draft head then
writes its KV context for the accepted positions and proposes the next ``block - 1`` tokens,
all into the device-side token pool. The committed length of every request lives on the device
too, so a verify step takes only the table rows from the host: the whole step (target pipeline,
head + acceptance, draft chain) is one CUDA graph per bucket and the coordinator may queue the
next step before this one's acceptance has reached it.

The expert GPUs just see a wider decode bucket (bucket * block tokens per micro-batch).

Reference: python/minisgl/spec/attn_side.py (verify :91-136, greedy head :375-383, propose
:228-244,361-371), python/minisgl/spec/graph.py:234-322 (verify graphs),
python/minisgl/spec/device_inputs.py:79-116 (device-resident committed lengths), python/minisgl/spec/config.py:85-124 (acceptance rule, reply packing),
python/minisgl/afd_scheduler.py:516-552 (verify scheduled as a block-token extend).
"""
from __future__ import annotations

from typing import List, Optional

import numpy as np
import torch

from .. import ops
from ..models.transformer import AttnMeta
from ..protocol import AgStepPlan, AgStepReply
from ..reference import ops_ref as ref
from .eagle3 import Eagle3Config, Eagle3Draft


def simulated_accept(n_rows: int, block: int, mean_accept: float, rng: np.random.Generator) -> np.ndarray:
    """Emitted-token counts with a fixed mean in [1, block] (timing runs with a fixed acceptance
    instead of a trained draft head): each row emits floor(mean) or ceil(mean) tokens."""
    mean = min(max(mean_accept, 1.0), float(block))
    lo = int(np.floor(mean))
    p_hi = mean - lo
    n = lo + (rng.random(n_rows) < p_hi).astype(np.int32)
    return np.clip(n, 1, block).astype(np.int32)


class SpecRunner:
    """Bound to an AttentionWorker; owns the draft head and the verify step."""

    def __init__(self, worker, block: int, draft_path: str = "", seed: int = 0, sim_accept: float = 0.0):
        self.w, self.block, self.sim_accept = worker, block, sim_accept
        self.rng = np.random.default_rng(seed)
        cfg = worker.cfg
        # a published head brings its own sizes, vocabulary and auxiliary layers; a synthetic one follows the target
        self.dcfg = Eagle3Config.from_dir(draft_path, cfg) if draft_path else Eagle3Config.for_target(cfg)
        slots = worker.kv.num_pages * worker.kv.page_size
        self.draft = Eagle3Draft(self.dcfg, worker.device, worker.dtype, slots)
        if draft_path:
            tw = worker.model.w
            self.draft.load(draft_path, share_embedding=tw["model.embed_tokens.weight"],
                            share_lm_head=tw.get("lm_head.weight", tw["model.embed_tokens.weight"]))
        else:
            self.draft.init_random(seed, share_embedding=worker.model.w["model.embed_tokens.weight"])
        self.capture_layers = list(self.dcfg.target_layers)
        self.accept_hist = np.zeros(block + 1, np.int64)
        # committed KV length of every table row, on the device (the padding row stays at 0)
        self.committed = torch.zeros(worker.max_running + 1, dtype=torch.int32, device=worker.device)

    # ------------------------------------------------------------------ helpers
    def _meta(self, rows: torch.Tensor, first_pos: torch.Tensor, q_len: int) -> AttnMeta:
        w, ps = self.w, self.w.page_size
        B = rows.shape[0]
        pos = (first_pos[:, None] + torch.arange(q_len, device=rows.device, dtype=first_pos.dtype)[None]).reshape(-1)
        pt = w.page_table_all[rows]
        page = torch.gather(pt, 1, (pos.view(B, q_len) // ps).long()).reshape(-1)
        loc = (page * ps + pos % ps).to(torch.int32)
        return AttnMeta(positions=pos.to(torch.int32), out_loc=loc, page_table=pt, seq_lens=(first_pos + q_len).to(torch.int32),
                        q_len=q_len, state_slots=rows.to(torch.int32), status=w.status)

    def write_prefill_context(self, rows: torch.Tensor, starts: List[int], lens: List[int], ids: torch.Tensor,
                              aux: List[torch.Tensor], first_tokens: Optional[torch.Tensor], sample_mask) -> None:
        """Draft KV for the prompt chunk just prefilled: position p gets (token p+1, feature p).
        The chunk's last position needs the token after the chunk: the sampled first token when
        the prompt ended here, else it is left for the next chunk (only acceptance can suffer)."""
        feat = self.draft.fuse_features(aux)
        off, si = 0, 0
        for b, n in enumerate(lens):
            if n == 0:
                continue
            nxt = ids[off + 1:off + n]
            use = n - 1
            if sample_mask[b]:
                nxt = torch.cat([nxt, first_tokens[si:si + 1].to(ids.dtype)])
                use = n
                si += 1
            if use > 0:
                meta = self._meta(rows[b:b + 1], torch.tensor([starts[b]], device=rows.device, dtype=torch.int32), use)
                self.draft.layer(nxt[:use].contiguous(), feat[off:off + use].contiguous(), meta, self.w.page_size)
            off += n

    # ------------------------------------------------------------------ verify step
    def set_committed(self, rows: torch.Tensor, lengths: torch.Tensor) -> None:
        """Prefill finished for `rows`: their committed KV length (the first sampled token sits at
        that position of the token pool)."""
        self.committed[rows.long()] = lengths.to(torch.int32)

    def _body(self, bucket: int) -> None:
        """One verify step for every lane, on device state only: the committed length of every
        request lives in `self.committed` (device), so the step needs nothing from the host but the
        table rows, can be captured in a CUDA graph, and the next step can be queued before this
        one's acceptance is known to the host."""
        w, k, dev = self.w, self.block, self.w.device
        mbs = []
        for lane in range(w.num_mb):
            rows = w.bufs[lane].rows[:bucket]
            L = self.committed[rows]                                                 # committed KV length
            meta = self._meta(rows, L, k)
            meta.lane = lane
            ids = w.token_pool[rows[:, None], (L[:, None] + self._ar[None]).long()].reshape(-1).contiguous()
            mb = w.make_ctx(lane, ids, meta)
            mb.capture = {}
            mb.rows, mb.L = rows, L
            mbs.append(mb)
        w.pipeline(mbs, capture_layers=self.capture_layers)
        for lane, mb in enumerate(mbs):
            B, rows, L = bucket, mb.rows, mb.L
            logits = w.model.lm_head(w.full_tokens(mb.normed))
            target = ops.argmax(logits).view(B, k).to(torch.int64)
            drafts = mb.ids.view(B, k)[:, 1:].to(torch.int64)
            n, emitted = ref.greedy_accept(drafts, target)
            j = self._ar[None]
            if self.sim_accept > 0:
                # timing runs: a fixed mean acceptance from a pre-drawn table, one row per step
                step = (self.sim_step % self.sim_table.shape[0]).long().view(1)      # stays on the device (graph capture)
                n = self.sim_table.index_select(0, step)[0, lane, :B].reshape(B)
                emitted = torch.where(j < n[:, None], target, torch.full_like(target, -1))
            n = n.to(torch.int64)
            valid = j < n[:, None]
            # commit: pool[row, L+1+j] = emitted[j] for j < n (fixed shapes: the other positions keep
            # their value; they are overwritten by the new drafts below)
            pos = (L[:, None].long() + 1 + j)
            old = w.token_pool[rows[:, None], pos]
            w.token_pool[rows[:, None], pos] = torch.where(valid, emitted.to(torch.int32), old)
            # draft: context for positions L..L+k-1 (the ones past L+n-1 are overwritten later), then chain
            feat = self.draft.fuse_features([mb.capture[l] for l in self.capture_layers])
            nxt = torch.where(valid, emitted, torch.zeros_like(emitted)).to(torch.int32).reshape(-1).contiguous()
            h = self.draft.layer(nxt, feat, self._meta(rows, L, k), w.page_size).view(B, k, -1)
            last = h[torch.arange(B, device=dev), (n - 1).clamp(0, k - 1)]            # output at position L' - 1
            newL = L.long() + n                                                        # L' (bonus token sits at L')
            for i in range(k - 1):
                tok = self.draft.logits_to_tokens(last)                               # draft i+1 -> position L'+1+i
                w.token_pool[rows, newL + 1 + i] = tok
                if i + 1 < k - 1:
                    meta1 = self._meta(rows, (newL + i).to(torch.int32), 1)
                    last = self.draft.layer(tok.contiguous(), last.contiguous(), meta1, w.page_size)
            # padding rows (all the lane's dummy row) stay at length 0
            self.committed[rows] = torch.where(rows != w.dummy_row, newL, torch.zeros_like(newL)).to(torch.int32)
            self.out_tokens[lane][:B * k].copy_(emitted.to(torch.int32).reshape(-1))
            self.out_n[lane][:B].copy_(n.to(torch.int32))
        if self.sim_accept > 0:
            self.sim_step.add_(1)

    def _buffers(self) -> None:
        w, k, dev = self.w, self.block, self.w.device
        if getattr(self, "_ready", False):
            return
        from ..worker.attention_worker import RING

        self._ar = torch.arange(k, device=dev, dtype=torch.int32)
        self.out_tokens = [torch.zeros(w.cap * k, dtype=torch.int32, device=dev) for _ in range(w.num_mb)]
        self.out_n = [torch.zeros(w.cap, dtype=torch.int32, device=dev) for _ in range(w.num_mb)]
        self.sim_step = torch.zeros((), dtype=torch.int32, device=dev)
        if self.sim_accept > 0:
            tab = np.stack([simulated_accept(w.num_mb * w.cap, k, self.sim_accept, self.rng).reshape(w.num_mb, w.cap)
                            for _ in range(257)])
            self.sim_table = torch.from_numpy(tab.astype(np.int64)).to(dev)
        if w.cuda:
            self.host_tokens = [torch.zeros(RING, w.cap * k, dtype=torch.int32).pin_memory() for _ in range(w.num_mb)]
            self.host_n = [torch.zeros(RING, w.cap, dtype=torch.int32).pin_memory() for _ in range(w.num_mb)]
        else:
            self._host = [None] * RING
        self.graphs = {}
        self._ready = True

    def launch_verify(self, plan: AgStepPlan) -> None:
        """Queue one verify step: page grants, H2D of the rows, graph replay (or the eager body), D2H of
        the emitted tokens and counts into this step's ring slot."""
        from contextlib import nullcontext

        from ..worker.attention_worker import RING

        w, k, bucket = self.w, self.block, plan.bucket
        self._buffers()
        ctx = torch.cuda.stream(w.main_stream) if w.cuda else nullcontext()
        with ctx:
            w.apply_grants(plan)
            w._stage_decode(plan)
            if w.cuda and w.rt.use_cuda_graph:
                if bucket not in self.graphs:
                    for b in w.bufs:                      # warm-up and capture on padding rows only
                        b.rows.fill_(w.dummy_row)
                    self._body(bucket)
                    torch.cuda.synchronize(w.device)
                    g = torch.cuda.CUDAGraph()
                    with torch.cuda.graph(g, stream=w.main_stream, capture_error_mode="thread_local"):
                        self._body(bucket)
                    self.graphs[bucket] = g
                    w._stage_decode(plan)
                self.graphs[bucket].replay()
            else:
                self._body(bucket)
            slot = plan.step_id % RING
            if w.cuda:
                for lane in range(w.num_mb):
                    self.host_tokens[lane][slot, :bucket * k].copy_(self.out_tokens[lane][:bucket * k], non_blocking=True)
                    self.host_n[lane][slot, :bucket].copy_(self.out_n[lane][:bucket], non_blocking=True)
                w.status_host[slot, 0:1].copy_(w.status, non_blocking=True)
                w.d2h_events[slot].record()
            else:
                self._host[slot] = ([t[:bucket * k].numpy().copy() for t in self.out_tokens],
                                    [t[:bucket].numpy().copy() for t in self.out_n])

    def finish_verify(self, plan: AgStepPlan) -> AgStepReply:
        from ..worker.attention_worker import RING

        w, k, bucket = self.w, self.block, plan.bucket
        slot = plan.step_id % RING
        if w.cuda:
            w.d2h_events[slot].synchronize()
            toks = [self.host_tokens[l][slot, :bucket * k].numpy().copy() for l in range(w.num_mb)]
            ns = [self.host_n[l][slot, :bucket].numpy().copy() for l in range(w.num_mb)]
            status = int(w.status_host[slot, 0])
        else:
            toks, ns = self._host[slot]
            status = w.read_status()
        for mbp, nn in zip(plan.mbs, ns):
            for v in nn[:mbp.num_real]:
                self.accept_hist[int(v)] += 1
        return AgStepReply(step_id=plan.step_id, rank=w.rank, next_tokens=np.concatenate(toks).astype(np.int32),
                           accepted=np.concatenate(ns).astype(np.int32), status=status)

    def run_verify(self, plan: AgStepPlan) -> AgStepReply:
        self.launch_verify(plan)
        return self.finish_verify(plan)

    def mean_accept(self) -> float:
        tot = self.accept_hist.sum()
        return float((self.accept_hist * np.arange(len(self.accept_hist))).sum() / tot) if tot else 0.0
