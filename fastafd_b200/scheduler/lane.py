"""Per-lane CPU scheduler of the AFD coordinator.

One instance per attention DP lane. It owns the lane's request table (rows of the worker's
token pool / page table), the page ledger, chunked prefill, decode batching with bucket
padding balanced over micro-batches, explicit page grants, and the bookkeeping that lets the
coordinator plan decode step N+1 before the tokens of step N are known.

Reference: python/minisgl/afd_scheduler.py:420-1013 (CentralizedAfdDpScheduler:
schedule_step :613, dummy_decode_step :656, complete_results :684, _pad_and_split_batch :839,
_balanced_decode_padded_reqs :868, page_grants :942), python/minisgl/scheduler/prefill.py:23-171.
"""
from __future__ import annotations

from collections import deque
from dataclasses import dataclass, field
from typing import Deque, Dict, List, Optional, Sequence, Tuple

import numpy as np

from ..core import Req, SamplingParams
from ..protocol import AgStepPlan, MicroBatchPlan
from .buckets import balanced_split, per_mb_real, split_prefill
from .cache import NaivePageLedger, OutOfPages, make_page_cache


class AdmissionError(RuntimeError):
    """A request can never be admitted (larger than the lane's whole capacity)."""


@dataclass
class _ReqState:
    req: Req
    planned_len: int = 0          # KV length after every step planned so far
    planned_out: int = 0          # output tokens planned (incl. in-flight)
    inflight: int = 0             # planned steps whose results are still outstanding
    prefix_handle: object = None
    reserved_pages: int = 0
    dead: bool = False            # finished; waiting for in-flight steps to drain


@dataclass
class StepRecord:
    """What a planned step contained, needed to interpret the worker's reply."""
    step_id: int
    phase: str
    # per micro-batch: list of (uid or -1 for padding, emits_token)
    slots: List[List[Tuple[int, bool]]] = field(default_factory=list)


class LaneScheduler:
    def __init__(self, lane: int, *, num_pages: int, page_size: int, max_running: int, max_seq_len: int,
                 num_mb: int = 2, max_batched_tokens: int = 8192, max_comm_tokens: int = 2048,
                 cache_type: str = "naive", eos_token_ids: Sequence[int] = (), spec_block: int = 0,
                 spec_pending: int = 1):
        self.lane, self.page_size, self.max_running, self.max_seq_len = lane, page_size, max_running, max_seq_len
        self.num_mb, self.max_batched_tokens, self.max_comm_tokens = num_mb, max_batched_tokens, max_comm_tokens
        self.cache: NaivePageLedger = make_page_cache(cache_type, num_pages, page_size)
        self.eos = set(int(e) for e in eos_token_ids)
        self.spec_block = spec_block
        # Verify steps are planned before the acceptance of the steps in flight is known, so a
        # request's planned length is an upper bound that runs ahead of its committed length by up to
        # one block per step in flight (plus the block being planned): that much KV is reserved.
        self.spec_slack = spec_block * (max(spec_pending, 1) + 1) if spec_block > 1 else 0
        self.max_pages_per_req = (max_seq_len + page_size - 1) // page_size
        self.dummy_row = max_running                    # extra row owned by padding requests
        self.waiting: Deque[Req] = deque()
        self.states: Dict[int, _ReqState] = {}          # uid -> state (admitted requests)
        self.free_rows: List[int] = list(range(max_running - 1, -1, -1))
        self.reserved_pages = 0
        self.records: Dict[int, StepRecord] = {}
        self._pending_free_rows: List[int] = []
        self._carry_grants: List[Tuple[int, int, int]] = []     # grants made outside a plan
        from ..env import ENV
        self.page_audit = bool(ENV.PAGE_AUDIT.value)

    # ------------------------------------------------------------------ admission
    def add_req(self, uid: int, input_ids: Sequence[int], sampling: SamplingParams) -> None:
        total = len(input_ids) + sampling.max_tokens + self.spec_slack
        if len(input_ids) == 0:
            raise AdmissionError(f"request {uid} has an empty prompt")
        if total > self.max_seq_len:
            raise AdmissionError(f"request {uid} needs {total} tokens > max_seq_len {self.max_seq_len}")
        if self.cache.pages_for(total) > self.cache.num_pages - 1:
            raise AdmissionError(f"request {uid} needs more KV pages than the lane has")
        self.waiting.append(Req(uid=uid, input_ids=list(input_ids), sampling=sampling, lane=self.lane))

    def add_prefilled(self, uid: int, prompt_len: int, sampling: SamplingParams, first_token: int = 0) -> Req:
        """Admit a request whose prompt KV is already in the cache (synthetic benchmark state,
        or a request migrated from a prefill instance): rows and pages are assigned now and the
        page grants travel with the next plan."""
        if not self.free_rows:
            raise AdmissionError("no free request row")
        req = Req(uid=uid, input_ids=[0] * prompt_len, sampling=sampling, lane=self.lane)
        req.table_idx = self.free_rows.pop()
        need = self.cache.pages_for(req.max_total_len + self.spec_slack)
        if self.reserved_pages + need > self.cache.num_pages - 1:
            self.free_rows.append(req.table_idx)
            raise AdmissionError(f"request {uid} needs {need} pages; lane has {self.cache.num_pages - 1 - self.reserved_pages}")
        st = _ReqState(req, planned_len=prompt_len, planned_out=1, reserved_pages=need)
        req.cached_len = prompt_len
        req.output_ids = [first_token]
        self.reserved_pages += need
        self.states[uid] = st
        self._grow_pages(st, prompt_len + 1, self._carry_grants)
        return req

    def abort(self, uid: int) -> None:
        for r in list(self.waiting):
            if r.uid == uid:
                self.waiting.remove(r)
                return
        st = self.states.get(uid)
        if st is not None and not st.dead:
            st.req.finished = True
            self._retire(st)

    @property
    def load(self) -> int:
        return len(self.waiting) + sum(1 for s in self.states.values() if not s.dead)

    def prefix_hit_len(self, input_ids: Sequence[int]) -> int:
        pages, handle = self.cache.match_prefix(input_ids)
        for node in handle or []:
            node.ref -= 1
        return len(pages) * self.page_size

    def _try_admit(self) -> bool:
        if not self.waiting or not self.free_rows:
            return False
        req = self.waiting[0]
        shared, handle = self.cache.match_prefix(req.input_ids)
        need = self.cache.pages_for(req.max_total_len + self.spec_slack) - len(shared)
        if self.reserved_pages + need > self.cache.num_pages - 1:
            if handle:
                for n in handle:
                    n.ref -= 1
            return False
        self.waiting.popleft()
        req.table_idx = self.free_rows.pop()
        req.pages = [int(p) for p in shared]
        req.cached_len = req.prefix_hit = len(shared) * self.page_size
        st = _ReqState(req, planned_len=req.cached_len, prefix_handle=handle, reserved_pages=need)
        self.reserved_pages += need
        self.states[req.uid] = st
        return True

    # ------------------------------------------------------------------ phase queries
    def has_prefill(self) -> bool:
        while self._try_admit():
            pass
        return any((not s.dead) and s.planned_len < s.req.prompt_len for s in self.states.values())

    def decodable(self) -> List[_ReqState]:
        return [s for s in self.states.values()
                if not s.dead and s.planned_len >= s.req.prompt_len and s.planned_out < s.req.sampling.max_tokens
                and (self.spec_block <= 1 or s.planned_len + self.spec_block <= s.req.max_total_len + self.spec_slack)]

    def decode_real(self) -> int:
        return len(self.decodable())

    def idle(self) -> bool:
        return not self.waiting and all(s.dead for s in self.states.values())

    def check_admission_stall(self) -> None:
        """Nothing runs, nothing is in flight, yet a request waits: it can never be admitted."""
        if self.waiting and not self.states:
            req = self.waiting[0]
            raise AdmissionError(
                f"lane {self.lane}: request {req.uid} (prompt {req.prompt_len}, max_tokens {req.sampling.max_tokens}) "
                f"cannot be admitted: {len(self.free_rows)} free rows, {self.cache.free_pages} free pages")

    # ------------------------------------------------------------------ planning
    def _grow_pages(self, st: _ReqState, new_len: int, grants: List[Tuple[int, int, int]]) -> None:
        have = len(st.req.pages)
        need = self.cache.pages_for(new_len)
        if need > have:
            pages = self.cache.allocate(need - have)
            for i, p in enumerate(pages):
                grants.append((st.req.table_idx, have + i, int(p)))
            st.req.pages.extend(int(p) for p in pages)

    def _shared_prefix_grants(self, st: _ReqState, grants: List[Tuple[int, int, int]]) -> None:
        """First time a request with a prefix hit is planned: its shared pages must be written
        into its page-table row too."""
        if st.req.prefix_hit and st.planned_len == st.req.prefix_hit and not getattr(st, "_prefix_granted", False):
            for i, p in enumerate(st.req.pages):
                grants.append((st.req.table_idx, i, int(p)))
            st._prefix_granted = True

    def _finish_plan(self, step_id: int, phase: str, bucket: int, mbs: List[MicroBatchPlan],
                     grants: List[Tuple[int, int, int]], record: StepRecord,
                     sampling_rows: List[Optional[_ReqState]]) -> AgStepPlan:
        g = np.asarray(self._carry_grants + grants, dtype=np.int32).reshape(-1, 3)
        self._carry_grants = []
        plan = AgStepPlan(step_id=step_id, phase=phase, bucket=bucket, mbs=mbs,
                          grant_rows=g[:, 0].copy(), grant_slots=g[:, 1].copy(), grant_pages=g[:, 2].copy(),
                          free_rows=np.asarray(self._pending_free_rows, dtype=np.int32), spec_block=self.spec_block)
        self._pending_free_rows = []
        if any(s is not None and not s.req.sampling.is_greedy for s in sampling_rows):
            plan.temperatures = np.asarray([0.0 if s is None else s.req.sampling.temperature for s in sampling_rows], np.float32)
            plan.top_ks = np.asarray([-1 if s is None else s.req.sampling.top_k for s in sampling_rows], np.int32)
            plan.top_ps = np.asarray([1.0 if s is None else s.req.sampling.top_p for s in sampling_rows], np.float32)
        self.records[step_id] = record
        if self.page_audit:
            self.audit_pages()
        return plan

    def schedule_prefill(self, step_id: int) -> AgStepPlan:
        """Chunked prefill: up to max_batched_tokens new tokens this step (and at most
        max_comm_tokens per micro-batch), oldest requests first."""
        while self._try_admit():
            pass
        budget = min(self.max_batched_tokens, self.max_comm_tokens * self.num_mb)
        chosen: List[Tuple[_ReqState, int]] = []
        grants: List[Tuple[int, int, int]] = []
        for st in self.states.values():
            if st.dead or st.planned_len >= st.req.prompt_len or budget <= 0:
                continue
            n = min(st.req.prompt_len - st.planned_len, budget, self.max_comm_tokens)
            try:
                self._shared_prefix_grants(st, grants)
                self._grow_pages(st, st.planned_len + n, grants)
            except OutOfPages:
                break
            chosen.append((st, n))
            budget -= n
        ranges = split_prefill([n for _, n in chosen], self.num_mb)
        # a micro-batch may not exceed the comm capacity: move overflow to later steps
        mbs, record, sampling_rows = [], StepRecord(step_id, "prefill"), []
        for (a, b) in ranges:
            part = chosen[a:b]
            tok = 0
            kept: List[Tuple[_ReqState, int]] = []
            for st, n in part:
                if tok + n > self.max_comm_tokens:
                    n = self.max_comm_tokens - tok
                if n <= 0:
                    continue
                kept.append((st, n))
                tok += n
            rows = np.asarray([st.req.table_idx for st, _ in kept], np.int32)
            ext = np.asarray([n for _, n in kept], np.int32)
            seq = np.asarray([st.planned_len + n for st, n in kept], np.int32)
            ids = [st.req.input_ids[st.planned_len:st.planned_len + n] for st, n in kept]
            flat = np.asarray([t for chunk in ids for t in chunk], np.int32)
            done = np.asarray([st.planned_len + n >= st.req.prompt_len for st, n in kept], bool)
            mbs.append(MicroBatchPlan(rows=rows, seq_lens=seq, num_real=len(kept), input_ids=flat, extend_lens=ext,
                                      sample_rows=done))
            slots = []
            for (st, n), d in zip(kept, done):
                st.planned_len += n
                st.inflight += 1
                if d:
                    st.planned_out += 1
                slots.append((st.req.uid, bool(d)))
                sampling_rows.append(st)
            record.slots.append(slots)
        return self._finish_plan(step_id, "prefill", 0, mbs, grants, record, sampling_rows)

    def schedule_decode(self, step_id: int, bucket: int, tokens_per_req: int = 1) -> AgStepPlan:
        """One decode (or `tokens_per_req`-token verify) step over every decodable request, padded
        to `bucket` rows per micro-batch with the dummy row, real requests spread evenly."""
        reqs = self.decodable()
        if per_mb_real(len(reqs), self.num_mb) > bucket and reqs:
            raise ValueError(f"bucket {bucket} too small for {len(reqs)} requests over {self.num_mb} micro-batches")
        split = balanced_split(len(reqs), self.num_mb)
        grants: List[Tuple[int, int, int]] = []
        mbs, record, sampling_rows = [], StepRecord(step_id, "decode" if tokens_per_req == 1 else "verify"), []
        pos = 0
        for m in range(self.num_mb):
            part = reqs[pos:pos + split[m]]
            pos += split[m]
            rows = np.full(bucket, self.dummy_row, np.int32)
            seq = np.full(bucket, tokens_per_req, np.int32)
            slots: List[Tuple[int, bool]] = []
            ps = self.page_size
            for i, st in enumerate(part):
                if (st.planned_len + tokens_per_req + ps - 1) // ps > len(st.req.pages):   # a new page only every ps tokens
                    self._grow_pages(st, st.planned_len + tokens_per_req, grants)
                st.planned_len += tokens_per_req
                st.planned_out += 1 if tokens_per_req == 1 else 0
                st.inflight += 1
                rows[i] = st.req.table_idx
                seq[i] = st.planned_len
                slots.append((st.req.uid, True))
            slots += [(-1, False)] * (bucket - len(part))
            sampling_rows += list(part) + [None] * (bucket - len(part))
            mbs.append(MicroBatchPlan(rows=rows, seq_lens=seq, num_real=len(part)))
            record.slots.append(slots)
        return self._finish_plan(step_id, record.phase, bucket, mbs, grants, record, sampling_rows)

    def shadow_decode(self, tokens_per_req: int = 1) -> int:
        """Advance this lane by one decode step without planning it: only the counters that decide
        how many requests are still decoding move (no pages, no plan, no record). For a process
        that does not serve this lane but must know its size to agree on the step's bucket.
        Returns the number of requests that took part."""
        n = 0
        for st in self.states.values():
            if not st.dead and st.planned_len >= st.req.prompt_len and st.planned_out < st.req.sampling.max_tokens:
                if tokens_per_req == 1:      # a verify step's progress depends on acceptance, known to its own rank only
                    st.planned_len += 1
                    st.planned_out += 1
                n += 1
        return n

    def dummy_step(self, step_id: int, phase: str, bucket: int, prefill_tokens: Sequence[int] = ()) -> AgStepPlan:
        """A lane with nothing to do still takes part in every step (N2M / M2N involve all ranks)."""
        mbs, record = [], StepRecord(step_id, phase)
        for m in range(self.num_mb):
            if phase == "prefill":
                mbs.append(MicroBatchPlan(rows=np.zeros(0, np.int32), seq_lens=np.zeros(0, np.int32), num_real=0,
                                          input_ids=np.zeros(0, np.int32), extend_lens=np.zeros(0, np.int32),
                                          sample_rows=np.zeros(0, bool)))
                record.slots.append([])
            else:
                mbs.append(MicroBatchPlan(rows=np.full(bucket, self.dummy_row, np.int32),
                                          seq_lens=np.full(bucket, self.spec_block if phase == "verify" else 1, np.int32),
                                          num_real=0))
                record.slots.append([(-1, False)] * bucket)
        return self._finish_plan(step_id, phase, bucket, mbs, [], record, [])

    # ------------------------------------------------------------------ completion
    def _retire(self, st: _ReqState) -> None:
        st.dead = True
        if st.inflight == 0:
            self._release(st)

    def _release(self, st: _ReqState) -> None:
        req = st.req
        valid = min(req.total_len - 1, st.planned_len) if req.output_ids else min(req.cached_len, st.planned_len)
        self.cache.release(st.prefix_handle, req.all_ids(), req.pages, max(valid, 0))
        self.reserved_pages -= st.reserved_pages
        self.free_rows.append(req.table_idx)
        self._pending_free_rows.append(req.table_idx)
        del self.states[req.uid]

    def complete(self, step_id: int, next_tokens: np.ndarray,
                 accepted: Optional[np.ndarray] = None) -> List[Tuple[int, List[int], bool]]:
        """Apply a step reply. `next_tokens` is the concatenation over micro-batches of one token
        per row (or, for verify steps, `spec_block` tokens per row with `accepted` counts).
        Returns [(uid, new_tokens, finished)]. Tokens of requests that finished in an earlier
        step (planned ahead, then hit EOS) are dropped."""
        rec = self.records.pop(step_id)
        out: List[Tuple[int, List[int], bool]] = []
        i = 0
        blk = self.spec_block if rec.phase == "verify" else 1
        tok_list = next_tokens.tolist()            # one conversion; per-row numpy slices cost more than the work
        acc_list = accepted.tolist() if (accepted is not None and blk > 1) else None
        for slots in rec.slots:
            for uid, emits in slots:
                row = i
                i += 1
                if uid < 0:
                    continue
                n_acc = int(acc_list[row]) if acc_list is not None else 1
                toks = tok_list[row * blk:row * blk + n_acc] if blk > 1 else tok_list[row:row + 1]
                st = self.states.get(uid)
                if st is None:
                    continue
                st.inflight -= 1
                req = st.req
                if rec.phase == "prefill":
                    req.cached_len = min(st.planned_len, req.prompt_len)
                if st.dead:
                    if st.inflight == 0:
                        self._release(st)
                    continue
                if not emits:
                    continue
                new: List[int] = []
                finished = False
                for t in toks:
                    req.output_ids.append(t)
                    new.append(t)
                    if (t in self.eos and not req.sampling.ignore_eos) or t in req.sampling.stop_token_ids \
                            or len(req.output_ids) >= req.sampling.max_tokens:
                        finished = True
                        break
                if rec.phase == "verify":
                    # the plan advanced by a whole block; only n_acc tokens were committed
                    st.planned_len -= (blk - len(new))
                    st.planned_out += len(new)
                req.finished = finished
                out.append((uid, new, finished))
                if finished:
                    self._retire(st)
        if self.page_audit:
            self.audit_pages()
        return out

    def check_integrity(self) -> None:
        self.cache.check_integrity()
        rows = [s.req.table_idx for s in self.states.values()]
        if len(set(rows)) != len(rows) or set(rows) & set(self.free_rows):
            raise RuntimeError("request table rows corrupted")

    def audit_pages(self) -> None:
        """Page ledger audit (``FASTAFD_PAGE_AUDIT=1`` runs it after every planned and every
        completed step): no page is both free and held, a page is held by two requests only as a
        shared cached prefix, every request holds enough pages for its planned length, and free +
        held + cached-only pages account for the whole pool.
        Reference: the PAGE_AUDIT knob of python/minisgl/afd_scheduler.py."""
        self.check_integrity()
        c = self.cache
        free = set(int(p) for p in c._free[:c._n_free])
        held: Dict[int, int] = {}
        for st in self.states.values():
            need = c.pages_for(st.planned_len)
            if len(st.req.pages) < need:
                raise RuntimeError(f"page audit: request {st.req.uid} holds {len(st.req.pages)} pages, needs {need}")
            for p in st.req.pages:
                if p <= 0 or p >= c.num_pages:
                    raise RuntimeError(f"page audit: request {st.req.uid} holds page {p} outside the pool")
                held[p] = held.get(p, 0) + 1
        both = free & set(held)
        if both:
            raise RuntimeError(f"page audit: pages {sorted(both)[:8]} are free and held at once")
        cached = set()
        if hasattr(c, "_iter_nodes"):
            cached = {int(n.page) for n in c._iter_nodes()}
            if cached & free:
                raise RuntimeError("page audit: a cached page is on the free list")
        shared_wrongly = [p for p, n in held.items() if n > 1 and p not in cached]
        if shared_wrongly:
            raise RuntimeError(f"page audit: pages {sorted(shared_wrongly)[:8]} are held twice without being a cached prefix")
        accounted = len(free) + len(set(held) | cached)
        if accounted != c.num_pages - 1:
            raise RuntimeError(f"page audit: {accounted} pages accounted for, the pool has {c.num_pages - 1}")
