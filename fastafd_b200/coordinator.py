"""AFD coordinator: admission, global step planning one or more steps ahead, result
collection and failure detection. CPU only.

The coordinator owns one :class:`LaneScheduler` per attention DP lane. Each *global step*
has one phase for all lanes (prefill wins over decode; lanes with nothing to do run a dummy
step because N2M / M2N involve every rank), one shared decode bucket, one plan per attention
rank and one plan per expert rank. Up to ``async_pending_steps`` steps are in flight: decode
step N+1 is planned as if step N produced one token per request, and the attention GPU reads
the real token from its device-side token pool, so planning never waits for the GPU.

The transport to the workers is abstract (:class:`WorkerTransport`): ZeroMQ PUSH/PULL
between processes, or direct calls for in-process use and tests.

Reference: python/minisgl/afd_coordinator.py (_admit_dp :817, _afd_prepare_step_launch
:1060-1165, _afd_launch_step :1308-1469, _afd_normal_loop :1484, _afd_overlap_loop :1566-1689,
_afd_next_global_phase :1768, _afd_complete_global :1818-1970, admission stall :1741,
get_failure :615, _log_step_time :1537).
"""
from __future__ import annotations

import os
import time
from collections import deque
from dataclasses import dataclass, field
from typing import Callable, Deque, Dict, List, Optional, Sequence, Tuple


from .config import ModelConfig, RuntimeConfig
from .core import SamplingParams
from .protocol import AfdTopology, AgStepPlan, AgStepReply, EgStepPlan, EgStepReply, WorkerFailure
from .scheduler.buckets import normalize_buckets, per_mb_real, select_bucket
from .scheduler.lane import LaneScheduler
from .utils.logger import init_logger

logger = init_logger("coordinator")


class WorkerTransport:
    """How plans reach the workers and replies come back."""

    def send_step(self, step_id: int, ag_plans: Dict[int, Tuple[AgStepPlan, List[int]]],
                  eg_plans: Dict[int, EgStepPlan]) -> None:
        """ag_plans: attention rank -> (plan, mb_tokens); eg_plans: expert rank -> plan."""
        raise NotImplementedError

    def poll(self, timeout_s: float) -> List[object]:
        """Replies (AgStepReply / EgStepReply / WorkerFailure) that arrived within timeout."""
        raise NotImplementedError

    def stop(self) -> None:
        pass


@dataclass
class _Inflight:
    step_id: int
    phase: str
    bucket: int
    t_launch: float
    waiting_ag: set = field(default_factory=set)
    waiting_eg: set = field(default_factory=set)
    replies: Dict[int, AgStepReply] = field(default_factory=dict)
    sizes: Dict[int, int] = field(default_factory=dict)
    real: List[int] = field(default_factory=list)


class CoordinatorError(RuntimeError):
    pass


def check_cache_type(cfg: ModelConfig, rt: RuntimeConfig) -> None:
    """A prefix hit skips the cached tokens, which is sound for attention (their K/V are in the shared pages) but
    not for the recurrent state of linear-attention layers: that state after the shared prefix is not kept
    anywhere. Hybrid models therefore run without prefix reuse.
    Reference: python/minisgl/scheduler/scheduler.py:155-159."""
    if cfg.num_linear_layers and rt.cache_type != "naive":
        raise ValueError(f"models with linear-attention layers need --cache-type naive (got {rt.cache_type!r}): the "
                         "recurrent state at the end of a cached prefix is not kept")
    if cfg.num_linear_layers and rt.spec_block > 1:
        raise ValueError("speculative decoding is not available for models with linear-attention layers: the recurrent "
                         "state cannot be rolled back past rejected draft tokens")


class AfdCoordinator:
    def __init__(self, cfg: ModelConfig, rt: RuntimeConfig, topo: AfdTopology, transport: WorkerTransport, *,
                 num_pages: int, max_comm_tokens: int = 2048,
                 on_tokens: Optional[Callable[[List[Tuple[int, List[int], bool]]], None]] = None,
                 worker_timeout_s: float = 120.0):
        self.cfg, self.rt, self.topo, self.transport = cfg, rt, topo, transport
        check_cache_type(cfg, rt)
        self.on_tokens = on_tokens or (lambda items: None)
        self.worker_timeout_s = worker_timeout_s
        self.buckets = [b for b in normalize_buckets(rt.decode_graph_bs, rt.cuda_graph_max_bs) if b % topo.attn_tp == 0] or [topo.attn_tp]
        self.num_lanes = 1 if topo.colocated else topo.attn_dp
        self.lanes = [LaneScheduler(l, num_pages=num_pages, page_size=rt.page_size, max_running=rt.max_running_requests,
                                    max_seq_len=rt.max_seq_len or cfg.max_position, num_mb=rt.num_mb,
                                    max_batched_tokens=rt.max_batched_tokens, max_comm_tokens=max_comm_tokens,
                                    cache_type=rt.cache_type, eos_token_ids=cfg.eos_token_ids, spec_block=rt.spec_block,
                                    spec_pending=2)
                      for l in range(self.num_lanes)]
        # Under speculation the committed lengths live on the attention GPUs, so verify steps are planned
        # ahead too (two in flight: the lane scheduler reserves KV for the unknown acceptance).
        if rt.disable_overlap:
            self.pending = 1
        elif rt.spec_block > 1:
            self.pending = min(2, max(1, rt.async_pending_steps))
        else:
            self.pending = max(1, rt.async_pending_steps)
        self.inflight: Deque[_Inflight] = deque()
        self.step_id = 0
        self.uid_lane: Dict[int, int] = {}
        self._rr = 0
        self.failure: Optional[str] = None
        self.stopped = False
        self.step_times: List[Tuple[int, str, int, float]] = []
        self.log_step_times = False
        self.reply_latency: Dict[int, List[float]] = {}      # rank -> [replies, sum of ms, max ms] from launch to reply
        self.spec_rows = self.spec_tokens = self.spec_steps = 0
        from .env import ENV
        self.log_steps = bool(ENV.LOG_STEPS.value)        # one line per launched step (plan summary)
        self._log_file = None
        if ENV.LOG_DIR.value:
            from .utils.logger import BufferedLogFile
            self._log_file = BufferedLogFile(os.path.join(ENV.LOG_DIR.value, "coordinator.log"))

    # ------------------------------------------------------------------ admission
    def _pick_lane(self, input_ids: Sequence[int]) -> int:
        """Round-robin over lanes, or the lane with the longest cached prefix under the radix
        cache (ties -> least loaded)."""
        if self.rt.cache_type == "radix" and self.num_lanes > 1:
            hits = [l.prefix_hit_len(input_ids) for l in self.lanes]
            best = max(hits)
            if best > 0:
                cands = [i for i, h in enumerate(hits) if h == best]
                return min(cands, key=lambda i: self.lanes[i].load)
        lane = self._rr % self.num_lanes
        self._rr += 1
        return lane

    def add_request(self, uid: int, input_ids: Sequence[int], sampling: SamplingParams) -> None:
        if self.failure:
            raise CoordinatorError(self.failure)
        lane = self._pick_lane(input_ids)
        self.lanes[lane].add_req(uid, input_ids, sampling)      # raises AdmissionError when impossible
        self.uid_lane[uid] = lane

    def abort(self, uid: int) -> None:
        lane = self.uid_lane.pop(uid, None)
        if lane is not None:
            self.lanes[lane].abort(uid)

    # ------------------------------------------------------------------ planning
    def _next_phase(self) -> Optional[str]:
        if any(l.has_prefill() for l in self.lanes):
            return "prefill"
        if any(l.decode_real() > 0 for l in self.lanes):
            return "verify" if self.rt.spec_block > 1 else "decode"
        return None

    def idle(self) -> bool:
        return not self.inflight and all(l.idle() for l in self.lanes)

    def plan_and_launch(self) -> bool:
        """Plan one global step and hand it to the transport. False when there is nothing to run."""
        phase = self._next_phase()
        if phase is None:
            if not self.inflight:
                for l in self.lanes:
                    l.check_admission_stall()
            return False
        sid = self.step_id
        self.step_id += 1
        nmb = self.rt.num_mb
        if phase == "prefill":
            plans = [l.schedule_prefill(sid) if l.has_prefill() else l.dummy_step(sid, "prefill", 0) for l in self.lanes]
            tp = self.topo.attn_tp       # token counts are per dispatch source (= per attention rank)
            mb_tokens = [max((max(p.mbs[m].num_tokens for p in plans) + tp - 1) // tp, 1) for m in range(nmb)]
            bucket = 0
        else:
            q = self.rt.spec_block if phase == "verify" else 1
            real = max(l.decode_real() for l in self.lanes)
            bucket = select_bucket(per_mb_real(real, nmb), self.buckets)
            plans = [l.schedule_decode(sid, bucket, q) if l.decode_real() else l.dummy_step(sid, phase, bucket)
                     for l in self.lanes]
            mb_tokens = [bucket * q // self.topo.attn_tp] * nmb
        rec = _Inflight(sid, phase, bucket, time.perf_counter())
        rec.real = [sum(mb.num_real for mb in p.mbs) for p in plans]
        ag_plans, eg_plans = {}, {}
        if self.topo.colocated:
            ag_plans[0] = (plans[0], mb_tokens)
            rec.waiting_ag.add(0)
            rec.sizes[0] = sum(len(mb.rows) for mb in plans[0].mbs)
        else:
            for lane, plan in enumerate(plans):
                for r in self.topo.attn_tp_group(lane):
                    ag_plans[r] = (plan, mb_tokens)
                    rec.waiting_ag.add(r)
                rec.sizes[lane] = sum(len(mb.rows) for mb in plan.mbs)
            for r in self.topo.expert_ranks():
                eg_plans[r] = EgStepPlan(step_id=sid, phase=phase, tokens_per_mb=mb_tokens)
                rec.waiting_eg.add(r)
        self.transport.send_step(sid, ag_plans, eg_plans)
        self.inflight.append(rec)
        if self.log_steps:
            self._step_log(f"[afd-step] launch step={sid} phase={phase} bucket={bucket} mb_tokens={list(mb_tokens)} "
                           f"real={rec.real} inflight={len(self.inflight)} waiting="
                           f"{sum(len(l.waiting) for l in self.lanes)}")
        return True

    def _step_log(self, text: str) -> None:
        """Step lines go to the buffered per-process file under FASTAFD_LOG_DIR when set (no write
        syscall per step on the hot loop), else to the logger."""
        if self._log_file is not None:
            self._log_file.line(text)
        else:
            logger.info(text)

    # ------------------------------------------------------------------ completion
    def _on_reply(self, msg) -> None:
        if isinstance(msg, WorkerFailure):
            self.failure = f"worker {msg.rank} failed: {msg.error}"
            return
        rec = next((r for r in self.inflight if r.step_id == msg.step_id), None)
        if rec is None:
            return
        self._note_latency(msg.rank, rec)
        if msg.status:
            self.failure = f"rank {msg.rank} reported device status {msg.status} in step {msg.step_id}"
        if isinstance(msg, AgStepReply):
            rec.waiting_ag.discard(msg.rank)
            rec.replies[msg.rank] = msg
        elif isinstance(msg, EgStepReply):
            rec.waiting_eg.discard(msg.rank)

    def _note_latency(self, rank: int, rec: _Inflight) -> None:
        ms = (time.perf_counter() - rec.t_launch) * 1e3
        st = self.reply_latency.setdefault(rank, [0, 0.0, 0.0])
        st[0] += 1
        st[1] += ms
        st[2] = max(st[2], ms)

    def latency_summary(self) -> Dict[int, Dict[str, float]]:
        """Per rank: replies seen, mean and worst time from a step's launch to that rank's reply (ms). A rank
        whose mean stands out is the one the others wait for.
        Reference: python/minisgl/afd_coordinator.py:484-528 (worker reply-latency logs)."""
        return {r: {"replies": n, "mean_ms": round(tot / n, 3), "max_ms": round(mx, 3)}
                for r, (n, tot, mx) in sorted(self.reply_latency.items()) if n}

    def spec_stats(self) -> Dict[str, float]:
        """Speculative decoding so far: verify steps, request rows verified, tokens emitted, and their ratio
        (mean accepted length, between 1 and the block size).
        Reference: python/minisgl/afd_attention_worker.py:1432 (acceptance statistics)."""
        mean = self.spec_tokens / self.spec_rows if self.spec_rows else 0.0
        return {"verify_steps": self.spec_steps, "rows": self.spec_rows, "tokens": self.spec_tokens, "mean_accepted": round(mean, 4)}

    def _complete_oldest(self) -> None:
        rec = self.inflight.popleft()
        items: List[Tuple[int, List[int], bool]] = []
        for lane, sched in enumerate(self.lanes):
            src = 0 if self.topo.colocated else self.topo.attn_tp_group(lane)[0]
            reply = rec.replies[src]
            items += sched.complete(rec.step_id, reply.next_tokens, reply.accepted)
        if rec.phase == "verify":
            self.spec_steps += 1
            self.spec_rows += sum(1 for _u, toks, _f in items if toks)
            self.spec_tokens += sum(len(toks) for _u, toks, _f in items)
        ms = (time.perf_counter() - rec.t_launch) * 1e3
        self.step_times.append((rec.step_id, rec.phase, rec.bucket, ms))
        if self.log_step_times:
            self._step_log(f"[afd-step-time] step={rec.step_id} phase={rec.phase} bucket={rec.bucket} "
                           f"num_mb={self.rt.num_mb} ms={ms:.3f} real={rec.real}")
        for uid, _toks, fin in items:
            if fin:
                self.uid_lane.pop(uid, None)
        if items:
            self.on_tokens(items)

    def collect(self, block: bool) -> bool:
        """Take replies; completes the oldest in-flight step once all its workers answered.
        Returns True if a step completed. Raises on worker failure or timeout."""
        if not self.inflight:
            return False
        deadline = time.monotonic() + self.worker_timeout_s
        while True:
            head = self.inflight[0]
            if not head.waiting_ag and not head.waiting_eg:
                self._complete_oldest()
                return True
            msgs = self.transport.poll(0.05 if block else 0.0)
            for m in msgs:
                self._on_reply(m)
            if self.failure:
                raise CoordinatorError(self.failure)
            if not msgs and not block:
                return False
            if time.monotonic() > deadline:
                missing = sorted(head.waiting_ag | head.waiting_eg)
                self.failure = f"step {head.step_id}: no reply from ranks {missing} within {self.worker_timeout_s}s"
                raise CoordinatorError(self.failure)

    # ------------------------------------------------------------------ loops
    def run_until_idle(self) -> None:
        """Drive all admitted requests to completion (offline use)."""
        while not self.idle():
            self.step_loop_once(block=True)

    def step_loop_once(self, block: bool) -> bool:
        """One iteration of the overlap loop: fill the in-flight window, then collect.
        Returns True if anything was launched or completed."""
        progressed = False
        while len(self.inflight) < self.pending:
            if not self.plan_and_launch():
                break
            progressed = True
        if self.inflight:
            progressed |= self.collect(block)
        return progressed

    def get_failure(self) -> Optional[str]:
        return self.failure

    def shutdown(self) -> None:
        if not self.stopped:
            self.stopped = True
            if self.log_step_times or self.log_steps:
                self._step_log(f"[afd-summary] reply latency per rank (ms): {self.latency_summary()}")
                if self.spec_steps:
                    self._step_log(f"[afd-summary] speculative decoding: {self.spec_stats()}")
            self.transport.stop()


class InProcTransport(WorkerTransport):
    """Workers are engine objects in this process (colocated runs, tests). Steps execute
    synchronously inside send_step."""

    def __init__(self, engines: Dict[int, object]):
        self.engines = engines
        self._out: List[object] = []

    def send_step(self, step_id, ag_plans, eg_plans):
        for r, (plan, mb_tokens) in ag_plans.items():
            self._out.append(self.engines[r].step(plan, mb_tokens))
        for r, plan in eg_plans.items():
            self._out.append(self.engines[r].step(plan))

    def poll(self, timeout_s):
        out, self._out = self._out, []
        return out


class ZmqWorkerTransport(WorkerTransport):
    """Coordinator side of the ZeroMQ link: one PUSH socket per worker, one shared PULL."""

    def __init__(self, cmd_addrs: Dict[int, str], reply_addr: str):
        from .protocol import RunStepCmd, StopCmd, decode, encode
        from .utils.mp import ZmqPullQueue, ZmqPushQueue

        self._Run, self._Stop = RunStepCmd, StopCmd
        self.replies = ZmqPullQueue(reply_addr, bind=True, encode=encode, decode=decode)
        self.cmd = {r: ZmqPushQueue(a, bind=False, encode=encode, decode=decode) for r, a in cmd_addrs.items()}

    def send_step(self, step_id, ag_plans, eg_plans):
        for r, (plan, mb_tokens) in ag_plans.items():
            self.cmd[r].put(self._Run(plan=plan, mb_tokens=list(mb_tokens)))
        for r, plan in eg_plans.items():
            self.cmd[r].put(self._Run(plan=plan))

    def send_cad_init(self, cmd) -> None:
        """Core-attention disaggregation (cad/coordinator.py): the init command goes to every rank."""
        for q in self.cmd.values():
            q.put(cmd)

    def send_cad_step(self, step_id, attn_cmds, model_cmds) -> None:
        for r, c in list(attn_cmds.items()) + list(model_cmds.items()):
            self.cmd[r].put(c)

    def poll(self, timeout_s):
        out = []
        m = self.replies.get(timeout_ms=int(timeout_s * 1000)) if timeout_s > 0 else self.replies.get_nowait()
        while m is not None:
            out.append(m)
            m = self.replies.get_nowait()
        return out

    def wait_ready(self, n: int, timeout_s: float) -> List[object]:
        """Block until n workers said ready; raises on a reported failure or on timeout."""
        from .protocol import WorkerFailure, WorkerReady

        ready, deadline = [], time.monotonic() + timeout_s
        while len(ready) < n:
            m = self.replies.get(timeout_ms=500)
            if isinstance(m, WorkerFailure):
                raise CoordinatorError(f"worker {m.rank} failed during start-up: {m.error}")
            if isinstance(m, WorkerReady):
                ready.append(m)
            if time.monotonic() > deadline:
                raise CoordinatorError(f"only {len(ready)} of {n} workers became ready within {timeout_s}s")
        return ready

    def stop(self):
        for q in self.cmd.values():
            try:
                q.put(self._Stop())
            except Exception:
                pass
