"""One process of an AFD deployment, and an SPMD driver for it.

:class:`AfdEngine` builds what this rank needs from the topology:

* world 1 (colocated): attention stage and expert stage in one process on one device; the
  expert layer is launched right behind each dispatch.
* world > 1: rank < attn_world is an attention worker, the others are expert workers. On
  CUDA they share peer-mapped heaps (:class:`fastafd_b200.parallel.fabric.Fabric`) and talk
  through the fused kernels; on CPU they exchange tensors over gloo.

:class:`SpmdDriver` runs requests through the engines without a separate coordinator
process: every rank holds the lane schedulers and the ranks agree on each step's phase and
sizes with one small all-gather (used by the offline ``LLM`` API, the tests and the
benchmark; the server uses :mod:`fastafd_b200.coordinator` instead).

Reference: python/minisgl/afd_worker_base.py:560-715 (_init_afd_runtime),
python/minisgl/engine/engine.py:212-433 (colocated Engine).
"""
from __future__ import annotations

import os

from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np
import torch
import torch.distributed as dist

from .config import ModelConfig, RuntimeConfig
from .core import SamplingParams
from .models.transformer import ExpertStage
from .protocol import AfdTopology, AgStepPlan, AgStepReply, EgStepPlan
from .scheduler.buckets import normalize_buckets, per_mb_real, select_bucket
from .scheduler.lane import LaneScheduler
from .worker.attention_worker import AttentionWorker
from .worker.expert_worker import ExpertWorker
from .worker.moe_client import (FabricMoeClient, FabricMoeServer, GlooMoeClient, GlooMoeServer, LocalMoeClient)


def _torch_dtype(name: str, device: torch.device) -> torch.dtype:
    if device.type != "cuda":
        return torch.float32
    return {"bfloat16": torch.bfloat16, "float16": torch.float16, "float32": torch.float32}[name]


def resolve_checkpoint(rt: RuntimeConfig) -> Optional[str]:
    """Directory whose safetensors files hold the served weights, or None for random-init
    weights (a preset name, or ``dummy_weights`` with a directory that only has config.json).
    A directory without safetensors files is refused rather than served with random weights.
    Reference: python/minisgl/engine/engine.py:330 (use_dummy_weight), models/weight.py:419."""
    path = rt.model_path
    if not os.path.isdir(path) or rt.dummy_weights:
        return None
    import glob

    if not glob.glob(os.path.join(path, "*.safetensors")):
        raise FileNotFoundError(f"{path} has no .safetensors files; pass --dummy-weights to serve random weights "
                                f"of the architecture in its config.json")
    return path


def decode_buckets(rt: RuntimeConfig, topo: AfdTopology) -> List[int]:
    """Decode graph sizes; with attention TP every bucket is a multiple of the TP size (the
    residual stream is sharded by tokens across the TP ranks)."""
    b = [x for x in normalize_buckets(rt.decode_graph_bs, rt.cuda_graph_max_bs) if x % topo.attn_tp == 0]
    return b or [topo.attn_tp]


def make_tp_comms(topo: AfdTopology, rank: int, device: torch.device, group=None):
    """One communicator per attention lane. Every rank of the world takes part in the set-up, in the
    same order. On CUDA the lane leaders' NCCL ids travel in one all-gather over the host group and no
    sub-group is made (torch's new_group on a default group that is bound to a device splits an NCCL
    communicator on the non-member ranks only, and blocks there if the new group is a gloo group). On
    CPU each lane gets a gloo sub-group. Returns this rank's communicator or None."""
    if topo.colocated or topo.attn_tp == 1:
        return None
    from .parallel.comm import NcclComm, TorchDistComm

    lanes = [topo.attn_tp_group(lane) for lane in range(topo.attn_dp)]
    if device.type == "cuda":
        my_lane = next((r for r in lanes if rank in r), None)
        uid = NcclComm.new_unique_id() if my_lane is not None and my_lane[0] == rank else None
        ids = [None] * dist.get_world_size(group)
        dist.all_gather_object(ids, uid, group=group)
        return NcclComm(my_lane, device, uid=ids[my_lane[0]]) if my_lane is not None else None
    mine = None
    for ranks in lanes:
        g = dist.new_group(ranks)
        if rank in ranks:
            mine = TorchDistComm(g, ranks)
    return mine


class AfdEngine:
    def __init__(self, cfg: ModelConfig, rt: RuntimeConfig, topo: AfdTopology, rank: int, device,
                 group=None, seed: int = 0, fast_init: bool = False, max_comm_tokens: Optional[int] = None):
        self.cfg, self.rt, self.topo, self.rank, self.group = cfg, rt, topo, rank, group
        self.device, self.seed = torch.device(device), seed
        self.dtype = _torch_dtype(rt.dtype, self.device)
        self.colocated = topo.world == 1
        if not self.colocated:
            from .protocol import validate_parallel_args

            validate_parallel_args(topo, max(cfg.num_experts, topo.mlp_ep), cfg.num_q_heads, cfg.num_kv_heads,
                                   cfg.gdn_num_k_heads if cfg.num_linear_layers else 0,
                                   cfg.gdn_num_v_heads if cfg.num_linear_layers else 0)
        self.is_attention = self.colocated or topo.is_attention(rank)
        self.is_expert = self.colocated or topo.is_expert(rank)
        cuda = self.device.type == "cuda"
        self.buckets = decode_buckets(rt, topo)
        cap = self.buckets[-1]
        self.max_comm_tokens = max_comm_tokens or max(cap, min(2048, rt.max_batched_tokens // max(rt.num_mb, 1)))
        self.fabric = None
        self.attn: Optional[AttentionWorker] = None
        self.expert: Optional[ExpertWorker] = None
        # MLP TP with mlp_ep == 1: the ranks of a replica all hold every expert with a slice of the
        # intermediate dimension and return partial sums. mlp_ep == mlp_tp means expert parallelism
        # inside the TP group, i.e. plain EP. On GPUs the slices are "virtual experts": slice r of
        # expert e is expert r * E + e, owned by expert rank r, and a token that chose e with weight w
        # chooses all its slices with weight w - dispatch, grouping and the combine sum then work
        # unchanged on E * tp experts with top-(K * tp) routing.
        mlp_tp_shard = (not self.colocated) and topo.mlp_tp > 1 and topo.mlp_ep == 1
        tp_expand = topo.mlp_tp if (mlp_tp_shard and cuda) else 1
        if tp_expand > 1 and cfg.num_experts_per_tok * tp_expand > 32:
            raise ValueError("MLP TP on GPUs needs num_experts_per_tok x mlp_tp <= 32")
        # One replica of the expert set (mlp_dp of them) serves the lanes l with l % mlp_dp == replica:
        # an attention rank talks to its replica's expert ranks, an expert rank to its lanes' ranks.
        if self.colocated:
            eg_ranks, ag_ranks, my_ag_index = [0], [0], 0
        elif self.is_attention:
            eg_ranks = topo.expert_ranks_for(rank)
            ag_ranks = topo.attention_ranks_for(eg_ranks[0])
            my_ag_index = ag_ranks.index(rank)
        else:
            ag_ranks = topo.attention_ranks_for(rank)
            eg_ranks = topo.expert_ranks_for(ag_ranks[0])
            my_ag_index = -1
        num_eg, num_ag = len(eg_ranks), len(ag_ranks)

        ckpt = resolve_checkpoint(rt)
        self.checkpoint = ckpt
        # ONE device status word per process: every kernel of every communicator on this GPU reports
        # into it and polls it inside its waits, so the first wait that runs out is the only one that
        # costs its full time limit; the rest of the step drains at once and the host raises.
        self.status_word = torch.zeros(1, dtype=torch.int32, device=self.device) if cuda else None
        sw = self.status_word
        stage = None
        if self.is_expert and cfg.is_moe and os.environ.get("FASTAFD_DEBUG_NULL_MOE") != "1":
            ep_rank = 0 if self.colocated else topo.ep_rank(rank)
            if mlp_tp_shard:
                stage = ExpertStage(cfg, self.device, self.dtype, 0, 1, tp_rank=ep_rank, tp_size=topo.mlp_tp)
            else:
                stage = ExpertStage(cfg, self.device, self.dtype, ep_rank, num_eg)
            if ckpt is not None:
                from .models.loader import load_expert_stage

                load_expert_stage(stage, ckpt)
            else:
                stage.init_random(seed, fast=fast_init)
        self.expert_stage = stage

        from .worker.moe_client import MoeClient

        client, server = MoeClient(), None      # dense models: no experts to reach
        eg_status = None
        tp_heap_base = 0
        if os.environ.get("FASTAFD_DEBUG_NULL_MOE") == "1" and cfg.is_moe:
            from .worker.moe_client import NullMoeClient

            client, stage = NullMoeClient(), None
        elif cfg.is_moe:
            if cuda:
                from .moe.afd_moe import AgMoeEndpoint, EgMoeEndpoint, MoeCommConfig, ag_layout, eg_layout
                from .parallel.fabric import Fabric

                # decode-sized steps store rows straight into the experts' pool stripes (moe/afd_moe.py)
                direct = min(self.max_comm_tokens, max(cap * max(rt.spec_block, 1) // topo.attn_tp, 1))
                experts_local = (cfg.num_experts * tp_expand + num_eg - 1) // num_eg
                if os.environ.get("FASTAFD_DIRECT", "1") == "0" or num_ag * direct > 1024 or experts_local > 512:
                    direct = 0
                mcfg = MoeCommConfig(num_ag=num_ag, num_eg=num_eg, num_lanes=rt.num_mb, max_tokens=self.max_comm_tokens,
                                     hidden=cfg.hidden_size, topk=cfg.num_experts_per_tok * tp_expand,
                                     num_experts=cfg.num_experts * tp_expand,
                                     intermediate=cfg.moe_intermediate_size // tp_expand, fp8=cfg.quant.is_fp8,
                                     block_tok=rt.moe_block_tok, direct_tokens=direct)
                timeout_ns = int(rt.flag_timeout_s * 1e9)
                if self.colocated:
                    fabs = Fabric.local([ag_layout(mcfg).size, eg_layout(mcfg).size], self.device)
                    self.fabric = fabs
                    eg_ep = EgMoeEndpoint(mcfg, fabs[1], 0, [0], self.device, timeout_ns, status=sw)
                    server = FabricMoeServer(eg_ep, stage)
                    client = FabricMoeClient(AgMoeEndpoint(mcfg, fabs[0], 0, [1], self.device, timeout_ns, status=sw), colocated=server)
                    eg_status = eg_ep.status
                else:
                    size = ag_layout(mcfg).size if self.is_attention else eg_layout(mcfg).size
                    fuse_tp = (self.is_attention and topo.attn_tp > 1 and cfg.hidden_size % 128 == 0
                               and os.environ.get("FASTAFD_TP_FUSED", "1") == "1")     # FASTAFD_TP_FUSED=0: NCCL collectives
                    if fuse_tp:
                        from .parallel.tp_fused import tp_layout

                        tp_heap_base = size
                        size += tp_layout(topo.attn_tp, rt.num_mb, self.max_comm_tokens, cfg.hidden_size).size
                    self.fabric = Fabric.ipc(size, self.device, group)
                    if self.is_attention:
                        client = FabricMoeClient(AgMoeEndpoint(mcfg, self.fabric, my_ag_index, eg_ranks, self.device, timeout_ns, status=sw),
                                                 tp_expand=tp_expand, base_experts=cfg.num_experts)
                    else:
                        eg_ep = EgMoeEndpoint(mcfg, self.fabric, topo.ep_rank(rank), ag_ranks,
                                              self.device, timeout_ns, status=sw)
                        server = FabricMoeServer(eg_ep, stage)
                        eg_status = eg_ep.status
            else:
                if self.colocated:
                    client = LocalMoeClient([stage])
                elif self.is_attention:
                    client = GlooMoeClient(eg_ranks, cfg.hidden_size, cfg.num_experts_per_tok, group)
                else:
                    server = GlooMoeServer(stage, ag_ranks, cfg.hidden_size, cfg.num_experts_per_tok,
                                           self.dtype, group)
        tp_comm = make_tp_comms(topo, rank, self.device, group)
        if tp_comm is not None and cuda and cfg.is_moe and self.fabric is not None and self.is_attention \
                and not self.colocated and tp_heap_base > 0:
            from .parallel.tp_fused import TpFusedComm

            lane_ranks = topo.attn_tp_group(topo.attn_lane(rank))
            tp_comm = TpFusedComm(tp_comm, self.fabric, lane_ranks, topo.attn_tp_rank(rank), tp_heap_base, rt.num_mb,
                                  self.max_comm_tokens, cfg.hidden_size, self.device, int(rt.flag_timeout_s * 1e9), status=sw)
        if self.is_attention:
            tp_rank = 0 if self.colocated else topo.attn_tp_rank(rank)
            self.attn = AttentionWorker(cfg, rt, self.device, client, tp_rank=tp_rank, tp_size=topo.attn_tp,
                                        tp_comm=tp_comm, dtype=self.dtype, rank=rank, max_bucket=cap, status=sw,
                                        dp_lane=0 if self.colocated else topo.attn_lane(rank),
                                        weight_init=self._attention_weight_init(ckpt, seed, fast_init))
        if self.attn is not None and rt.spec_block > 1:

            from .spec.attn_side import SpecRunner

            self.attn.spec = SpecRunner(self.attn, rt.spec_block, rt.spec_draft_path, seed,
                                        float(os.environ.get("FASTAFD_SPEC_SIM_ACCEPT", "0") or 0))
        if self.is_expert and not self.colocated:
            self.expert = ExpertWorker(cfg, rt, self.device, stage, server, rank, eg_status)
        self._server = server

    @staticmethod
    def _attention_weight_init(ckpt: Optional[str], seed: int, fast_init: bool):
        if ckpt is None:
            return lambda m: m.init_random(seed, fast=fast_init)
        from .models.loader import load_attention_stage

        return lambda m: load_attention_stage(m, ckpt)

    # ------------------------------------------------------------------ stepping
    def step(self, plan, mb_tokens: Optional[List[int]] = None):
        """Run one planned step on this rank and wait for it (attention: returns the sampled
        tokens; expert: returns after the kernels were queued)."""
        if isinstance(plan, EgStepPlan):
            return self.expert.run_step(plan)
        return self.attn.run_step(plan, mb_tokens)

    def launch(self, plan: AgStepPlan) -> None:
        self.attn.launch_decode(plan)

    def finish(self, plan: AgStepPlan) -> AgStepReply:
        return self.attn.finish_decode(plan)

    def synchronize(self) -> int:
        """Wait for queued work; returns the device status word (0 = ok)."""
        if self.device.type == "cuda":
            torch.cuda.synchronize(self.device)
        code = 0
        if self.attn is not None:
            code = self.attn.read_status()
        if self.expert is not None:
            code = code or self.expert.finish()
        return code

    def describe_waits(self) -> Dict[str, object]:
        """After a step that ended with a device status: where the flag protocols of this rank stand (which
        peers' flags are behind). Never raises; what cannot be read is left out."""
        out: Dict[str, object] = {}
        for name, ep in (("dispatch_client", getattr(getattr(self.attn, "client", None), "ep", None)),
                         ("expert_server", getattr(self._server, "ep", None))):
            try:
                if ep is not None and hasattr(ep, "flag_report"):
                    out[name] = ep.flag_report()
            except Exception as e:       # triage output must not mask the failure it describes
                out[name] = f"unreadable: {e!r}"
        return out

    def close(self) -> None:
        if self.fabric is None:
            return
        for f in (self.fabric if isinstance(self.fabric, list) else [self.fabric]):
            f.close()
        self.fabric = None


class SpmdDriver:
    """Coordinator logic replicated on every rank (no separate coordinator process).

    Every rank builds the same lane schedulers from the same request list; attention rank r
    executes lane r's plans, expert ranks execute the matching expert plans. Step decisions
    depend on the sampled tokens only through request completion, which the attention ranks
    share with one gloo all-gather per step."""

    def __init__(self, engine: AfdEngine, num_pages: Optional[int] = None):
        self.e = engine
        topo, rt, cfg = engine.topo, engine.rt, engine.cfg
        from .coordinator import check_cache_type

        check_cache_type(cfg, rt)
        self.num_lanes = 1 if engine.colocated else topo.attn_dp
        pages = num_pages or (engine.attn.num_pages if engine.attn is not None else rt.num_pages)
        if not engine.colocated and dist.is_initialized():
            t = torch.tensor([pages if engine.attn is not None else 1 << 30], dtype=torch.int64)
            dist.all_reduce(t, op=dist.ReduceOp.MIN, group=engine.group)
            pages = int(t[0])
        self.lanes = [LaneScheduler(l, num_pages=pages, page_size=rt.page_size, max_running=rt.max_running_requests,
                                    max_seq_len=rt.max_seq_len or cfg.max_position, num_mb=rt.num_mb,
                                    max_batched_tokens=rt.max_batched_tokens, max_comm_tokens=engine.max_comm_tokens,
                                    cache_type=rt.cache_type, eos_token_ids=cfg.eos_token_ids, spec_block=rt.spec_block,
                                    spec_pending=2)
                      for l in range(self.num_lanes)]
        self.step_id = 0
        self.my_lane = None
        if engine.attn is not None:
            self.my_lane = 0 if engine.colocated else topo.attn_lane(engine.rank)

    def add_requests(self, prompts: Sequence[Sequence[int]], sampling: SamplingParams) -> List[int]:
        uids = []
        for i, p in enumerate(prompts):
            lane = min(range(self.num_lanes), key=lambda l: (self.lanes[l].load, l))
            uid = getattr(self, "_next_uid", 0)
            self._next_uid = uid + 1
            self.lanes[lane].add_req(uid, p, sampling)
            uids.append(uid)
        return uids

    def _exchange_tokens(self, reply: Optional[AgStepReply], sizes: List[int], q: int = 1):
        """Every rank learns every lane's sampled tokens (and accepted counts) of this step.
        sizes[lane] = rows of that lane; a verify step carries q tokens per row."""
        if self.e.colocated or not dist.is_initialized():
            return [reply.next_tokens], [reply.accepted]
        n = max(sizes) if sizes else 0
        mine = torch.full((1 + n * q + n,), -1, dtype=torch.int64)
        mine[0] = 0
        if reply is not None:
            mine[0] = reply.status
            mine[1:1 + len(reply.next_tokens)] = torch.from_numpy(reply.next_tokens.astype(np.int64))
            if reply.accepted is not None:
                mine[1 + n * q:1 + n * q + len(reply.accepted)] = torch.from_numpy(reply.accepted.astype(np.int64))
        bufs = [torch.empty_like(mine) for _ in range(self.e.topo.world)]
        dist.all_gather(bufs, mine, group=self.e.group)
        toks, acc = [], []
        for lane in range(self.num_lanes):
            src = lane * self.e.topo.attn_tp
            if int(bufs[src][0]) != 0:
                raise RuntimeError(f"attention rank {src} reported device status {int(bufs[src][0])}")
            toks.append(bufs[src][1:1 + sizes[lane] * q].numpy().astype(np.int32))
            acc.append(bufs[src][1 + n * q:1 + n * q + sizes[lane]].numpy().astype(np.int32) if q > 1 else None)
        return toks, acc

    def run_step(self) -> Optional[List[Tuple[int, List[int], bool]]]:
        """Plan and execute one global step; returns [(uid, new_tokens, finished)] or None when idle."""
        lanes = self.lanes
        if all(l.idle() for l in lanes):
            return None
        sid = self.step_id
        self.step_id += 1
        if any(l.has_prefill() for l in lanes):
            plans = [l.schedule_prefill(sid) if l.has_prefill() else l.dummy_step(sid, "prefill", 0) for l in lanes]
            tp = self.e.topo.attn_tp
            mb_tokens = [max((max(p.mbs[m].num_tokens for p in plans) + tp - 1) // tp, 1) for m in range(self.e.rt.num_mb)]
            phase, bucket, q = "prefill", 0, 1
        else:
            real = max(l.decode_real() for l in lanes)
            if real == 0:
                for l in lanes:
                    l.check_admission_stall()
                return []
            bucket = select_bucket(per_mb_real(real, self.e.rt.num_mb), self.e.buckets)
            q = self.e.rt.spec_block if self.e.rt.spec_block > 1 else 1
            phase = "verify" if q > 1 else "decode"
            plans = [l.schedule_decode(sid, bucket, q) if l.decode_real() else l.dummy_step(sid, phase, bucket) for l in lanes]
            mb_tokens = [bucket * q // self.e.topo.attn_tp] * self.e.rt.num_mb
        reply = None
        if self.e.attn is not None:
            reply = self.e.step(plans[self.my_lane], mb_tokens)
        if self.e.expert is not None:
            self.e.step(EgStepPlan(step_id=sid, phase=phase, tokens_per_mb=mb_tokens))
        sizes = [sum(len(mb.rows) for mb in p.mbs) for p in plans]
        toks, acc = self._exchange_tokens(reply, sizes, q if phase == "verify" else 1)
        out = []
        for lane, l in enumerate(lanes):
            out += l.complete(sid, toks[lane], acc[lane])
        return out

    # ------------------------------------------------------------------ steady-state decode
    def install_prefilled(self, per_lane: int, prompt_len: int, max_tokens: int, seed: int = 0) -> None:
        """Synthetic serving state: `per_lane` requests per attention lane whose prompts of
        `prompt_len` tokens are taken as already prefilled. The KV cache of the attention ranks is
        filled with N(0,1) values and each request's last token is a random id, so decode steps
        do the same work as after a real prefill of random prompts."""
        sp = SamplingParams(max_tokens=max_tokens, ignore_eos=True)
        my_rows = []
        for li, lane in enumerate(self.lanes):
            for _ in range(per_lane):
                uid = getattr(self, "_next_uid", 0)
                self._next_uid = uid + 1
                req = lane.add_prefilled(uid, prompt_len, sp)
                if li == self.my_lane:
                    my_rows.append(req.table_idx)
        a = self.e.attn
        if a is not None and a.spec is not None and my_rows:
            rows = torch.tensor(my_rows, dtype=torch.int64, device=a.device)
            a.spec.set_committed(rows, torch.full((len(my_rows),), prompt_len, dtype=torch.int32, device=a.device))
        if a is not None:
            g = torch.Generator(device=a.device).manual_seed(seed + 17 * self.e.rank)
            for t in (a.kv.k, a.kv.v):
                for li in range(t.shape[0]):
                    t[li].normal_(0.0, 1.0, generator=g)
            a.token_pool.copy_(torch.randint(0, self.e.cfg.vocab_size, a.token_pool.shape, generator=g,
                                             device=a.device, dtype=torch.int32))

    def run_decode_steps(self, n: int, pipelined: bool = True, events: Optional[list] = None, event_stream=None) -> int:
        """n decode steps of the running batch through plan -> H2D -> replay -> D2H -> complete.
        Requests must be greedy / ignore_eos with enough max_tokens left, so that every rank can
        plan without exchanging tokens (the one-step-ahead assumption of the coordinator: step
        N+1 is planned as if step N produced one token per request). With `pipelined`, step N+1
        is planned and queued before step N's tokens are read back. `events`: a list that receives one
        CUDA timing event per step, recorded on `event_stream` behind the step's work. Returns tokens
        generated by this rank's lane."""
        e, rt = self.e, self.e.rt
        produced = 0
        pending = None
        q = rt.spec_block if rt.spec_block > 1 else 1       # verify steps: q tokens per request
        for _ in range(n):
            sid = self.step_id
            self.step_id += 1
            real = max(l.decode_real() for l in self.lanes)
            bucket = select_bucket(per_mb_real(real, rt.num_mb), e.buckets)
            # Only this rank's lane is planned in full; the other lanes are advanced as shadows
            # (their sizes decide the common bucket, their pages and plans belong to other ranks).
            mine = None
            for lane, l in enumerate(self.lanes):
                if e.attn is not None and lane == self.my_lane:
                    mine = l.schedule_decode(sid, bucket, q)
                else:
                    l.shadow_decode(q)
            if e.attn is not None:
                e.attn.launch_decode(mine)
                if pending is not None:
                    produced += self._finish_fast(*pending)
                    pending = None
                if pipelined:
                    pending = (sid, mine)
                else:
                    produced += self._finish_fast(sid, mine)
            if e.expert is not None:
                e.step(EgStepPlan(step_id=sid, phase="decode" if q == 1 else "verify",
                                  tokens_per_mb=[bucket * q // e.topo.attn_tp] * rt.num_mb))
            if events is not None:          # one timing event per queued step (per-step device times)
                ev = torch.cuda.Event(enable_timing=True)
                ev.record(event_stream)
                events.append(ev)
        if pending is not None:
            produced += self._finish_fast(*pending)
        return produced

    def _finish_fast(self, sid: int, mine) -> int:
        reply = self.e.attn.finish_decode(mine)
        if reply.status:
            raise RuntimeError(f"device status {reply.status} in step {sid}")
        out = self.lanes[self.my_lane].complete(sid, reply.next_tokens, reply.accepted)
        return sum(len(t) for _, t, _ in out)

    def generate(self, prompts: Sequence[Sequence[int]], sampling: SamplingParams) -> List[List[int]]:
        uids = self.add_requests(prompts, sampling)
        results: Dict[int, List[int]] = {u: [] for u in uids}
        while True:
            out = self.run_step()
            if out is None:
                break
            for uid, toks, _ in out:
                results[uid] += toks
        code = self.e.synchronize()
        if code:
            raise RuntimeError(f"device status {code}")
        return [results[u] for u in uids]
