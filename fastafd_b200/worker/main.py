"""Worker process of a served deployment: one per GPU (or per CPU rank in tests).

It joins the host-side process group, builds its :class:`AfdEngine`, then serves step
commands from the coordinator over ZeroMQ until told to stop. Decode steps are software
pipelined: when the next command is already waiting, it is queued on the GPU before the
previous step's tokens are read back, so host work hides behind device work.

Reference: python/minisgl/afd_worker_base.py:1183-1276 (start_hot_rpc_loop, shutdown),
python/minisgl/afd_attention_worker.py:1013 (centralized_overlap_loop),
python/minisgl/afd_expert_worker.py:648.
"""
from __future__ import annotations

import os
import traceback
from collections import deque
from typing import Dict

from ..protocol import (AgStepPlan, CadInitCmd, CadStepCmd, EgStepPlan, RunStepCmd, StopCmd, WorkerFailure, WorkerReady,
                        decode, encode)


def host_group_options(server_args) -> Dict[str, object]:
    """Keyword arguments of the host-side process group: `--distributed-timeout SECONDS` bounds its rendezvous
    and every blocking receive on it (0 keeps the library's default of half an hour).
    Reference: python/minisgl/server/args.py (--distributed-timeout), forwarded to every worker."""
    import datetime

    t = float(getattr(server_args, "distributed_timeout", 0.0) or 0.0)
    if t < 0:
        raise ValueError("--distributed-timeout must not be negative")
    return {"timeout": datetime.timedelta(seconds=t)} if t > 0 else {}


def worker_main(rank: int, world: int, server_args, addrs: Dict[str, object], master_port: int) -> None:
    import torch
    import torch.distributed as dist

    from ..config import get_model_config
    from ..engine import AfdEngine
    from ..utils.mp import ZmqPullQueue, ZmqPushQueue

    reply_q = ZmqPushQueue(addrs["reply"], bind=False, encode=encode, decode=decode)
    try:
        topo = server_args.topology
        rt = server_args.runtime_config()
        cfg = get_model_config(server_args.model_path)
        cuda = server_args.device == "cuda"
        if cuda:
            torch.cuda.set_device(rank % torch.cuda.device_count())
            device = torch.device("cuda", rank % torch.cuda.device_count())
        else:
            device = torch.device("cpu")
            torch.set_num_threads(1)
        if world > 1:
            os.environ["MASTER_ADDR"] = str(addrs.get("master_addr", "127.0.0.1"))     # the head node under a multi-node launch
            os.environ["MASTER_PORT"] = str(master_port)
            # The host-side group is gloo only: it carries plans, tokens and barriers. Device
            # collectives go through the framework's own NCCL communicator / fabric kernels. (A default
            # group bound to a device makes torch split its NCCL communicator inside new_group on
            # non-member ranks only, which blocks when the new group itself is a gloo group.)
            dist.init_process_group("gloo", rank=rank, world_size=world, **host_group_options(server_args))
        engine = AfdEngine(cfg, rt, topo, rank, device, seed=server_args.seed, fast_init=cuda,
                           max_comm_tokens=addrs.get("max_comm_tokens"))
        cad = None
        from ..cad.config import CadConfig

        if CadConfig.from_env().enabled:        # core-attention disaggregation: decode steps arrive as CAD commands
            from ..cad.worker import CadWorkerState

            cad = CadWorkerState(engine, rank)
        cmd_q = ZmqPullQueue(addrs["cmd"][rank], bind=True, encode=encode, decode=decode)
        reply_q.put(WorkerReady(rank=rank, role="attention" if engine.attn is not None else "expert",
                                num_pages=engine.attn.num_pages if engine.attn is not None else 0,
                                info={"max_comm_tokens": engine.max_comm_tokens}))
        from .profiler import StepProfiler

        prof = StepProfiler()
        pending = deque()
        send_reply, reported = reply_q.put, []

        def put_reply(reply) -> None:
            """Replies pass through here: the first one that carries a device status also prints where this rank's
            flag protocols stand (which peers are behind), once."""
            if getattr(reply, "status", 0) and not reported:
                reported.append(reply.step_id)
                print(f"[worker {rank}] step {reply.step_id} ended with device status {reply.status}; flags: "
                      f"{engine.describe_waits()}", flush=True)
            send_reply(reply)
        while True:
            cmd = cmd_q.get_nowait() if pending else cmd_q.get()
            if cmd is None:                      # nothing new: finish the oldest queued decode step
                put_reply(engine.finish(pending.popleft()))
                continue
            if isinstance(cmd, StopCmd):
                break
            if isinstance(cmd, CadInitCmd):
                cad.init(cmd)
                reply_q.put(WorkerReady(rank=rank, role="cad-" + cad.role))
                continue
            if isinstance(cmd, CadStepCmd):
                prof.on_step(cmd.step_id)
                reply_q.put(cad.run(cmd))
                continue
            plan = cmd.plan
            prof.on_step(plan.step_id)
            if isinstance(plan, EgStepPlan):
                put_reply(engine.step(plan))
            elif plan.phase == "prefill":
                while pending:
                    put_reply(engine.finish(pending.popleft()))
                put_reply(engine.step(plan, cmd.mb_tokens))
            else:
                engine.launch(plan)
                pending.append(plan)
                while len(pending) > 1:
                    put_reply(engine.finish(pending.popleft()))
        prof.close()
        engine.synchronize()
        if cuda:        # what this rank needed at its worst: the figure to size memory_ratio and the page count against
            free, total = torch.cuda.mem_get_info(device)
            print(f"[worker {rank}] peak device memory: {torch.cuda.max_memory_allocated(device) / 2**30:.2f} GiB allocated by torch, "
                  f"{(total - free) / 2**30:.2f} of {total / 2**30:.2f} GiB in use at exit", flush=True)
        engine.close()
        if world > 1:
            dist.destroy_process_group()
    except Exception as e:  # report instead of dying silently: the coordinator turns it into a failure
        reply_q.put(WorkerFailure(rank=rank, error=f"{type(e).__name__}: {e}\n{traceback.format_exc()[-1500:]}"))
        raise
