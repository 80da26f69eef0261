"""Process supervision of a served deployment on one machine.

    HTTP frontend (this process, asyncio)
        |  ZMQ  TokenizeMsg / UserReply
    tokenizer + detokenizer process
        |  ZMQ  UserMsg / BatchDetokenizeMsg
    coordinator process (CPU only: admission, planning, completion)
        |  ZMQ  RunStepCmd / step replies
    worker processes, one per GPU (attention ranks first, then expert ranks)

``LocalSupervisor.start()`` picks free ports, spawns every process with the ``spawn`` start
method, waits until all workers reported ready (bounded by the start-up timeout, with early
detection of a process that died), and returns the addresses the frontend needs.
``get_failures()`` lists dead processes; ``shutdown()`` stops everything (stop message,
then terminate, then kill) and is idempotent.

The reference runs workers as Ray actors (python/minisgl/server/supervisor_ray.py,
supervisor_afd.py) or local processes (supervisor_local.py); on a single 8-GPU machine
plain processes are enough, so this build has the local flavour only and refuses
``--launch-backend ray`` when Ray is absent.

Reference: python/minisgl/server/supervisor.py:172-181, supervisor_local.py,
python/minisgl/afd_worker_launcher.py:26-346 (start-up sequence, timeouts, early death).
"""
from __future__ import annotations

import os

import multiprocessing as mp
import time
from dataclasses import dataclass
from typing import Dict, List, Optional

from ..env import ENV
from ..utils.logger import init_logger
from ..utils.mp import pick_free_ports
from .args import ServerArgs

logger = init_logger("supervisor")


@dataclass
class FrontendAddrs:
    to_tokenizer: str
    from_tokenizer: str


def _coordinator_main(server_args: ServerArgs, addrs: Dict[str, object], world: int, ready_evt, stop_evt) -> None:
    """Coordinator process: owns the schedulers; never touches a GPU."""
    import gc

    from ..config import get_model_config
    from ..coordinator import AfdCoordinator, CoordinatorError, ZmqWorkerTransport
    from ..message import AbortMsg, BatchDetokenizeMsg, DetokenizeMsg, ExitMsg, UserMsg
    from ..scheduler.lane import AdmissionError
    from ..utils.mp import ZmqPullQueue, ZmqPushQueue

    cfg = get_model_config(server_args.model_path)
    rt = server_args.runtime_config()
    topo = server_args.topology
    transport = ZmqWorkerTransport(addrs["cmd"], addrs["reply"])
    from_tok = ZmqPullQueue(addrs["tok_to_backend"], bind=True)
    to_tok = ZmqPushQueue(addrs["backend_to_tok"], bind=False)
    ready = transport.wait_ready(world, ENV.STARTUP_TIMEOUT_S.value)
    pages = [r.num_pages for r in ready if r.role == "attention"]
    comm = [r.info.get("max_comm_tokens", 2048) for r in ready]

    def emit(items):
        to_tok.put(BatchDetokenizeMsg([DetokenizeMsg(uid=u, token_ids=t, finished=f) for u, t, f in items]))

    from ..cad.config import CadConfig

    if CadConfig.from_env().enabled:          # FASTAFD_MODE=cad: decode steps with the attention core on the attention ranks only
        from ..cad.coordinator import CadCoordinator as Coordinator
    else:
        Coordinator = AfdCoordinator
    coord = Coordinator(cfg, rt, topo, transport, num_pages=min(pages), max_comm_tokens=min(comm), on_tokens=emit)
    coord.log_step_times = bool(ENV.STEP_TIMES.value)
    ready_evt.set()
    gc.disable()          # the hot loop allocates little; collector pauses would show up as step jitter
    try:
        while not stop_evt.is_set():
            msg = from_tok.get_nowait() if not coord.idle() else from_tok.get(timeout_ms=50)
            while msg is not None:
                if isinstance(msg, ExitMsg):
                    stop_evt.set()
                    break
                if isinstance(msg, UserMsg):
                    try:
                        coord.add_request(msg.uid, msg.input_ids, msg.sampling)
                    except (AdmissionError, CoordinatorError) as e:
                        to_tok.put(DetokenizeMsg(uid=msg.uid, token_ids=[], finished=True, error=str(e)))
                elif isinstance(msg, AbortMsg):
                    coord.abort(msg.uid)
                msg = from_tok.get_nowait()
            if stop_evt.is_set():
                break
            try:
                coord.step_loop_once(block=True)
            except CoordinatorError as e:
                logger.error(f"coordinator stops: {e}")
                for uid in list(coord.uid_lane):
                    to_tok.put(DetokenizeMsg(uid=uid, token_ids=[], finished=True, error=str(e)))
                break
            except AdmissionError as e:
                logger.error(str(e))
    finally:
        coord.shutdown()


def make_addresses(world: int, probe_host: str = "127.0.0.1", head_host: str = "127.0.0.1",
                   rank_hosts: Optional[Dict[int, str]] = None):
    """ZMQ endpoints of one server: a command queue per worker rank (bound on that rank's node),
    the shared reply queue and the tokenizer queues on the head node. Returns (addresses, ports);
    ports[world + 5] is the torch.distributed rendezvous port."""
    ports = pick_free_ports(world + 6, probe_host)
    rank_hosts = rank_hosts or {}
    tcp = lambda h, p: f"tcp://{h}:{p}"  # noqa: E731
    addrs = {
        "cmd": {r: tcp(rank_hosts.get(r, head_host), ports[r]) for r in range(world)},
        "reply": tcp(head_host, ports[world]),
        "front_to_tok": tcp(head_host, ports[world + 1]), "tok_to_front": tcp(head_host, ports[world + 2]),
        "tok_to_backend": tcp(head_host, ports[world + 3]), "backend_to_tok": tcp(head_host, ports[world + 4]),
        "master_addr": head_host,
    }
    return addrs, ports


def _child_entry(target, args) -> None:
    """Entry of every backend process: leave when the parent is gone (killed without running
    its shutdown), so that no worker outlives the server holding a GPU."""
    import multiprocessing as mp
    import os
    import threading

    parent = mp.parent_process()
    if parent is not None:
        def watch():
            parent.join()
            os._exit(1)
        threading.Thread(target=watch, name="parent-watch", daemon=True).start()
    target(*args)


class LocalSupervisor:
    def __init__(self, args: ServerArgs):
        self.args = args
        self.procs: List[mp.Process] = []
        self.names: Dict[int, str] = {}
        self._stopped = False
        self.ctx = mp.get_context("spawn")
        self.stop_evt = self.ctx.Event()
        self.addrs: Dict[str, object] = {}

    def start(self) -> FrontendAddrs:
        from ..config import get_model_config
        from ..tokenizer import tokenize_worker
        from ..worker.main import worker_main

        a = self.args
        world = a.topology.world
        self.addrs, ports = make_addresses(world, a.host if a.host != "0.0.0.0" else "127.0.0.1")
        master_port = ports[world + 5]
        for r in range(world):
            self._spawn(f"worker{r}", worker_main, (r, world, a, self.addrs, master_port))
        return self.start_frontend_side(self.addrs)

    def start_frontend_side(self, addrs: Dict[str, object]) -> FrontendAddrs:
        """Tokenizer and coordinator processes on this node; the workers are already starting
        (here, or as remote actors under the multi-node supervisor)."""
        from ..config import get_model_config
        from ..tokenizer import tokenize_worker

        a = self.args
        world = a.topology.world
        self.addrs = addrs
        cfg = get_model_config(a.model_path)
        rt = a.runtime_config()
        tok_ready, coord_ready = self.ctx.Event(), self.ctx.Event()
        self._spawn("tokenizer", tokenize_worker, (a.model_path, cfg.vocab_size, rt.max_seq_len or cfg.max_position,
                                                   self.addrs["front_to_tok"], self.addrs["tok_to_backend"],
                                                   self.addrs["backend_to_tok"], self.addrs["tok_to_front"], tok_ready))
        self._spawn("coordinator", _coordinator_main, (a, self.addrs, world, coord_ready, self.stop_evt))
        deadline = time.monotonic() + ENV.STARTUP_TIMEOUT_S.value
        while not (tok_ready.is_set() and coord_ready.is_set()):
            dead = self.get_failures()
            if dead:
                self.shutdown()
                raise RuntimeError(f"process died during start-up: {', '.join(dead)}")
            if time.monotonic() > deadline:
                self.shutdown()
                raise TimeoutError("backend did not become ready in time")
            time.sleep(0.2)
        logger.info(f"backend ready: {world} worker(s), topology {a.topology}")
        return FrontendAddrs(self.addrs["front_to_tok"], self.addrs["tok_to_front"])

    def _spawn(self, name: str, target, args) -> None:
        p = self.ctx.Process(target=_child_entry, args=(target, args), name=name, daemon=True)
        p.start()
        self.names[p.pid] = name
        self.procs.append(p)
        if getattr(self.args, "pid_file", ""):
            from .stop import load, record_process

            if not any(e.get("pid") == os.getpid() for e in load(self.args.pid_file)):
                record_process(self.args.pid_file, os.getpid(), "server")       # the front end itself, ended last
            record_process(self.args.pid_file, p.pid, name)

    def get_failures(self) -> List[str]:
        """Names of processes that exited although nobody asked them to."""
        if self._stopped:
            return []
        return [f"{p.name} (exit code {p.exitcode})" for p in self.procs if p.exitcode is not None]

    def shutdown(self) -> None:
        if self._stopped:
            return
        self._stopped = True
        self.stop_evt.set()
        try:
            from ..message import ExitMsg
            from ..utils.mp import ZmqPushQueue

            q = ZmqPushQueue(self.addrs["front_to_tok"], bind=False)
            q.put(ExitMsg("shutdown"))
            q.close()
        except Exception:
            pass
        deadline = time.monotonic() + 5.0
        for p in self.procs:
            p.join(max(0.0, deadline - time.monotonic()))
        for p in self.procs:
            if p.is_alive():
                p.terminate()
        for p in self.procs:
            p.join(2.0)
            if p.is_alive():
                p.kill()


def create_backend_supervisor(args: ServerArgs):
    """`--launch-backend mp` (default): processes on this node; `ray`: one actor per rank across a
    Ray cluster (raises where Ray is not installed)."""
    if getattr(args, "launch_backend", "mp") == "ray":
        from .supervisor_ray import RaySupervisor

        return RaySupervisor(args)
    return LocalSupervisor(args)
