"""Multi-node launch of the AFD workers as Ray actors.

The planning half is pure Python and runs anywhere: which node and GPU each rank gets
(`plan_placement`), which environment variables travel to the actors (`actor_env`), and whether
the nodes report compatible runtimes (`check_runtime_versions`). The launching half
(`RaySupervisor`) imports Ray on use; where Ray is not installed it raises `RayUnavailable`
naming the local supervisor as the alternative.

Placement rules: attention ranks fill nodes first, expert ranks after them, a TP group never
straddles nodes, the head node (this process) is preferred for rank 0, and nodes are taken in a
stable order (head first, then by address) so that every launch of the same cluster gives the
same plan.

Reference: python/minisgl/server/supervisor_ray.py (rank plan :54-100, env forwarding, version
guard), python/minisgl/ray_env_keys.py (the forwarded-key registry),
python/minisgl/afd_worker_launcher.py:26 (placement of AG / EG workers).
"""
from __future__ import annotations

import os
from dataclasses import dataclass, field
from typing import Dict, Iterable, List, Mapping, Optional, Sequence, Tuple

from ..protocol import AfdTopology

# Environment that an actor needs to behave like the driver process. Prefix rules cover the knob
# families; the explicit names are the ones outside those families.
FORWARDED_ENV_PREFIXES: Tuple[str, ...] = ("FASTAFD_", "MINISGL_", "NCCL_", "TORCH_NCCL_", "CUDA_DEVICE_", "HF_", "TRANSFORMERS_")
FORWARDED_ENV_KEYS: Tuple[str, ...] = ("CUDA_HOME", "CUDA_MODULE_LOADING", "LD_LIBRARY_PATH", "PYTHONPATH", "TOKENIZERS_PARALLELISM",
                                       "OMP_NUM_THREADS", "GLOO_SOCKET_IFNAME", "MASTER_ADDR", "MASTER_PORT")
# Never forwarded: Ray assigns the GPUs of an actor itself, and the caches are per node.
NODE_SCOPED_ENV_KEYS: Tuple[str, ...] = ("CUDA_VISIBLE_DEVICES", "TORCH_EXTENSIONS_DIR", "TRITON_CACHE_DIR", "TMPDIR",
                                         "FASTAFD_LOG_DIR")


class RayUnavailable(RuntimeError):
    pass


@dataclass(frozen=True)
class NodeReport:
    """What a node says about itself before placement."""
    address: str
    gpus: int
    is_head: bool = False
    versions: Mapping[str, str] = field(default_factory=dict)   # e.g. {"torch": ..., "cuda": ..., "driver": ..., "package": ...}


@dataclass(frozen=True)
class Slot:
    rank: int
    role: str            # "attention" | "expert"
    node: str
    gpu: int


def order_nodes(nodes: Iterable[NodeReport]) -> List[NodeReport]:
    return sorted((n for n in nodes if n.gpus > 0), key=lambda n: (not n.is_head, n.address))


def plan_placement(nodes: Sequence[NodeReport], topo: AfdTopology) -> List[Slot]:
    """One slot per rank of the union world (attention ranks first, then expert ranks)."""
    free = [[n.address, list(range(n.gpus))] for n in order_nodes(nodes)]
    total = sum(len(g) for _, g in free)
    if total < topo.world:
        raise ValueError(f"{topo.world} ranks need {topo.world} GPUs, the cluster reports {total}")
    slots: List[Slot] = []

    def take(count: int, role: str, first_rank: int) -> None:
        """`count` consecutive ranks on one node (a TP group, or a single rank)."""
        for entry in free:
            if len(entry[1]) >= count:
                for i in range(count):
                    slots.append(Slot(first_rank + i, role, entry[0], entry[1].pop(0)))
                return
        raise ValueError(f"no node has {count} free GPUs for {role} ranks {first_rank}..{first_rank + count - 1} "
                         f"(a tensor-parallel group must stay on one node)")

    rank = 0
    for _lane in range(topo.attn_dp):
        take(topo.attn_tp, "attention", rank)
        rank += topo.attn_tp
    for _ in range(topo.mlp_world):
        take(1, "expert", rank)
        rank += 1
    return slots


def actor_env(env: Optional[Mapping[str, str]] = None, extra_keys: Sequence[str] = ()) -> Dict[str, str]:
    """The part of `env` (default: this process's) that every actor receives."""
    env = os.environ if env is None else env
    out = {}
    for k, v in env.items():
        if k in NODE_SCOPED_ENV_KEYS:
            continue
        if k in FORWARDED_ENV_KEYS or k in extra_keys or any(k.startswith(p) for p in FORWARDED_ENV_PREFIXES):
            out[k] = v
    return out


CACHE_ENV_KEYS: Tuple[str, ...] = ("TVM_FFI_CACHE_DIR", "FLASHINFER_WORKSPACE_BASE", "XDG_CACHE_HOME", "CUDA_CACHE_PATH")


def nsys_prefix(ray_log_dir: str = "", output_prefix: str = "") -> str:
    """Where a rank's Nsight Systems report goes: the explicit prefix, else <ray-log-dir>/nsys/fastafd,
    else fastafd-ray (in the actor's working directory). The rank number is appended per actor."""
    if output_prefix:
        return output_prefix
    return os.path.join(ray_log_dir, "nsys", "fastafd") if ray_log_dir else "fastafd-ray"


def actor_options(slot: "Slot", env: Mapping[str, str], *, ray_log_dir: str = "", ray_nsys: bool = False,
                  nsys_output_prefix: str = "", node_scoped_cache: bool = False) -> Dict[str, object]:
    """Ray options of one rank's actor: pinned to its node, the forwarded environment, the rank's log
    file when a log directory is given, an `nsys` runtime-env entry when profiling is on, and - with
    node-scoped caches - without the driver's cache directories (every node then builds its own)."""
    env = {k: v for k, v in env.items() if not (node_scoped_cache and k in CACHE_ENV_KEYS)}
    if ray_log_dir:
        env["FASTAFD_LOG_DIR"] = ray_log_dir
        env["FASTAFD_RANK_LOG"] = os.path.join(ray_log_dir, f"rank{slot.rank}.log")
    runtime_env: Dict[str, object] = {"env_vars": env}
    if ray_nsys:
        runtime_env["nsight"] = {"o": f"{nsys_prefix(ray_log_dir, nsys_output_prefix)}-rank{slot.rank}", "t": "cuda,nvtx",
                                 "cuda-graph-trace": "node"}
    return {"resources": {f"node:{slot.node}": 0.001}, "runtime_env": runtime_env}


def check_runtime_versions(nodes: Sequence[NodeReport], keys: Sequence[str] = ("torch", "cuda", "package")) -> List[str]:
    """Problems that would make ranks disagree at run time: differing versions of the named
    components between nodes. Returns human-readable lines (empty = compatible)."""
    problems = []
    nodes = list(nodes)
    if not nodes:
        return ["no nodes reported"]
    head = next((n for n in nodes if n.is_head), nodes[0])
    for k in keys:
        want = head.versions.get(k)
        for n in nodes:
            got = n.versions.get(k)
            if got != want:
                problems.append(f"{k}: node {n.address} has {got!r}, head {head.address} has {want!r}")
    return problems


def local_report(is_head: bool = True) -> NodeReport:
    """This node's report (runs inside a probe task on every node)."""
    import socket

    import torch

    from .. import __version__ as pkg_version
    gpus = torch.cuda.device_count() if torch.cuda.is_available() else 0
    return NodeReport(address=socket.gethostbyname(socket.gethostname()) if not is_head else "127.0.0.1", gpus=gpus,
                      is_head=is_head, versions={"torch": torch.__version__, "cuda": str(torch.version.cuda), "package": pkg_version})


class RaySupervisor:
    """Starts one Ray actor per rank according to `plan_placement` and runs the worker entry in
    each. Construction fails with `RayUnavailable` where Ray cannot be imported."""

    def __init__(self, server_args, address: Optional[str] = None):
        try:
            import ray  # noqa: F401
        except ImportError as e:
            raise RayUnavailable("Ray is not installed: use --launch-backend mp (one node) or install ray") from e
        self.ray = ray
        self.args = server_args
        self.address = (address or os.environ.get("FASTAFD_RAY_ADDRESS") or os.environ.get("MINISGL_RAY_ADDRESS")
                        or getattr(server_args, "ray_address", "") or "auto")
        self.actors: List[object] = []
        self.plan: List[Slot] = []

    def reports(self) -> List[NodeReport]:
        ray = self.ray
        if not ray.is_initialized():
            ray.init(address=self.address, ignore_reinit_error=True)
        head_ip = ray.util.get_node_ip_address()
        out = []
        for n in ray.nodes():
            if n.get("Alive"):
                ip = n.get("NodeManagerAddress")
                out.append(NodeReport(address=ip, gpus=int(n.get("Resources", {}).get("GPU", 0)), is_head=(ip == head_ip)))
        return out

    def start(self):
        """Place the ranks, start one actor per rank, and run the tokenizer and the coordinator on
        the head node (this process's node) like the local supervisor does."""
        from ..worker.main import worker_main
        from .supervisor import LocalSupervisor, make_addresses

        ray = self.ray
        topo = self.args.topology
        nodes = self.reports()
        self.plan = plan_placement(nodes, topo)
        head = getattr(self.args, "control_host", "") or next((n.address for n in nodes if n.is_head), self.plan[0].node)
        if head == "127.0.0.1" and len({sl.node for sl in self.plan}) > 1:     # more than one node: a routable address
            head = next((n.address for n in nodes if n.is_head), self.plan[0].node)
        addrs, ports = make_addresses(topo.world, head, head, {s.rank: s.node for s in self.plan})
        env = actor_env()

        @ray.remote(num_gpus=1)
        class _Rank:
            def run(self, rank, world, args, addresses, port):
                return worker_main(rank, world, args, addresses, port)

        a = self.args
        for s in self.plan:
            opts = actor_options(s, env, ray_log_dir=getattr(a, "ray_log_dir", ""), ray_nsys=getattr(a, "ray_nsys", False),
                                 nsys_output_prefix=getattr(a, "ray_nsys_output_prefix", ""),
                                 node_scoped_cache=getattr(a, "ray_node_scoped_cache", False))
            actor = _Rank.options(**opts).remote()
            self.actors.append((actor, actor.run.remote(s.rank, topo.world, self.args, addrs, ports[topo.world + 5])))
        self.local = LocalSupervisor(self.args)
        return self.local.start_frontend_side(addrs)

    def shutdown(self) -> None:
        if getattr(self, "local", None) is not None:
            self.local.shutdown()
        for actor, _ in self.actors:
            try:
                self.ray.kill(actor)
            except Exception:
                pass
        self.actors = []
