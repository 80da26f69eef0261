"""Command line of the server: ``python -m fastafd_b200 --mode afd-serve --model-path ...``.

Flag names follow the reference CLI (scripts/serve/fastafd_server.sh:9-43,
python/minisgl/server/args.py:15-113,213-792) so that launch scripts carry over; flags that
selected among the reference's interchangeable back ends are accepted and checked but select
nothing here (there is one implementation per path).
"""
from __future__ import annotations

import argparse
from dataclasses import dataclass
from typing import Optional, Sequence, Tuple

from ..config import RuntimeConfig, get_model_config
from ..protocol import AfdTopology, validate_parallel_args


@dataclass
class ServerArgs:
    mode: str = "afd-serve"              # serve (colocated) | afd-serve
    model_path: str = "tiny-qwen3-moe"
    host: str = "127.0.0.1"
    port: int = 1919
    launch_backend: str = "mp"           # mp | ray (ray is accepted only when importable)
    ray_address: str = "auto"            # cluster address for --launch-backend ray
    ray_log_dir: str = ""                # per-rank actor logs (empty: Ray's own log directory)
    ray_nsys: bool = False               # profile every rank's actor with Nsight Systems
    ray_nsys_output_prefix: str = ""     # default <ray-log-dir>/nsys/fastafd, else fastafd-ray
    ray_node_scoped_cache: bool = False  # keep compile / kernel caches per node instead of forwarding the driver's
    control_host: str = "127.0.0.1"      # driver address for control sockets and the rendezvous
    afd_attn_dp_size: int = 1
    afd_attn_tp_size: int = 1
    afd_mlp_dp_size: int = 1
    afd_mlp_tp_size: int = 1
    afd_mlp_ep_size: int = 1
    afd_moe_a2a_backend: str = "none"
    afd_moe_runner_backend: str = "auto"
    afd_batch_size: int = 0
    afd_max_batched_tokens: int = 8192
    afd_max_running_requests: int = 256
    afd_max_new_tokens: int = 1024
    afd_decode_graph_bs: Tuple[int, ...] = ()
    afd_num_mb: int = 1
    afd_async_pending_steps: int = 3
    afd_disable_overlap: bool = False
    afd_force_multi_mb_graph_overlap: bool = False
    afd_device_comm_num_sms: int = 0
    cache_type: str = "naive"
    cuda_graph_max_bs: int = 256
    page_size: int = 16
    num_pages: int = 0
    max_seq_len_override: int = 0
    attention_backend: str = "auto"
    memory_ratio: float = 0.9
    device: str = "cuda"
    dtype: str = "bfloat16"
    dummy_weights: bool = False
    disable_cuda_graph: bool = False
    num_tokenizers: int = 1
    spec_block: int = 0
    spec_draft_path: str = ""
    seed: int = 0
    tp_size: int = 1                     # colocated tensor parallelism of the reference; here TP belongs to afd-serve lanes
    shell_mode: bool = False             # an interactive shell on the started backend instead of the HTTP server
    model_source: str = "huggingface"    # accepted for compatibility: models are read from local directories only
    moe_backend: str = "auto"            # accepted for compatibility: one expert path (tcgen05 grouped GEMM)
    disable_pynccl: bool = False         # TP collectives without the own NCCL communicator (= FASTAFD_TP_FUSED=1 only)
    distributed_timeout: float = 0.0     # seconds for the workers' host-side process group: rendezvous and blocking receives (0: library default)
    afd_disable_attention_decode_graph: bool = False
    afd_disable_model_decode_graph: bool = False
    # runtime replay: prompts given on the command line run through the started backend once, the
    # continuations go to a sample bundle (what the alignment scripts score), then the process leaves
    afd_prompt: Tuple[str, ...] = ()
    afd_prompt_file: str = ""
    afd_prompt_repeat: int = 1
    afd_report_dir: str = ""
    afd_sample_json: str = ""
    pid_file: str = ""                   # the supervisor records its processes here; `python -m fastafd_b200.server.stop` ends exactly those
    log_level: str = "INFO"

    @property
    def topology(self) -> AfdTopology:
        if self.mode == "serve":
            return AfdTopology(colocated=True)
        return AfdTopology(self.afd_attn_dp_size, self.afd_attn_tp_size, self.afd_mlp_dp_size,
                           self.afd_mlp_tp_size, self.afd_mlp_ep_size)

    def runtime_config(self) -> RuntimeConfig:
        cfg = get_model_config(self.model_path)
        return RuntimeConfig(
            model_path=self.model_path, attn_dp=self.afd_attn_dp_size, attn_tp=self.afd_attn_tp_size,
            mlp_dp=self.afd_mlp_dp_size, mlp_tp=self.afd_mlp_tp_size, mlp_ep=self.afd_mlp_ep_size,
            num_mb=self.afd_num_mb, async_pending_steps=self.afd_async_pending_steps,
            disable_overlap=self.afd_disable_overlap, page_size=self.page_size, num_pages=self.num_pages,
            memory_ratio=self.memory_ratio, max_running_requests=self.afd_max_running_requests,
            max_batched_tokens=self.afd_max_batched_tokens,
            max_seq_len=self.max_seq_len_override or min(cfg.max_position, 32768),
            max_new_tokens=self.afd_max_new_tokens, decode_graph_bs=self.afd_decode_graph_bs,
            cuda_graph_max_bs=min(self.cuda_graph_max_bs, max(1, self.afd_max_running_requests)),
            cache_type=self.cache_type, use_cuda_graph=not self.disable_cuda_graph and self.device == "cuda",
            spec_block=self.spec_block, spec_draft_path=self.spec_draft_path, seed=self.seed,
            dummy_weights=self.dummy_weights, dtype=self.dtype if self.device == "cuda" else "float32",
            device=self.device)


def _int_list(s: str) -> Tuple[int, ...]:
    return tuple(int(x) for x in s.replace(",", " ").split() if x)


def validate(args: ServerArgs) -> None:
    """Mutual consistency of the parallel sizes and back-end switches."""
    if args.mode not in ("serve", "afd-serve"):
        raise ValueError("--mode must be serve or afd-serve")
    if args.launch_backend not in ("mp", "ray"):
        raise ValueError("--launch-backend must be mp or ray")
    if args.tp_size != 1:
        raise ValueError("--tensor-parallel-size: the colocated mode runs on one GPU; tensor parallelism is "
                         "--afd-attn-tp-size under --mode afd-serve")
    if args.afd_prompt_repeat < 1:
        raise ValueError("--afd-prompt-repeat must be at least 1")
    if args.afd_disable_attention_decode_graph or args.afd_disable_model_decode_graph:
        args.disable_cuda_graph = True          # one graph per decode bucket holds both sides' work here
    if args.ray_nsys:
        # preflight: a profile that cannot start must stop the launch, not a rank later
        import shutil

        if args.launch_backend != "ray":
            raise ValueError("--ray-nsys needs --launch-backend ray")
        if shutil.which("nsys") is None:
            raise ValueError("--ray-nsys: Nsight Systems (nsys) is not installed on this node")
    if args.launch_backend == "ray":
        try:
            import ray  # noqa: F401
        except ImportError as e:
            raise ValueError("--launch-backend ray needs the ray package; use mp (one process per GPU)") from e
    if args.afd_moe_a2a_backend not in ("none", "deepep"):
        raise ValueError("--afd-moe-a2a-backend must be none or deepep")
    if args.afd_moe_runner_backend not in ("auto", "triton", "triton_fp8", "triton_kernel", "deep_gemm"):
        raise ValueError("unknown --afd-moe-runner-backend")
    if args.cache_type not in ("naive", "radix"):
        raise ValueError("--cache-type must be naive or radix")
    if args.page_size & (args.page_size - 1):
        raise ValueError("--page-size must be a power of two")
    if not 1 <= args.afd_num_mb <= 4:
        raise ValueError("--afd-num-mb must be between 1 and 4")
    from ..spec.config import SpecConfig
    spec = SpecConfig.from_env(args.spec_block, args.spec_draft_path)     # FASTAFD_SPEC* may switch it on without flags
    if spec.enabled:
        args.spec_block, args.spec_draft_path = spec.block, spec.draft_path
    if args.spec_block and args.afd_attn_tp_size != 1:
        raise ValueError("speculative decoding needs attention TP 1")
    if args.spec_block and args.cache_type != "naive":
        raise ValueError("speculative decoding needs --cache-type naive")
    cfg = get_model_config(args.model_path)
    if args.mode == "afd-serve":
        topo = args.topology      # raises on bad ep / tp combinations
        if not cfg.is_moe:
            raise ValueError("afd-serve needs a mixture-of-experts model; use --mode serve for dense models")
        validate_parallel_args(topo, cfg.num_experts, cfg.num_q_heads, cfg.num_kv_heads,
                               cfg.gdn_num_k_heads if cfg.num_linear_layers else 0,
                               cfg.gdn_num_v_heads if cfg.num_linear_layers else 0)


def build_parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser("fastafd_b200", description="B200-native AFD MoE serving")
    d = ServerArgs()
    p.add_argument("--mode", default=d.mode, choices=["serve", "afd-serve"])
    p.add_argument("--model-path", "--model", dest="model_path", default=d.model_path)
    p.add_argument("--host", default=d.host)
    p.add_argument("--port", type=int, default=d.port)
    p.add_argument("--launch-backend", default=d.launch_backend)
    p.add_argument("--ray-address", default=d.ray_address, help="Ray cluster address (--launch-backend ray)")
    p.add_argument("--ray-log-dir", default=d.ray_log_dir, help="directory for per-rank actor logs")
    p.add_argument("--ray-nsys", action="store_true", help="profile every rank's actor with Nsight Systems")
    p.add_argument("--ray-nsys-output-prefix", default=d.ray_nsys_output_prefix,
                   help="default: <ray-log-dir>/nsys/fastafd when --ray-log-dir is set, else fastafd-ray")
    p.add_argument("--ray-node-scoped-cache", action="store_true",
                   help="every node keeps its own compile / kernel caches (the driver's cache paths are not forwarded)")
    p.add_argument("--control-host", default=d.control_host, help="driver address for control sockets and the rendezvous")
    for name in ("attn-dp", "mlp-dp", "attn-tp", "mlp-tp", "mlp-ep"):
        p.add_argument(f"--afd-{name}-size", type=int, default=1)
    p.add_argument("--afd-moe-a2a-backend", default=d.afd_moe_a2a_backend)
    p.add_argument("--afd-moe-runner-backend", default=d.afd_moe_runner_backend)
    p.add_argument("--afd-batch-size", type=int, default=0)
    p.add_argument("--afd-max-batched-tokens", "--max-extend-length", "--max-prefill-length", dest="afd_max_batched_tokens",
                   type=int, default=d.afd_max_batched_tokens, help="tokens of one step (the chunk size of chunked prefill)")
    p.add_argument("--afd-max-running-requests", "--max-running-requests", dest="afd_max_running_requests", type=int,
                   default=d.afd_max_running_requests)
    p.add_argument("--afd-max-new-tokens", type=int, default=d.afd_max_new_tokens)
    p.add_argument("--afd-decode-graph-bs", type=_int_list, default=())
    p.add_argument("--afd-num-mb", type=int, default=d.afd_num_mb)
    p.add_argument("--afd-async-pending-steps", type=int, default=d.afd_async_pending_steps)
    p.add_argument("--afd-disable-overlap", action="store_true")
    p.add_argument("--afd-force-multi-mb-graph-overlap", action="store_true")
    p.add_argument("--afd-device-comm-num-sms", type=int, default=0)
    p.add_argument("--cache-type", default=d.cache_type)
    p.add_argument("--cuda-graph-max-bs", "--graph", dest="cuda_graph_max_bs", type=int, default=d.cuda_graph_max_bs)
    p.add_argument("--page-size", type=int, default=d.page_size)
    p.add_argument("--num-pages", type=int, default=0)
    p.add_argument("--max-seq-len-override", type=int, default=0)
    p.add_argument("--attention-backend", "--attn", dest="attention_backend", default="auto")
    p.add_argument("--memory-ratio", type=float, default=d.memory_ratio)
    p.add_argument("--device", default=d.device)
    p.add_argument("--dtype", default=d.dtype)
    p.add_argument("--dummy-weights", "--dummy-weight", dest="dummy_weights", action="store_true")
    p.add_argument("--disable-cuda-graph", action="store_true")
    p.add_argument("--num-tokenizers", "--num-tokenizer", "--tokenizer-count", dest="num_tokenizers", type=int, default=1)
    p.add_argument("--spec-block", type=int, default=0)
    p.add_argument("--spec-draft-path", default="")
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--tensor-parallel-size", "--tp-size", dest="tp_size", type=int, default=1,
                   help="the reference's colocated TP size; here 1 (tensor parallelism is --afd-attn-tp-size under afd-serve)")
    p.add_argument("--shell-mode", action="store_true", help="interactive shell on the started backend instead of HTTP")
    p.add_argument("--model-source", default=d.model_source, choices=["huggingface", "modelscope"])
    p.add_argument("--moe-backend", default=d.moe_backend)
    p.add_argument("--disable-pynccl", action="store_true")
    p.add_argument("--distributed-timeout", type=float, default=0.0)
    p.add_argument("--afd-disable-attention-decode-graph", action="store_true")
    p.add_argument("--afd-disable-model-decode-graph", action="store_true")
    p.add_argument("--afd-prompt", action="append", default=[], help="runtime prompt text (repeatable)")
    p.add_argument("--afd-prompt-file", default="", help="UTF-8 file, one runtime prompt per line")
    p.add_argument("--afd-prompt-repeat", type=int, default=1)
    p.add_argument("--afd-report-dir", default="")
    p.add_argument("--afd-sample-json", default="", help="where the runtime replay writes its sample bundle")
    p.add_argument("--pid-file", default="", help="record the backend's process ids here (see fastafd_b200.server.stop)")
    p.add_argument("--log-level", default="INFO")
    return p


def parse_args(argv: Optional[Sequence[str]] = None) -> ServerArgs:
    ns = build_parser().parse_args(argv)
    ns.afd_prompt = tuple(ns.afd_prompt)
    args = ServerArgs(**{k: v for k, v in vars(ns).items() if k in ServerArgs.__dataclass_fields__})
    if args.afd_batch_size and not args.afd_decode_graph_bs:
        args.afd_decode_graph_bs = (args.afd_batch_size,)
    validate(args)
    return args
