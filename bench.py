#!/usr/bin/env python
"""Headline benchmark: steady-state decode throughput of Attention-FFN-disaggregated MoE serving.

    python bench.py --gpus N --steps K --warmup W            # N = 1: single process
    python -m torch.distributed.run --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 \
        --master-port P bench.py --gpus N --steps K --warmup W

Layout: N = 1 runs attention and expert stages on one GPU; N >= 2 splits the GPUs into N/2
attention ranks and N/2 expert ranks (expert-parallel). The attention ranks are data-parallel
lanes at N = 2 and 4 and one tensor-parallel lane at N = 8 (attention TP4 + MLP EP4, the
configuration the benchmark is named for; --attn-tp 1 gives four data-parallel lanes). The number
of micro-batches comes from `pick_num_mb`. Per-attention-GPU batch is fixed (weak scaling). Data: synthetic - random-init
weights of the named architecture, KV cache of `--context` tokens per request filled with
random values, random token ids.

Two numbers are produced:
  value : K decode steps queued back to back and timed on the device with CUDA events
          (max over ranks).
  e2e   : the same K steps through the public engine API in its serving mode (one step ahead):
          plan on the host, copy the step's inputs from pinned host memory, replay, read the
          sampled tokens back to the host; `lock_step` is the same with nothing of step n+1 started
          before step n's tokens are on the host.
Prints one JSON line on rank 0.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

# Published reference numbers (GB200 NVL72, 4 attention + 4 FFN GPUs, scripts/benchmark/configs.json:366), tok/s/GPU.
PUBLISHED_TOK_S_PER_GPU = {"qwen3-235b-a22b-fp8": 1542.0}
# the same model with EAGLE-3, 3 draft tokens, 4K context, 194 requests per attention GPU (configs.json:403)
PUBLISHED_SPEC_TOK_S_PER_GPU = {("qwen3-235b-a22b-fp8", 4): 3764.0}
METRIC = ("decode tok/s of the whole job, AFD attention + expert GPUs on N x B200, max over ranks "
          "(per-GPU decode tok/s: per_gpu_tok_s; TPOT p50: tpot_p50_ms; N2M/M2N GB/s: n2m_m2n)")


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--model", default="qwen3-30b-a3b")
    ap.add_argument("--batch-per-attn-gpu", type=int, default=64)
    ap.add_argument("--context", type=int, default=1024)
    ap.add_argument("--num-mb", type=int, default=0, help="micro-batches in flight; 0 = 1 when colocated or with a single expert GPU, else 2")
    ap.add_argument("--block-tok", type=int, default=16)
    ap.add_argument("--layers", type=int, default=0, help="debug only: truncate the model (marks the result invalid)")
    ap.add_argument("--no-graph", action="store_true")
    ap.add_argument("--attn-gpus", type=int, default=0, help="attention GPUs of the N (0 = N/2, the 1:1 split)")
    ap.add_argument("--attn-tp", type=int, default=0,
                    help="tensor-parallel size of an attention lane (0 = the named configuration: one TP-4 lane on "
                         "8 GPUs, data-parallel lanes otherwise; 1 = data-parallel lanes)")
    ap.add_argument("--router-bias", default="", help="zipf:S - router selection bias drawn so that expert popularity follows "
                                                      "Zipf(S) (models with a selection bias, e.g. minimax-m2.5-fp8)")
    ap.add_argument("--also-router-bias", default="", help="after the main measurement, apply this router bias (zipf:S) in the "
                                                           "same process and time the decode steps again (extra JSON field)")
    ap.add_argument("--spec-block", type=int, default=0, help="speculative decoding: verified tokens per step (drafts + 1)")
    ap.add_argument("--spec-sim-accept", type=float, default=0.0, help="fixed mean acceptance (tokens per verify step) for timing runs")
    return ap.parse_args()


def reference_arm(args) -> None:
    """Runs the unmodified reference (baseline/_ref) through its own offline API; see
    baseline/reference_arm.py. Prints the same JSON line with "impl": "reference", or an
    "unavailable" line whose reason is the text of the failed attempt."""
    sys.path.insert(0, os.path.join(HERE, "baseline"))
    import reference_arm as ref

    args.metric = METRIC
    out = ref.run(args, clock_sampler_cls=ClockSampler)
    if int(os.environ.get("RANK", "0")) == 0:
        print(json.dumps(out), flush=True)


def default_attn_tp(world: int, attn_gpus: int = 0) -> int:
    """Tensor-parallel size of an attention lane when the caller names none. 8 GPUs split 4+4: one TP-4
    lane + EP-4, the configuration the benchmark is named for (it runs with the fused collectives;
    attention DP4, --attn-tp 1, measured 6.66 against 7.85 ms/step on Qwen3-30B-A3B). Otherwise
    data-parallel lanes."""
    return 4 if (world == 8 and attn_gpus in (0, 4)) else 1


def pick_num_mb(cfg, topo, batch_per_attn_gpu: int, context: int) -> int:
    """1 or 2 micro-batches from a two-term model of a layer (times in us, constants fitted to the
    device timelines measured on B200). A second micro-batch hides the expert round trip behind the
    other one's attention, but every micro-batch streams the expert weights again, so it pays only
    when an expert GPU's weight stream per pass is short next to the attention-side chain:
        chain(b)  = 35 + KV bytes of b requests / 5.0 TB/s      attention GPU, one micro-batch of b requests
        expert    = 12 + local expert bytes / 6.0 TB/s          expert GPU, one pass over its experts
        2 micro-batches: max(2 x expert, chain(b/2) + expert + 20)   per layer
        1 micro-batch  : chain(b) + expert + 20
    Measured (Qwen3-30B-A3B, 64 requests per attention GPU): 1+1 GPUs 12.7 ms with 1 against 16.8 ms with 2;
    2+2 GPUs 8.9 ms with 1 against 10.1 ms with 2; 4+4 GPUs (attention DP4) 6.66 ms with 2 against 6.92 ms with 1."""
    if topo.colocated or not cfg.is_moe:
        return 1
    wbytes = 1 if cfg.quant.is_fp8 else 2
    e_local = (cfg.num_experts + topo.mlp_ep - 1) // topo.mlp_ep
    expert_us = 12 + e_local * 3 * cfg.moe_intermediate_size * cfg.hidden_size * wbytes / 6.0e6
    kv_per_req = context * max(1, cfg.num_kv_heads // topo.attn_tp) * cfg.head_dim * 2 * 2 * (
        cfg.num_full_attn_layers / max(cfg.num_layers, 1))

    def chain(b):
        return 35 + b * kv_per_req / 5.0e6

    b = batch_per_attn_gpu
    two = max(2 * expert_us, chain(b / 2) + expert_us + 20)
    one = chain(b) + expert_us + 20
    return 2 if two < one else 1


def apply_router_bias(eng, cfg, spec: str) -> None:
    """`zipf:S`: the selection bias of every MoE layer is set so that expert popularity is skewed like a
    Zipf(S) law over the experts (a different expert order per layer): bias = popularity / max popularity,
    on the scale of the sigmoid scores it is added to."""
    import torch

    kind, _, val = spec.partition(":")
    if kind != "zipf" or not cfg.router_bias:
        raise SystemExit(f"--router-bias {spec}: needs zipf:S and a model whose router has a selection bias")
    if eng.attn is None:
        return
    s_exp, E = float(val or 1.2), cfg.num_experts
    pop = 1.0 / torch.arange(1, E + 1, dtype=torch.float32) ** s_exp
    g = torch.Generator().manual_seed(1234)
    for name, w in eng.attn.model.w.items():
        if name.endswith("mlp.gate.e_score_correction_bias"):
            w.copy_((pop / pop.max())[torch.randperm(E, generator=g)].to(w.device))


def summarize_clock_samples(lines, t0=None, t1=None) -> dict:
    """Median SM clock, maximum SM clock and the throttle reasons seen in nvidia-smi csv lines
    (timestamp, index, clocks.sm, clocks.max.sm, power, reasons.active, hw_slowdown, hw_thermal_slowdown,
    sw_thermal_slowdown, sw_power_cap). With [t0, t1] (epoch seconds) only the samples taken inside the
    timed region count; if the region was shorter than the sampling period, the nearest sample on each
    side stands in and `in_region` says 0."""
    import datetime

    rows = []
    for line in lines:
        f = [x.strip() for x in line.split(",")]
        if len(f) < 10:
            continue
        try:
            ts = datetime.datetime.strptime(f[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
            rows.append((ts, float(f[2]), float(f[3]), [v.lower().startswith("active") for v in f[6:10]]))
        except ValueError:
            continue
    out = {"sm_mhz": None, "sm_max_mhz": None, "reasons": []}
    if not rows:
        return out
    used, inside = rows, None
    if t0 is not None and t1 is not None:
        inside = [r for r in rows if t0 <= r[0] <= t1]
        used = inside
        if not used:
            before = [r for r in rows if r[0] < t0][-1:]
            after = [r for r in rows if r[0] > t1][:1]
            used = before + after or rows[-1:]
    names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
    reasons = sorted({n for r in used for n, on in zip(names, r[3]) if on})
    out = {"sm_mhz": statistics.median(r[1] for r in used), "sm_max_mhz": max(r[2] for r in used), "reasons": reasons,
           "samples": len(used)}
    if inside is not None:
        out["in_region"] = len(inside)
    return out


class ClockSampler:
    """nvidia-smi clock / throttle-reason samples of one GPU. The process is started early (nvidia-smi takes
    a few hundred ms to come up); `mark_start` / `mark_end` bracket the timed region and only samples
    between them are reported."""

    Q = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu_index, self.proc, self.path = gpu_index, None, None
        self.t0 = self.t1 = None

    def _gpu_id(self) -> str:
        try:        # the UUID survives a permuted CUDA_VISIBLE_DEVICES, the index does not
            import torch

            return "GPU-" + str(torch.cuda.get_device_properties(self.gpu_index).uuid)
        except Exception:
            return str(self.gpu_index)

    def _spawn(self, gpu_id: str):
        return subprocess.Popen(["nvidia-smi", "-i", gpu_id, f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                 "-lms", "25"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = self._spawn(self._gpu_id())
            time.sleep(0.2)
            if self.proc.poll() is not None:            # the id was refused: fall back to the plain index
                self.proc = self._spawn(str(self.gpu_index))
        except Exception:
            self.proc = None

    def mark_start(self):
        self.t0 = time.time()

    def mark_end(self):
        self.t1 = time.time()

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": []}
        if self.t1 is not None:
            time.sleep(0.06)            # one more sample behind the region
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        try:
            lines = open(self.path).read().splitlines()
            os.unlink(self.path)
        except Exception:
            lines = []
        try:
            return summarize_clock_samples(lines, self.t0, self.t1)
        except Exception as e:          # noqa: BLE001 - a clock record must never cost the measurement
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "error": f"{type(e).__name__}: {e}"}


def main():
    args = parse_args()
    if args.impl == "reference":
        return reference_arm(args)

    import torch
    import torch.distributed as dist

    from fastafd_b200.config import RuntimeConfig, get_model_config
    from fastafd_b200.engine import AfdEngine, SpmdDriver
    from fastafd_b200.ops import _lib
    from fastafd_b200.protocol import AfdTopology

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}: launch with torch.distributed.run for N > 1")
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    nccl_world = None
    if world > 1:
        # device-side timeline of the N2M / M2N exchange (a few timer stores per kernel): the measured
        # round-trip and expert-busy times behind the n2m_m2n figures
        os.environ.setdefault("FASTAFD_COMM_TRACE", "1")
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        # host-side group: plans, tokens, barriers (gloo). Device collectives use the framework's own
        # NCCL communicator and fabric kernels, so torch needs no NCCL group of its own here.
        dist.init_process_group(backend="gloo", rank=rank, world_size=world)
        # ... and an NCCL group over all ranks for the harness's own device collectives (the barriers
        # around the timed regions and the max over ranks travel over NVLink). It is a sub-group of a
        # gloo default group, created by every rank, first used after the engine is built.
        if os.environ.get("FASTAFD_BENCH_NCCL_WORLD", "1") == "1":
            try:
                nccl_world = dist.new_group(backend="nccl")
            except Exception as e:      # noqa: BLE001 - fall back to host barriers, say so
                print(f"[bench rank {rank}] no NCCL world group ({type(e).__name__}: {e}); host barriers", file=sys.stderr)

    t_start = time.time()
    # A step that cannot finish (a peer that never arrives) must end the run with an error and the
    # Python stacks of every thread, not hold the GPUs until someone kills the job.
    import faulthandler

    watchdog_s = float(os.environ.get("FASTAFD_BENCH_WATCHDOG_S", "240"))

    def phase(name: str) -> None:
        print(f"[bench rank {rank}] {name} at +{time.time() - t_start:.1f}s", file=sys.stderr, flush=True)
        if watchdog_s > 0:
            faulthandler.dump_traceback_later(watchdog_s, exit=True)

    phase("process group up")
    cfg = get_model_config(args.model)
    truncated = False
    if args.layers and args.layers < cfg.num_layers:
        cfg = cfg.with_layers(args.layers)
        truncated = True
    if args.attn_tp <= 0:
        args.attn_tp = default_attn_tp(world, args.attn_gpus)
    topo = AfdTopology.for_world(world, attn_tp=args.attn_tp, attn_gpus=args.attn_gpus)
    if args.num_mb <= 0:
        args.num_mb = pick_num_mb(cfg, topo, args.batch_per_attn_gpu, args.context)
    b = args.batch_per_attn_gpu
    tp = topo.attn_tp
    lane_b = b * tp                      # a TP lane serves tp GPUs' worth of requests
    per_mb = (lane_b + args.num_mb - 1) // args.num_mb
    per_mb = (per_mb + tp - 1) // tp * tp
    total_steps = (4 if args.also_router_bias else 3) * args.steps + 2 * args.warmup + 12
    q = args.spec_block if args.spec_block > 1 else 1
    if q > 1:
        os.environ["FASTAFD_SPEC_SIM_ACCEPT"] = str(args.spec_sim_accept or 0)
    rt = RuntimeConfig(model_path=args.model, num_mb=args.num_mb, page_size=16, max_running_requests=lane_b,
                       max_seq_len=args.context + total_steps * q + 4 * q + 16, cuda_graph_max_bs=per_mb,
                       decode_graph_bs=(per_mb,), use_cuda_graph=not args.no_graph, moe_block_tok=args.block_tok,
                       max_batched_tokens=per_mb * args.num_mb * q, device="cuda", flag_timeout_s=2.0,
                       spec_block=args.spec_block if q > 1 else 0)
    t_build = time.time()
    eng = AfdEngine(cfg, rt, topo, rank, device, group=None, seed=0, fast_init=True, max_comm_tokens=per_mb * q // tp)
    if args.router_bias:
        apply_router_bias(eng, cfg, args.router_bias)
    drv = SpmdDriver(eng)
    drv.install_prefilled(lane_b, args.context, max_tokens=total_steps * q + 4)
    torch.cuda.synchronize()
    build_s = time.time() - t_build

    phase("engine built")

    sync_word = torch.zeros(1, device=device) if world > 1 else None

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            if nccl_world is not None:
                dist.all_reduce(sync_word, group=nccl_world)      # every rank's GPU has reached this point
            else:
                dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        if nccl_world is not None:
            t = torch.tensor([x], dtype=torch.float64, device=device)
            dist.all_reduce(t, op=dist.ReduceOp.MAX, group=nccl_world)
            return float(t.item())
        t = torch.tensor([x], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t[0])

    # ---- warm-up (captures the graphs) -------------------------------------------------
    sampler = ClockSampler(local_rank)
    sampler.start()                     # up and sampling by the time the timed region starts
    drv.run_decode_steps(max(args.warmup, 3), pipelined=False)
    barrier()
    phase("warm-up done")

    # ---- device-timed region: K steps queued back to back --------------------------------
    launches0 = _lib.LAUNCHES["count"]
    graph_kernels = getattr(eng.attn, "graph_kernel_count", 0) if eng.attn else 0
    barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    stream = eng.attn.main_stream if eng.attn is not None else eng.expert.stream
    sampler.mark_start()
    ev0.record(stream)
    step_events = [ev0]
    drv.run_decode_steps(args.steps, pipelined=True, events=step_events, event_stream=stream)
    ev1.record(stream)
    torch.cuda.synchronize()
    sampler.mark_end()
    dev_ms = ev0.elapsed_time(ev1)
    per_step = sorted(step_events[i].elapsed_time(step_events[i + 1]) for i in range(len(step_events) - 1))
    tpot_p50 = per_step[len(per_step) // 2] if per_step else dev_ms / args.steps
    barrier()
    clocks = sampler.stop()
    dev_ms = max_over_ranks(dev_ms)
    tpot_p50 = max_over_ranks(tpot_p50)

    # ---- end-to-end region: one step at a time through the public API ----------------------
    phase("device-timed region done")
    barrier()
    t0 = time.perf_counter()
    drv.run_decode_steps(args.steps, pipelined=False)
    torch.cuda.synchronize()
    e2e_ms = (time.perf_counter() - t0) * 1e3
    barrier()
    e2e_ms = max_over_ranks(e2e_ms)
    # the same public call in the server's default mode: step n+1 is planned and its inputs are
    # copied while step n runs (one step ahead); every step still has its H2D and D2H copies
    barrier()
    t0 = time.perf_counter()
    drv.run_decode_steps(args.steps, pipelined=True)
    torch.cuda.synchronize()
    ahead_ms = (time.perf_counter() - t0) * 1e3
    barrier()
    ahead_ms = max_over_ranks(ahead_ms)
    status = eng.synchronize()
    phase("end-to-end regions done")
    skewed = None
    if args.also_router_bias:
        apply_router_bias(eng, cfg, args.also_router_bias)
        barrier()
        drv.run_decode_steps(3, pipelined=True)
        barrier()
        ev2, ev3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev2.record(stream)
        drv.run_decode_steps(args.steps, pipelined=True)
        ev3.record(stream)
        torch.cuda.synchronize()
        skew_ms = max_over_ranks(ev2.elapsed_time(ev3))
        barrier()
        status = status or eng.synchronize()
        skewed = {"router_bias": args.also_router_bias, "ms_per_step": round(skew_ms / args.steps, 4)}

    trace_info = None
    if os.environ.get("FASTAFD_COMM_TRACE") == "1" and cfg.is_moe:
        from fastafd_b200.moe.afd_moe import summarize_trace

        mine = []
        if eng.attn is not None and getattr(eng.attn.client, "ep", None) is not None and eng.attn.client.ep.trace:
            mine.append(("attention", [summarize_trace(t, "attention") for t in eng.attn.client.ep.trace]))
        if eng._server is not None and eng._server.ep.trace:
            mine.append(("expert", [summarize_trace(t, "expert") for t in eng._server.ep.trace]))
        if world > 1:
            allinfo = [None] * world
            dist.all_gather_object(allinfo, mine)
            trace_info = {f"rank{r}": v for r, v in enumerate(allinfo)}
        else:
            trace_info = {"rank0": mine}
    n_attn = 1 if topo.colocated else topo.attn_world
    tokens = b * n_attn * args.steps
    spec_info = None
    if q > 1:
        # a verify step commits the accepted drafts + 1 token per request: count what was committed
        acc = eng.attn.spec.mean_accept() if eng.attn is not None else 0.0
        if world > 1:
            t_acc = torch.tensor([acc], dtype=torch.float64)
            dist.all_reduce(t_acc, op=dist.ReduceOp.MAX)
            acc = float(t_acc[0])
        tokens = b * n_attn * args.steps * acc
        spec_info = {"block": q, "drafts": q - 1, "mean_tokens_per_step": round(acc, 3),
                     "acceptance": "simulated fixed mean" if args.spec_sim_accept else "greedy verification of a random-init draft head"}
    value = tokens / (dev_ms / 1e3)
    e2e_value = tokens / (e2e_ms / 1e3)
    kernels_per_step = 0
    if eng.attn is not None:
        kernels_per_step = eng.attn.kernels_per_step.get(per_mb, 0)
    elif eng.expert is not None:
        kernels_per_step = eng.expert.kernels_per_step
    h2d = d2h = 0
    if eng.attn is not None:
        h2d = 2 * per_mb * 4 * args.num_mb + 24 * ((b + 15) // 16)   # rows + seq_lens (+ page grants, amortised)
        d2h = per_mb * 4 * args.num_mb + 8
    published = PUBLISHED_SPEC_TOK_S_PER_GPU.get((args.model, q)) if q > 1 else PUBLISHED_TOK_S_PER_GPU.get(args.model)
    # N2M / M2N traffic of one attention GPU per step (bytes that cross NVLink; 0 when colocated):
    # up = one row per expert GPU that owns one of the token's experts (expectation under uniform
    # routing), down = one bf16 row per (token, k).
    comm = None
    if cfg.is_moe and not topo.colocated:
        n_eg, K, H = topo.mlp_ep, cfg.num_experts_per_tok, cfg.hidden_size
        moe_layers = sum(1 for l in range(cfg.num_layers) if cfg.is_moe_layer(l))
        row_up = H * (1 if cfg.quant.is_fp8 else 2) + (H // 128 * 4 if cfg.quant.is_fp8 else 0)
        copies = n_eg * (1.0 - (1.0 - 1.0 / n_eg) ** K)
        per_tok_up, per_tok_down = row_up * copies + K * 4 * n_eg, K * H * 2
        step_s = dev_ms / args.steps / 1e3
        if os.environ.get("FASTAFD_DIRECT", "1") != "0":
            per_tok_up = K * (row_up + 4)          # direct exchange: one row copy (+ meta word) per chosen expert
        comm = {"n2m_bytes_per_step_per_attn_gpu": int(moe_layers * b * per_tok_up),
                "m2n_bytes_per_step_per_attn_gpu": int(moe_layers * b * per_tok_down),
                "n2m_GB_s_avg_over_step": round(moe_layers * b * per_tok_up / step_s / 1e9, 2),
                "m2n_GB_s_avg_over_step": round(moe_layers * b * per_tok_down / step_s / 1e9, 2),
                "note": "bytes counted from the exchanged tensors; averaged over the whole step (the transfers ride in "
                        "the route kernel and the down-projection epilogue)"}
        if trace_info is not None:
            # measured on the device timeline: the part of a micro-batch's round trip through the expert
            # GPUs that is not expert compute = both transfers + flag latencies
            rt_us = [v["round_trip_us"] for info in trace_info.values() for role, lanes in info if role == "attention"
                     for v in lanes if v.get("round_trip_us")]
            busy_us = [v["busy_us"] for info in trace_info.values() for role, lanes in info if role == "expert"
                       for v in lanes if v.get("busy_us")]
            if rt_us and busy_us:
                exposed = max(statistics.median(rt_us) - statistics.median(busy_us), 1e-3)
                per_round = (per_tok_up + per_tok_down) * b / args.num_mb
                comm.update({"round_trip_us_median": round(statistics.median(rt_us), 2),
                             "expert_busy_us_median": round(statistics.median(busy_us), 2),
                             "exposed_exchange_us": round(exposed, 2),
                             "n2m_plus_m2n_GB_s_over_exposed_time": round(per_round / exposed / 1e3, 2)})
    if rank == 0:
        out = {
            "metric": METRIC, "value": round(value, 2), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": max(args.warmup, 3), "ms_per_step": round(dev_ms / args.steps, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": (round(value / world / published, 4) if published else None),
            "dtype": "fp8-block128 weights, bf16 attention/KV" if cfg.quant.is_fp8 else "bf16",
            "data": "synthetic (random-init weights, random KV cache and token ids)",
            "per_gpu_tok_s": round(value / world, 2),
            "tpot_ms": round(dev_ms / args.steps, 4), "tpot_p50_ms": round(tpot_p50, 4),
            "config": {"model": args.model, "global_batch": b * n_attn, "seq_len": args.context,
                       "decode_tokens_timed": args.steps, "micro_batches": args.num_mb, "page_size": 16,
                       "parallelism": "colocated-1gpu" if topo.colocated else (f"attn_dp{topo.attn_dp}" + (f"xtp{tp}" if tp > 1 else "") + f"+mlp_ep{topo.mlp_ep}"),
                       "l2": "per-step working set (expert weights + KV) is far larger than the 126 MB L2; no flush needed",
                       "attention_parallelism_note": "attention GPUs are data-parallel lanes by default; --attn-tp N makes a lane "
                                                     "tensor-parallel over N GPUs (token-sharded residual, collectives fused with the GEMMs)",
                       "layers": cfg.num_layers, "truncated_model": truncated},
            "clocks": clocks,
            # end to end through the public engine API in its serving mode (one step ahead): every step is
            # planned on the host, its inputs are copied from pinned memory, the graph is replayed and the
            # sampled tokens are read back; step n+1 is planned and copied while step n runs
            "e2e": {"value": round(tokens / (ahead_ms / 1e3), 2), "unit": "tok/s", "ms_per_step": round(ahead_ms / args.steps, 4),
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "how": "wall clock of SpmdDriver.run_decode_steps(pipelined=True), the serving default: host plan -> pinned "
                           "H2D -> graph replay -> D2H tokens -> host completion per step, step n+1 planned and copied while step n runs",
                    "lock_step": {"value": round(e2e_value, 2), "ms_per_step": round(e2e_ms / args.steps, 4),
                                  "how": "the same with run_decode_steps(pipelined=False): nothing of step n+1 starts before step n's tokens are on the host"}},
            "gpu_launches": kernels_per_step * args.steps,
            "kernels_per_step_rank0": kernels_per_step,
            "device_status": status, "build_s": round(build_s, 1),
        }
        if spec_info is not None:
            out["speculative"] = spec_info
        if args.router_bias:
            out["config"]["router_bias"] = args.router_bias
        if skewed is not None:
            skewed["value"] = round(tokens / (skewed["ms_per_step"] * args.steps / 1e3), 2)
            out["skewed_routing"] = skewed
        if comm is not None:
            out["n2m_m2n"] = comm
        if trace_info is not None and os.environ.get("FASTAFD_COMM_TRACE_FULL") == "1":
            out["comm_trace"] = trace_info
        if world == 8 and tp == 1:
            out["config"]["deviation"] = "attention DP4 by request (--attn-tp 1); the named configuration is TP4, the default"
        if truncated:
            out["invalid"] = "model truncated with --layers (debug run)"
        print(json.dumps(out), flush=True)
    # The measurement is done and printed. Tearing down process groups and peer mappings needs every rank;
    # if one of them is slow to arrive, leave after a minute instead of holding the GPUs.
    import threading

    faulthandler.cancel_dump_traceback_later()
    quit_timer = threading.Timer(60.0, lambda: os._exit(0))
    quit_timer.daemon = True
    quit_timer.start()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    eng.close()
    quit_timer.cancel()
    faulthandler.cancel_dump_traceback_later()


if __name__ == "__main__":
    main()
