"""Single-kernel timing against the measured roofline.

    python -m fastafd_b200.benchmark.kernel_bench attention --batch 64 --ctx 2048
    python -m fastafd_b200.benchmark.kernel_bench gemm --experts 32 --tokens-per-expert 8 --n 1536 --k 2048
    python -m fastafd_b200.benchmark.kernel_bench route --tokens 32 --experts 128 --hidden 2048

Each case runs the kernel on its own with CUDA events after warm-up; between timed launches a
buffer larger than the 126 MB L2 is written so that the kernel's operands come from HBM. The
printed fraction divides the algorithmic bytes per second by the copy bandwidth in
``MEASURED_PEAKS.json`` at the repository root (fallback 6.65 TB/s when the file is absent).
"""
from __future__ import annotations

import argparse
import json
import math
import os

import torch

from .. import ops


def measured_peaks():
    path = os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))), "MEASURED_PEAKS.json")
    if os.path.exists(path):
        d = json.load(open(path))
        return d["hbm_gbs"], d["bf16_tflops"], "measured"
    return 6650.0, 1590.0, "fallback"


class L2Flusher:
    def __init__(self, device):
        self.buf = torch.empty(192 << 20, dtype=torch.uint8, device=device)

    def __call__(self):
        self.buf.fill_(1)


def time_kernel(fn, iters=20, warmup=5, flush=None):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    times = []
    for _ in range(iters):
        if flush:
            flush()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        torch.cuda.synchronize()
        times.append(e0.elapsed_time(e1) * 1e3)
    times.sort()
    return times[len(times) // 2], times[0]


def report(name, us_med, us_min, bytes_moved, flops=0.0, extra=None):
    hbm, tf, how = measured_peaks()
    gbs = bytes_moved / us_med / 1e3
    out = {"kernel": name, "us_median": round(us_med, 2), "us_min": round(us_min, 2), "GB_s": round(gbs, 1),
           f"frac_of_{how}_hbm": round(gbs / hbm, 3)}
    if flops:
        out["TFLOP_s"] = round(flops / us_med / 1e6, 1)
    if extra:
        out.update(extra)
    print(json.dumps(out))
    return out


def bench_attention(a):
    dev = "cuda"
    B, Hq, Hkv, D, page = a.batch, a.hq, a.hkv, a.head_dim, 16
    pages_per = (a.ctx + page - 1) // page
    n_pages = B * pages_per + 1
    pt = (torch.arange(B * pages_per, dtype=torch.int32, device=dev) + 1).view(B, pages_per)
    kc = torch.randn(n_pages * page, Hkv, D, device=dev, dtype=torch.bfloat16)
    vc = torch.randn_like(kc)
    q = torch.randn(B * a.q_len, Hq, D, device=dev, dtype=torch.bfloat16)
    lens = torch.full((B,), a.ctx, dtype=torch.int32, device=dev)
    m_tiles = (Hq // Hkv * a.q_len + 15) // 16
    splits = a.splits or ops.pick_attn_splits(B, Hkv, m_tiles, a.ctx, D)
    ws = ops.decode_attn_workspace(B, Hq, Hkv, a.q_len, D, splits, dev)
    out = torch.empty_like(q)
    fn = lambda: ops.decode_attention(q, kc, vc, pt, lens, Hq, Hkv, D, a.q_len, page, 1 / math.sqrt(D), splits=splits,  # noqa: E731
                                      workspace=ws, out=out)
    med, mn = time_kernel(fn, flush=L2Flusher(dev))
    kv_bytes = 2 * B * a.ctx * Hkv * D * 2
    report("decode_attention", med, mn, kv_bytes, extra={"B": B, "ctx": a.ctx, "Hq": Hq, "Hkv": Hkv, "D": D,
                                                          "q_len": a.q_len, "splits": splits})


def bench_attention_vs_library(a):
    """The paged decode attention kernel of this repository next to the TRT-LLM-gen decode kernel that
    FlashInfer ships as cubins (what the reference calls: python/minisgl/attention/trtllm.py:136-178),
    same shapes, same page table. Each launch follows a write of a buffer larger than the L2 inside one
    CUDA graph; the time of the flush-only graph is subtracted, so both numbers are device times per
    launch with KV read from HBM and without host launch cost."""
    from flashinfer.decode import trtllm_batch_decode_with_kv_cache

    dev = "cuda"
    B, Hq, Hkv, D, page = a.batch, a.hq, a.hkv, a.head_dim, 16
    pages_per = (a.ctx + page - 1) // page
    n_pages = B * pages_per + 1
    pt = (torch.arange(B * pages_per, dtype=torch.int32, device=dev) + 1).view(B, pages_per)
    kc = torch.randn(n_pages * page, Hkv, D, device=dev, dtype=torch.bfloat16)
    vc = torch.randn_like(kc)
    q = torch.randn(B, Hq, D, device=dev, dtype=torch.bfloat16)
    lens = torch.full((B,), a.ctx, dtype=torch.int32, device=dev)
    scale = 1 / math.sqrt(D)
    m_tiles = (Hq // Hkv + 15) // 16
    splits = a.splits or ops.pick_attn_splits(B, Hkv, m_tiles, a.ctx, D)
    ws = ops.decode_attn_workspace(B, Hq, Hkv, 1, D, splits, dev)
    out = torch.empty_like(q)
    lib_ws = torch.zeros(128 << 20, dtype=torch.uint8, device=dev)
    kv4 = (kc.view(n_pages, page, Hkv, D), vc.view(n_pages, page, Hkv, D))
    flush = L2Flusher(dev)

    def own():
        ops.decode_attention(q, kc, vc, pt, lens, Hq, Hkv, D, 1, page, scale, splits=splits, workspace=ws, out=out)

    def lib():
        return trtllm_batch_decode_with_kv_cache(query=q, kv_cache=kv4, workspace_buffer=lib_ws, block_tables=pt, seq_lens=lens,
                                                 max_seq_len=a.ctx, bmm1_scale=scale, bmm2_scale=1.0, kv_layout="NHD",
                                                 out_dtype=q.dtype, q_len_per_req=1)

    own()
    got_lib = lib()
    torch.cuda.synchronize()
    diff = (out.float() - got_lib.float().view_as(out)).abs().max().item()
    n = 10
    t_flush = time_graph(lambda: [flush() for _ in range(n)], n)
    t_own = time_graph(lambda: [(flush(), own()) for _ in range(n)], n) - t_flush
    t_lib = time_graph(lambda: [(flush(), lib()) for _ in range(n)], n) - t_flush
    hbm, _, how = measured_peaks()
    kv_bytes = 2 * B * a.ctx * Hkv * D * 2
    print(json.dumps({"kernel": "decode_attention_vs_trtllm_gen", "B": B, "ctx": a.ctx, "Hq": Hq, "Hkv": Hkv, "D": D,
                      "splits_own": splits, "us_own": round(t_own, 2), "us_trtllm_gen": round(t_lib, 2),
                      f"own_frac_of_{how}_hbm": round(kv_bytes / t_own / 1e3 / hbm, 3),
                      f"trtllm_frac_of_{how}_hbm": round(kv_bytes / t_lib / 1e3 / hbm, 3), "max_abs_diff": round(diff, 4)}))


def bench_gemm(a):
    dev = "cuda"
    E, N, K, bt = a.experts, a.n, a.k, a.block_tok
    per = a.tokens_per_expert
    info, row = [], 0
    for e in range(E):
        for j in range((per + bt - 1) // bt):
            info.append([e, row + j * bt, min(bt, per - j * bt), 0])
        row += (per + bt - 1) // bt * bt
    info_t = torch.tensor(info, dtype=torch.int32, device=dev)
    ntile = torch.tensor([len(info)], dtype=torch.int32, device=dev)
    x = torch.randn(row, K, device=dev, dtype=torch.bfloat16)
    w = (torch.randn(E, N, K, device=dev, dtype=torch.bfloat16) * 0.05)
    epi = ops.EPI_SWIGLU if a.swiglu else ops.EPI_STORE
    out = torch.empty(row, N // 2 if a.swiglu else N, device=dev, dtype=torch.bfloat16)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    if a.fp8:
        xq, xs = ops.group_quant_fp8(x, 128)
        wq = w.to(torch.float8_e4m3fn)
        ws = torch.ones(E, N // 128, 2, K // 128, device=dev)
        fn = lambda: ops.grouped_gemm(w=wq, x=xq, num_experts=E, n_per_expert=N, k=K, tile_info=info_t,  # noqa: E731
                                      num_tok_tiles=ntile, block_tok=bt, epilogue=ops.EPI_STORE, out=out, out_ld=N,
                                      fp8=True, x_scale=xs, w_scale=ws, status=status)
        wbytes = E * N * K
    else:
        if a.tile_major:
            ref_out = torch.empty_like(out)
            ops.grouped_gemm(w=w, x=x, num_experts=E, n_per_expert=N, k=K, tile_info=info_t, num_tok_tiles=ntile,
                             block_tok=bt, epilogue=epi, out=ref_out, out_ld=out.shape[1], status=status)
            w = ops.tile_major(w)
        fn = lambda: ops.grouped_gemm(w=w, x=x, num_experts=E, n_per_expert=N, k=K, tile_info=info_t,  # noqa: E731
                                      num_tok_tiles=ntile, block_tok=bt, epilogue=epi, out=out,
                                      out_ld=out.shape[1], status=status, w_tile_major=bool(a.tile_major))
        wbytes = E * N * K * 2
    med, mn = time_kernel(fn, flush=L2Flusher(dev))
    graph_us = time_graph(lambda: [fn() for _ in range(4)], 4)       # back to back, 1.2 GB of weights each: no L2 reuse
    assert int(status) == 0
    extra = {"E": E, "N": N, "K": K, "rows": row, "block_tok": bt, "tile_major": bool(a.tile_major),
             "us_in_graph": round(graph_us, 2), "GB_s_in_graph": round(wbytes / graph_us / 1e3, 1)}
    if a.l2_prefetch_mb > 0 and not a.fp8 and not a.tile_major:
        # What the L2 hint is worth when it has time to land: a launch without work (zero token tiles)
        # issues the prefetches, a spin kernel of about 20 us stands for the kernel in front of the GEMM,
        # then the GEMM runs. Same sequence with the hint off for comparison. (Measured on B200: no
        # difference in this form, where the issuing CTAs exit at once.)
        zero = torch.zeros(1, dtype=torch.int32, device=dev)
        ws_rot = [w, torch.randn_like(w) * 0.05]      # two weight sets in turn: nothing of a set survives in L2

        def seq(pf_bytes):
            for i in range(4):
                wi = ws_rot[i % 2]
                ops.grouped_gemm(w=wi, x=x, num_experts=E, n_per_expert=N, k=K, tile_info=info_t, num_tok_tiles=zero,
                                 block_tok=bt, epilogue=epi, out=out, out_ld=out.shape[1], status=status,
                                 l2_prefetch_bytes=pf_bytes)
                torch.cuda._sleep(40000)
                ops.grouped_gemm(w=wi, x=x, num_experts=E, n_per_expert=N, k=K, tile_info=info_t, num_tok_tiles=ntile,
                                 block_tok=bt, epilogue=epi, out=out, out_ld=out.shape[1], status=status)

        extra["seq_us_prefetch_off"] = round(time_graph(lambda: seq(0), 4), 2)
        extra["seq_us_prefetch_on"] = round(time_graph(lambda: seq(a.l2_prefetch_mb << 20), 4), 2)
    if a.tile_major and not a.fp8:
        valid = torch.zeros(row, dtype=torch.bool, device=dev)
        for e_, r0, n_, _ in info:
            valid[r0:r0 + n_] = True
        extra["max_abs_diff_vs_row_major"] = round((out[valid].float() - ref_out[valid].float()).abs().max().item(), 5)
    report("grouped_gemm" + ("_swiglu" if a.swiglu else "") + ("_fp8" if a.fp8 else ""), med, mn,
           wbytes + x.numel() * x.element_size(), flops=2.0 * row * N * K, extra=extra)


def time_graph(launch_all, n_launches: int, reps: int = 5) -> float:
    """Device time per launch (us) of a sequence captured into one CUDA graph: removes the host
    launch cost that dominates event timing of kernels of a few microseconds."""
    launch_all()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        launch_all()
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    best = float("inf")
    for _ in range(reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        g.replay()
        e1.record()
        torch.cuda.synchronize()
        best = min(best, e0.elapsed_time(e1) * 1e3 / n_launches)
    return best


def bench_dense(a):
    """Decode-shaped dense GEMM out[M,N] = x[M,K] @ w[N,K]^T: the tcgen05 kernel (weights on the
    UMMA M side) against cuBLAS through torch. Weights rotate over enough copies to exceed the L2."""
    dev = "cuda"
    M, N, K = a.tokens, a.n, a.k
    copies = max(2, int(160e6 // (N * K * 2)) + 1)
    ws = [(torch.randn(N, K, device=dev, dtype=torch.bfloat16) * 0.05) for _ in range(copies)]
    x = torch.randn(M, K, device=dev, dtype=torch.bfloat16)
    ref_out = torch.nn.functional.linear(x, ws[0])
    got = ops.dense_gemm(x, ws[0])
    torch.cuda.synchronize()
    err = (got.float() - ref_out.float()).abs().max().item()
    lib_t = time_graph(lambda: [torch.nn.functional.linear(x, w) for w in ws], copies)
    hbm, _, how = measured_peaks()
    wbytes = N * K * 2
    if a.fp8:
        # block-FP8 weights (e4m3, 128x128 scales): activation quantisation (1x128) + the FP8 kernel, which is
        # what a projection of an FP8 checkpoint costs per call, against cuBLAS on a bf16 copy of the weights
        from ..reference import ops_ref as ref

        qs = []
        for w in ws:
            q, sc = ref.block_quant_fp8(w.float())
            qs.append((q.contiguous(), ops.plain_tile_scales(sc[None].float()).contiguous()))

        def own_fp8(q, ksp):
            xq, xs = ops.group_quant_fp8(x, 128)
            return ops.dense_gemm(xq, q[0], x_scale=xs, w_scale=q[1], k_splits=ksp)

        got8 = own_fp8(qs[0], 0)
        torch.cuda.synchronize()
        err8 = (got8.float() - ref_out.float()).abs().max().item()
        quant_t = time_graph(lambda: [ops.group_quant_fp8(x, 128) for _ in ws], copies)
        for ksp in ([a.k_splits] if a.k_splits >= 0 else [0, 1, 2, 4, 8]):
            if ksp > 1 and (K // 128) % ksp:
                continue
            try:
                own = time_graph(lambda: [own_fp8(q, ksp) for q in qs], copies)
            except ValueError:
                continue
            print(json.dumps({"kernel": "dense_gemm_fp8", "M": M, "N": N, "K": K, "k_splits": ksp,
                              "us_own_fp8_with_quant": round(own, 2), "us_quant_alone": round(quant_t, 2),
                              "us_cublas_bf16": round(lib_t, 2), f"own_frac_of_{how}_hbm": round(N * K / own / 1e3 / hbm, 3),
                              "max_abs_diff_vs_bf16": round(err8, 4), "weight_copies": copies}))
        return
    for ksp in ([a.k_splits] if a.k_splits >= 0 else [0, 1, 2, 4, 8, 16]):
        if ksp > 1 and (K // 64) % ksp:
            continue
        try:
            own = time_graph(lambda: [ops.dense_gemm(x, w, k_splits=ksp) for w in ws], copies)
        except ValueError:
            continue
        print(json.dumps({"kernel": "dense_gemm", "M": M, "N": N, "K": K, "k_splits": ksp, "us_own_tcgen05": round(own, 2),
                          "us_cublas": round(lib_t, 2), f"own_frac_of_{how}_hbm": round(wbytes / own / 1e3 / hbm, 3),
                          f"cublas_frac_of_{how}_hbm": round(wbytes / lib_t / 1e3 / hbm, 3), "max_abs_diff": round(err, 4),
                          "weight_copies": copies}))


def bench_route(a):
    from ..moe.afd_moe import AgMoeEndpoint, MoeCommConfig, ag_layout, eg_layout
    from ..parallel.fabric import Fabric

    dev = torch.device("cuda:0")
    T, E, H, K = a.tokens, a.experts, a.hidden, a.topk
    cfg = MoeCommConfig(num_ag=1, num_eg=a.num_eg, num_lanes=1, max_tokens=T, hidden=H, topk=K, num_experts=E,
                        intermediate=768, block_tok=16)
    fabs = Fabric.local([ag_layout(cfg).size] + [eg_layout(cfg).size] * a.num_eg, dev)
    ag = AgMoeEndpoint(cfg, fabs[0], 0, list(range(1, 1 + a.num_eg)), dev)
    attn_out = torch.randn(T, H, device=dev, dtype=torch.bfloat16)
    residual = torch.randn(T, H, device=dev, dtype=torch.bfloat16)
    norm_w = torch.ones(H, device=dev, dtype=torch.bfloat16)
    gate = torch.randn(E, H, device=dev, dtype=torch.bfloat16) * 0.1
    x_out = torch.empty_like(attn_out)
    idx = torch.empty(T, K, dtype=torch.int32, device=dev)
    w = torch.empty(T, K, dtype=torch.float32, device=dev)
    fn = lambda: ag.route_dispatch(0, attn_out, residual, norm_w, gate, None, x_out, idx, w, scoring="softmax",  # noqa: E731
                                   renorm=True, eps=1e-6)
    med, mn = time_kernel(fn, flush=None)
    report("ag_route_dispatch", med, mn, T * H * 2 * 4 + E * H * 2, extra={"T": T, "E": E, "H": H, "K": K})


def bench_moe_layer(a):
    """One colocated MoE layer as the decode graph runs it - fused route + dispatch, expert-side
    schedule (or group + gather), the two grouped GEMMs, combine - captured `--reps` times into one
    CUDA graph and timed per layer; `front_us` times the part in front of the GEMMs alone. With
    --direct the rows go straight into per-expert pool stripes."""
    from ..moe.afd_moe import AgMoeEndpoint, EgMoeEndpoint, MoeCommConfig, ag_layout, eg_layout
    from ..parallel.fabric import Fabric

    dev = torch.device("cuda:0")
    T, E, H, K, I = a.tokens, a.experts, a.hidden, a.topk, a.intermediate
    cfg = MoeCommConfig(num_ag=1, num_eg=1, num_lanes=1, max_tokens=T, hidden=H, topk=K, num_experts=E, intermediate=I,
                        block_tok=a.block_tok, direct_tokens=T if a.direct else 0)
    fabs = Fabric.local([ag_layout(cfg).size, eg_layout(cfg).size], dev)
    ag = AgMoeEndpoint(cfg, fabs[0], 0, [1], dev, int(2e9))
    eg = EgMoeEndpoint(cfg, fabs[1], 0, [0], dev, int(2e9), status=ag.status)
    ag.route_tokens_per_cta, ag.route_cluster = a.tpc, a.cluster
    w13 = ops.interleave_gate_up((torch.randn(E, 2 * I, H, device=dev, dtype=torch.bfloat16) * 0.02))
    w2 = torch.randn(E, H, I, device=dev, dtype=torch.bfloat16) * 0.02
    attn_out = torch.randn(T, H, device=dev, dtype=torch.bfloat16) * 0.1
    residual = torch.randn(T, H, device=dev, dtype=torch.bfloat16)
    res0 = residual.clone()
    norm_w = torch.ones(H, device=dev, dtype=torch.bfloat16)
    gate = torch.randn(E, H, device=dev, dtype=torch.bfloat16) * 0.1
    x_out, normed = torch.empty_like(attn_out), torch.empty_like(attn_out)
    idx = torch.empty(T, K, dtype=torch.int32, device=dev)
    w = torch.empty(T, K, dtype=torch.float32, device=dev)

    def layer(full=True):
        ag.route_dispatch(0, attn_out, residual, norm_w, gate, None, x_out, idx, w, scoring="softmax", renorm=True, eps=1e-6)
        if full:
            eg.run_layer(0, T, w13, w2)
            ag.combine_reduce(0, w, idx, T, residual=residual, norm_w=norm_w, normed=normed)
        elif a.direct:
            eg._schedule(0)
        else:
            eg.group_gather(0, T)

    reps = a.reps
    full_us = time_graph(lambda: [layer(True) for _ in range(reps)], reps)
    residual.copy_(res0)
    # the front part alone leaves the M2N epochs untouched, so a full layer must not follow it
    front_us = time_graph(lambda: [layer(False) for _ in range(reps)], reps)
    torch.cuda.synchronize()
    hbm, _, how = measured_peaks()
    wbytes = E * 3 * I * H * 2
    print(json.dumps({"kernel": "moe_layer_colocated", "direct": bool(a.direct), "tpc": a.tpc, "cluster": a.cluster, "T": T,
                      "E": E, "H": H, "I": I, "layer_us": round(full_us, 2), "front_us": round(front_us, 2),
                      "weight_stream_us_at_copy_bw": round(wbytes / hbm / 1e3, 2), "status": int(ag.status)}))


def main(argv=None):
    ap = argparse.ArgumentParser()
    sub = ap.add_subparsers(dest="case", required=True)
    p = sub.add_parser("attention")
    p.add_argument("--batch", type=int, default=64)
    p.add_argument("--ctx", type=int, default=2048)
    p.add_argument("--hq", type=int, default=32)
    p.add_argument("--hkv", type=int, default=4)
    p.add_argument("--head-dim", type=int, default=128)
    p.add_argument("--q-len", type=int, default=1)
    p.add_argument("--splits", type=int, default=0)
    p = sub.add_parser("attention-vs-library")
    p.add_argument("--batch", type=int, default=32)
    p.add_argument("--ctx", type=int, default=1040)
    p.add_argument("--hq", type=int, default=32)
    p.add_argument("--hkv", type=int, default=4)
    p.add_argument("--head-dim", type=int, default=128)
    p.add_argument("--splits", type=int, default=0)
    p = sub.add_parser("gemm")
    p.add_argument("--experts", type=int, default=32)
    p.add_argument("--tokens-per-expert", type=int, default=8)
    p.add_argument("--n", type=int, default=1536)
    p.add_argument("--k", type=int, default=2048)
    p.add_argument("--block-tok", type=int, default=16)
    p.add_argument("--swiglu", action="store_true")
    p.add_argument("--fp8", action="store_true")
    p.add_argument("--tile-major", type=int, default=0)
    p.add_argument("--l2-prefetch-mb", type=int, default=0, help="also time the L2 weight hint (see bench_gemm)")
    p = sub.add_parser("dense")
    p.add_argument("--tokens", type=int, default=32)
    p.add_argument("--n", type=int, default=5120)
    p.add_argument("--k", type=int, default=2048)
    p.add_argument("--k-splits", type=int, default=-1, help="-1: sweep; 0: the heuristic")
    p.add_argument("--fp8", action="store_true", help="block-FP8 weights: quantise + FP8 kernel against cuBLAS on bf16")
    p = sub.add_parser("route")
    p.add_argument("--tokens", type=int, default=32)
    p.add_argument("--experts", type=int, default=128)
    p.add_argument("--hidden", type=int, default=2048)
    p.add_argument("--topk", type=int, default=8)
    p.add_argument("--num-eg", type=int, default=4)
    p = sub.add_parser("moe-layer")
    p.add_argument("--tokens", type=int, default=64)
    p.add_argument("--experts", type=int, default=128)
    p.add_argument("--hidden", type=int, default=2048)
    p.add_argument("--intermediate", type=int, default=768)
    p.add_argument("--topk", type=int, default=8)
    p.add_argument("--block-tok", type=int, default=16)
    p.add_argument("--direct", type=int, default=1)
    p.add_argument("--tpc", type=int, default=0)
    p.add_argument("--cluster", type=int, default=0)
    p.add_argument("--reps", type=int, default=20)
    a = ap.parse_args(argv)
    {"attention": bench_attention, "gemm": bench_gemm, "route": bench_route, "dense": bench_dense,
     "moe-layer": bench_moe_layer, "attention-vs-library": bench_attention_vs_library}[a.case](a)


if __name__ == "__main__":
    main()
