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
        fn = lambda: ops.grouped_gemm(w=w, x=x, num_experts=E, n_per_expert=N, k=K, tile_info=info_t,  # noqa: E731
                                      num_tok_tiles=ntile, block_tok=bt, epilogue=epi, out=out,
                                      out_ld=out.shape[1], status=status)
        wbytes = E * N * K * 2
    med, mn = time_kernel(fn, flush=L2Flusher(dev))
    assert int(status) == 0
    report("grouped_gemm" + ("_swiglu" if a.swiglu else "") + ("_fp8" if a.fp8 else ""), med, mn,
           wbytes + x.numel() * x.element_size(), flops=2.0 * row * N * K,
           extra={"E": E, "N": N, "K": K, "rows": row, "block_tok": bt})


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
    own = time_graph(lambda: [ops.dense_gemm(x, w) for w in ws], copies)
    lib_t = time_graph(lambda: [torch.nn.functional.linear(x, w) for w in ws], copies)
    hbm, _, how = measured_peaks()
    wbytes = N * K * 2
    print(json.dumps({"kernel": "dense_gemm", "M": M, "N": N, "K": K, "us_own_tcgen05": round(own, 2),
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
    p = sub.add_parser("gemm")
    p.add_argument("--experts", type=int, default=32)
    p.add_argument("--tokens-per-expert", type=int, default=8)
    p.add_argument("--n", type=int, default=1536)
    p.add_argument("--k", type=int, default=2048)
    p.add_argument("--block-tok", type=int, default=16)
    p.add_argument("--swiglu", action="store_true")
    p.add_argument("--fp8", action="store_true")
    p = sub.add_parser("dense")
    p.add_argument("--tokens", type=int, default=32)
    p.add_argument("--n", type=int, default=5120)
    p.add_argument("--k", type=int, default=2048)
    p = sub.add_parser("route")
    p.add_argument("--tokens", type=int, default=32)
    p.add_argument("--experts", type=int, default=128)
    p.add_argument("--hidden", type=int, default=2048)
    p.add_argument("--topk", type=int, default=8)
    p.add_argument("--num-eg", type=int, default=4)
    a = ap.parse_args(argv)
    {"attention": bench_attention, "gemm": bench_gemm, "route": bench_route, "dense": bench_dense}[a.case](a)


if __name__ == "__main__":
    main()
