"""The fused N2M -> grouped GEMMs -> M2N path with every rank emulated on one GPU.

All kernels run back to back on one stream, so each wait finds its flag already set;
nothing here spins on another launch."""
import pytest
import torch

from fastafd_b200 import ops
from fastafd_b200.moe.afd_moe import AgMoeEndpoint, EgMoeEndpoint, MoeCommConfig, ag_layout, check_status, eg_layout
from fastafd_b200.ops._lib import lib, ptr, cur_stream, check
from fastafd_b200.parallel.fabric import Fabric
from fastafd_b200.reference import ops_ref as ref

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def _setup(cfg, timeout_ns=int(2e9)):
    sizes = [ag_layout(cfg).size] * cfg.num_ag + [eg_layout(cfg).size] * cfg.num_eg
    fabs = Fabric.local(sizes, DEV)
    ag_ranks = list(range(cfg.num_ag))
    eg_ranks = list(range(cfg.num_ag, cfg.num_ag + cfg.num_eg))
    ags = [AgMoeEndpoint(cfg, fabs[r], i, eg_ranks, DEV, timeout_ns) for i, r in enumerate(ag_ranks)]
    egs = [EgMoeEndpoint(cfg, fabs[r], i, ag_ranks, DEV, timeout_ns) for i, r in enumerate(eg_ranks)]
    return fabs, ags, egs


@pytest.mark.parametrize("direct", [False, True], ids=["recv-slots", "direct-stripes"])
@pytest.mark.parametrize("fp8", [False, True])
@pytest.mark.parametrize("num_ag,num_eg,T,bt", [(2, 2, 24, 16), (1, 1, 7, 32), (3, 2, 33, 32), (3, 2, 700, 64)])
def test_moe_roundtrip(num_ag, num_eg, T, bt, fp8, direct):
    """`direct`: rows are stored straight into per-expert stripes of the expert GPU's pool (slots
    claimed with atomic adds) and the expert side only builds the tile schedule; otherwise rows go
    to per-source receive slots and the expert side groups and gathers them."""
    H, I, E, K = 512, 256, 16, 4
    if T > 100 and (fp8 or direct):
        pytest.skip("large case: bf16 receive-slot path only (the direct exchange is for decode-sized steps)")
    cfg = MoeCommConfig(num_ag=num_ag, num_eg=num_eg, num_lanes=2, max_tokens=max(40, T), hidden=H, topk=K,
                        num_experts=E, intermediate=I, fp8=fp8, block_tok=bt, direct_tokens=40 if direct else 0)
    fabs, ags, egs = _setup(cfg)
    g = torch.Generator().manual_seed(0)
    wgu = (torch.randn(E, 2 * I, H, generator=g) * 0.05).to(torch.bfloat16)
    wd = (torch.randn(E, H, I, generator=g) * 0.05).to(torch.bfloat16)
    El = cfg.experts_per_eg
    eg_w = []
    for e in range(num_eg):
        gu, dn = wgu[e * El:(e + 1) * El], wd[e * El:(e + 1) * El]
        if fp8:
            guq = [ref.block_quant_fp8(gu[i]) for i in range(El)]
            dnq = [ref.block_quant_fp8(dn[i]) for i in range(El)]
            gu_q = torch.stack([q for q, _ in guq]).view(torch.uint8)
            gu_s = torch.stack([s for _, s in guq])
            dn_q = torch.stack([q for q, _ in dnq])
            dn_s = torch.stack([s for _, s in dnq])
            w13 = ops.interleave_gate_up(gu_q).view(torch.float8_e4m3fn).to(DEV)
            w13s = ops.interleave_gate_up_scales(gu_s, I).to(DEV)
            eg_w.append((w13, dn_q.to(DEV), w13s, ops.plain_tile_scales(dn_s).to(DEV)))
        else:
            eg_w.append((ops.interleave_gate_up(gu).to(DEV), dn.contiguous().to(DEV), None, None))
    for step in range(3):          # epochs advance; lanes alternate
        lane = step % 2
        xs, idxs, ws = [], [], []
        for a in range(num_ag):
            x = (torch.randn(T, H, generator=g)).to(torch.bfloat16)
            logits = torch.randn(T, E, generator=g)
            idx, w = ref.topk_route(logits, None, K)
            xs.append(x); idxs.append(idx); ws.append(w)
            ags[a].dispatch(lane, x.to(DEV), idx.to(DEV))
        for e in range(num_eg):
            egs[e].run_layer(lane, T, *eg_w[e])
        for a in range(num_ag):
            y = ags[a].combine_reduce(lane, ws[a].to(DEV), idxs[a].to(DEV), T)
            torch.cuda.synchronize()
            check_status(ags[a].status, "ag")
            for e in range(num_eg):
                check_status(egs[e].status, "eg")
            if fp8:
                # oracle with the same quantisation points
                exp = torch.zeros(T, H)
                xq, xsc = ref.group_quant_fp8(xs[a], 128)
                for t in range(T):
                    for k in range(K):
                        ex = int(idxs[a][t, k])
                        gq, gs = ref.block_quant_fp8(wgu[ex]); dq, ds = ref.block_quant_fp8(wd[ex])
                        gu = ref.fp8_gemm_nt(xq[t:t + 1], xsc[t:t + 1], gq, gs, torch.float32)
                        h = (torch.nn.functional.silu(gu[:, :I]) * gu[:, I:]).to(torch.bfloat16)
                        hq, hs = ref.group_quant_fp8(h, 128)
                        o = ref.fp8_gemm_nt(hq, hs, dq, ds, torch.bfloat16)
                        exp[t] += ws[a][t, k] * o[0].float()
                torch.testing.assert_close(y.cpu().float(), exp, atol=6e-2, rtol=5e-2)
            else:
                exp = ref.moe_experts(xs[a], idxs[a], ws[a], wgu, wd)
                torch.testing.assert_close(y.cpu().float(), exp.float(), atol=4e-2, rtol=4e-2)
    for f in fabs:
        f.close()


def test_flag_wait_times_out_cleanly():
    """A flag that nothing sets: the bounded wait returns a timeout status and the context
    stays usable (no trap, no hang)."""
    flag = torch.zeros(1, dtype=torch.int32, device=DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    check(lib().afd_wait_flag(ptr(flag), 1, int(0.2e9), ptr(status), cur_stream()), "wait_flag")
    torch.cuda.synchronize()
    assert int(status) == 2
    status.zero_()
    check(lib().afd_set_flag(ptr(flag), 1, cur_stream()), "set_flag")
    check(lib().afd_wait_flag(ptr(flag), 1, int(0.2e9), ptr(status), cur_stream()), "wait_flag")
    torch.cuda.synchronize()
    assert int(status) == 0 and int(flag) == 1
    assert float((torch.ones(4, device=DEV) * 2).sum()) == 8.0


def test_combine_times_out_when_expert_rank_is_silent():
    cfg = MoeCommConfig(num_ag=1, num_eg=1, num_lanes=1, max_tokens=8, hidden=256, topk=2, num_experts=4,
                        intermediate=128, block_tok=16)
    fabs, ags, egs = _setup(cfg, timeout_ns=int(0.2e9))
    w = torch.ones(4, 2, device=DEV)
    idx = torch.zeros(4, 2, dtype=torch.int32, device=DEV)
    ags[0].combine_reduce(0, w, idx, 4)
    torch.cuda.synchronize()
    with pytest.raises(RuntimeError, match="peer flag wait timed out"):
        check_status(ags[0].status, "ag")
    for f in fabs:
        f.close()


@pytest.mark.parametrize("scoring,gate_fp32,H,E,K", [
    ("softmax", False, 512, 16, 4),        # FMA logits loop (shape outside the tensor-core GEMV)
    ("sigmoid", True, 512, 16, 4),         # fp32 gate
    ("softmax", False, 2048, 128, 8),      # tensor-core GEMV: 8 expert tiles x 4 slices of H
    ("softmax", False, 4096, 512, 10),     # 32 expert tiles, one slice
    ("sigmoid", False, 1024, 64, 6),       # 4 expert tiles x 8 slices
    ("softmax", False, 2048, 120, 8),      # 120 experts: last tile partly empty, 8 tiles
])
def test_fused_route_dispatch_matches_separate_ops(scoring, gate_fp32, H, E, K):
    _route_dispatch_case(scoring, gate_fp32, H, E, K, direct=False)


@pytest.mark.parametrize("tpc,cluster", [(0, 0), (4, 1), (8, 1), (4, 2), (8, 4), (8, 8)])
@pytest.mark.parametrize("scoring,gate_fp32,H,E,K,fp8", [
    ("softmax", False, 2048, 128, 8, False),     # tensor-core logits
    ("softmax", False, 4096, 128, 8, True),      # 235B shape, FP8 rows with 1x128 scales
    ("sigmoid", True, 3072, 256, 8, False),      # fp32 gate + bias (SIMT logits)
    ("softmax", False, 4096, 512, 10, False),    # 512 experts top-10
    ("softmax", False, 512, 16, 4, False),       # tiny: SIMT bf16 logits
])
def test_fused_route_direct_dispatch(scoring, gate_fp32, H, E, K, fp8, tpc, cluster):
    """The direct variant: TPC tokens per CTA, optional cluster split of the expert range; rows,
    scales and meta words land in the experts' stripes, counters hold the per-expert counts."""
    if cluster and (E % (cluster * 16) != 0 and not gate_fp32 and E >= 128):
        pytest.skip("expert range does not split over this cluster size")
    if cluster and E % cluster != 0:
        pytest.skip("expert range does not split over this cluster size")
    _route_dispatch_case(scoring, gate_fp32, H, E, K, direct=True, fp8=fp8, tpc=tpc, cluster=cluster)


def _route_dispatch_case(scoring, gate_fp32, H, E, K, direct, fp8=False, tpc=0, cluster=0):
    """residual add + RMSNorm + router + push in one launch == the four separate ops."""
    I, T = 256, 19
    cfg = MoeCommConfig(num_ag=1, num_eg=2, num_lanes=1, max_tokens=32, hidden=H, topk=K, num_experts=E,
                        intermediate=I, block_tok=16, fp8=fp8, direct_tokens=32 if direct else 0)
    fabs, ags, egs = _setup(cfg)
    ags[0].route_tokens_per_cta, ags[0].route_cluster = tpc, cluster
    g = torch.Generator().manual_seed(3)
    attn_out = torch.randn(T, H, generator=g).to(torch.bfloat16).to(DEV)
    residual = torch.randn(T, H, generator=g).to(torch.bfloat16).to(DEV)
    norm_w = (1 + 0.1 * torch.randn(H, generator=g)).to(torch.bfloat16).to(DEV)
    gate = (torch.randn(E, H, generator=g) * 0.1).to(torch.float32 if gate_fp32 else torch.bfloat16).to(DEV)
    bias = (torch.randn(E, generator=g) * 0.1).to(DEV) if scoring == "sigmoid" else None
    res_ref = residual.clone()
    x_ref = ops.add_rmsnorm(attn_out, res_ref, norm_w, 1e-6)
    logits = torch.nn.functional.linear(x_ref.float(), gate.float())
    idx_ref, w_ref = ref.topk_route(logits.cpu(), None if bias is None else bias.cpu(), K, scoring, True)
    x_out = torch.empty_like(attn_out)
    idx = torch.empty(T, K, dtype=torch.int32, device=DEV)
    w = torch.empty(T, K, dtype=torch.float32, device=DEV)
    ags[0].route_dispatch(0, attn_out, residual, norm_w, gate, bias, x_out, idx, w, scoring=scoring, renorm=True, eps=1e-6)
    torch.cuda.synchronize()
    check_status(ags[0].status, "ag")
    assert torch.equal(residual, res_ref) and torch.equal(x_out, x_ref)
    assert torch.equal(idx.cpu(), idx_ref)
    torch.testing.assert_close(w.cpu(), w_ref, atol=1e-5, rtol=1e-4)
    if direct:
        # what landed in the expert stripes: every (token, k) exactly once, with its row (and scales)
        El, cap = cfg.experts_per_eg, cfg.direct_cap
        xq_ref, xs_ref = (ref.group_quant_fp8(x_ref.cpu(), 128) if fp8 else (None, None))
        seen = set()
        for e, eg in enumerate(egs):
            counts = eg.dcount[0].cpu()
            want = torch.bincount((idx_ref[(idx_ref // El) == e] - e * El).flatten().long(), minlength=El)
            assert torch.equal(counts.long(), want)
            meta, pool = eg.dmeta[0].cpu(), eg.dpool_x[0]
            for el in range(El):
                for s_ in range(int(counts[el])):
                    row = el * cap + s_
                    m = int(meta[row]) & 0xffffffff
                    src, k, t = m >> 24, (m >> 16) & 0xff, m & 0xffff
                    assert src == 0 and int(idx_ref[t, k]) == e * El + el and (t, k) not in seen
                    seen.add((t, k))
                    if fp8:
                        sc = eg.dpool_xs[0][row].cpu()
                        torch.testing.assert_close(sc, xs_ref[t], rtol=1e-6, atol=0)
                        deq = pool[row].cpu().float().view(-1, 128) * sc[:, None]
                        want_deq = xq_ref[t].float().view(-1, 128) * xs_ref[t][:, None]
                        # same scale; the quantised value may differ by one e4m3 step where x / scale and
                        # x * (1 / scale) round differently
                        torch.testing.assert_close(deq, want_deq, rtol=0.13, atol=1e-6)
                    else:
                        assert torch.equal(pool[row], x_ref[t])
            assert int(eg.n2m_flag[0][0]) == 1
        assert len(seen) == T * K
        for f in fabs:
            f.close()
        return
    # what landed in the expert GPUs' receive slots
    for e, eg in enumerate(egs):
        assert torch.equal(eg.recv_idx[0][0, :T].cpu(), idx_ref)
        owns = ((idx_ref // cfg.experts_per_eg) == e).any(dim=1)
        assert torch.equal(eg.recv_x[0][0, :T][owns.to(DEV)], x_ref[owns.to(DEV)])
        assert int(eg.n2m_flag[0][0]) == 1
    for f in fabs:
        f.close()


# ------------------------------------------------------------- fused attention-TP collectives
@pytest.mark.parametrize("tp,T,K", [(2, 32, 512), (4, 64, 1024), (2, 24, 256)])
def test_tp_fused_oproj_reduce_scatter_and_all_gather_loopback(tp, T, K):
    """tp ranks emulated on one GPU over a local fabric: every producer launch is queued before
    any consumer launch (kernels that wait for one another never run as separate launches on one
    GPU). The fused o_proj -> reduce-scatter must equal the fp32 sum of the partial GEMMs, the
    all-gather the concatenation of the ranks' rows; two rounds check the epoch protocol."""
    from fastafd_b200.parallel.fabric import Fabric
    from fastafd_b200.parallel.tp_fused import TpFusedComm, tp_layout

    H, lanes, cap = 256, 2, 32
    Tl = T // tp
    size = tp_layout(tp, lanes, cap, H).size
    fabs = Fabric.local([size] * tp, DEV)
    comms = [TpFusedComm(None, fabs[r], list(range(tp)), r, 0, lanes, cap, H, DEV, timeout_ns=int(2e9))
             for r in range(tp)]
    g = torch.Generator(device="cpu").manual_seed(tp * 100 + T)
    for rnd in range(2):
        lane = rnd % lanes
        o = [(torch.randn(T, K, generator=g) * 0.5).to(torch.bfloat16).to(DEV) for _ in range(tp)]
        w = [(torch.randn(H, K, generator=g) * 0.1).to(torch.bfloat16).to(DEV) for _ in range(tp)]
        for r in range(tp):
            comms[r].oproj_push(lane, o[r], w[r])
        ys = [comms[r].reduce_wait(lane, Tl) for r in range(tp)]
        torch.cuda.synchronize()
        full = sum((o[r].float() @ w[r].float().t()).to(torch.bfloat16).float() for r in range(tp))
        for r in range(tp):
            assert int(comms[r].status) == 0
            torch.testing.assert_close(ys[r].float(), full[r * Tl:(r + 1) * Tl], atol=3e-2, rtol=3e-2)
        xs = [(torch.randn(Tl, H, generator=g)).to(torch.bfloat16).to(DEV) for _ in range(tp)]
        for r in range(tp):
            comms[r].gather_push(lane, xs[r])
        got = [comms[r].gather_wait(lane, Tl).clone() for r in range(tp)]
        torch.cuda.synchronize()
        want = torch.cat(xs, 0)
        for r in range(tp):
            assert int(comms[r].status) == 0
            assert torch.equal(got[r], want)
