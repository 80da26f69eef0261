"""Numerics of each sm_100a kernel against the PyTorch fp32 oracle of the same op."""
import math

import pytest
import torch

from fastafd_b200 import ops
from fastafd_b200.reference import ops_ref as ref

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _bf(*shape, scale=1.0, seed=0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    return (torch.randn(*shape, generator=g) * scale).to(torch.bfloat16).to(DEV)


@pytest.mark.parametrize("H", [256, 2048, 4096])
def test_rmsnorm_and_add(H):
    x, r, w = _bf(37, H, seed=1), _bf(37, H, seed=2), _bf(H, seed=3)
    out = ops.rmsnorm(x, w, 1e-6)
    torch.testing.assert_close(out.float(), ref.rmsnorm(x.cpu(), w.cpu(), 1e-6).float().to(DEV), atol=2e-2, rtol=2e-2)
    r_ref = r.cpu().clone()
    exp = ref.add_rmsnorm(x.cpu(), r_ref, w.cpu(), 1e-6, offset1=True)
    r_k = r.clone()
    got = ops.add_rmsnorm(x, r_k, w, 1e-6, offset1=True)
    torch.testing.assert_close(r_k.cpu(), r_ref)
    torch.testing.assert_close(got.float().cpu(), exp.float(), atol=3e-2, rtol=2e-2)


@pytest.mark.parametrize("D,rot", [(128, 128), (128, 64), (256, 64), (64, 64)])
def test_qk_norm_rope_store(D, rot):
    T, Hq, Hkv, slots = 19, 8, 2, 64
    qkv = _bf(T, (Hq + 2 * Hkv) * D, seed=4)
    qw, kw = _bf(D, seed=5) + 1, _bf(D, seed=6) + 1
    cs = ref.build_cos_sin_cache(512, rot, 1e6).to(DEV)
    pos = torch.randint(0, 512, (T,), dtype=torch.int32, device=DEV)
    loc = torch.randperm(slots, device=DEV)[:T].to(torch.int32)
    loc[3] = -1
    kc, vc = torch.zeros(slots, Hkv, D, dtype=torch.bfloat16, device=DEV), torch.zeros(slots, Hkv, D, dtype=torch.bfloat16, device=DEV)
    q_ref, kc_ref, vc_ref = qkv.cpu().clone(), kc.cpu().clone(), vc.cpu().clone()
    ref.qk_norm_rope_store(q_ref, qw.cpu(), kw.cpu(), cs.cpu(), pos.cpu(), loc.cpu(), kc_ref, vc_ref, Hq, Hkv, D, rot, 1e-6)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    ops.qk_norm_rope_store(qkv, qw, kw, cs, pos, loc, kc, vc, Hq, Hkv, D, rot, 1e-6, status=status)
    assert int(status) == 0
    qk_cols = (Hq + Hkv) * D
    torch.testing.assert_close(qkv.cpu().float()[:, :qk_cols], q_ref.float()[:, :qk_cols], atol=6e-2, rtol=3e-2)
    torch.testing.assert_close(kc.cpu().float(), kc_ref.float(), atol=6e-2, rtol=3e-2)
    torch.testing.assert_close(vc.cpu(), vc_ref)


@pytest.mark.parametrize("E,K,scoring", [(128, 8, "softmax"), (256, 8, "sigmoid"), (512, 10, "softmax"), (8, 2, "softmax")])
def test_topk_route(E, K, scoring):
    T = 45
    g = torch.Generator().manual_seed(7)
    logits = torch.randn(T, E, generator=g).to(DEV)
    bias = (torch.randn(E, generator=g) * 0.1).to(DEV) if scoring == "sigmoid" else None
    idx, w = ops.topk_route(logits, bias, K, scoring, True, 1.0)
    ridx, rw = ref.topk_route(logits.cpu(), None if bias is None else bias.cpu(), K, scoring, True, 1.0)
    assert torch.equal(idx.cpu(), ridx)
    torch.testing.assert_close(w.cpu(), rw, atol=1e-5, rtol=1e-4)


def test_argmax_and_embedding():
    logits = _bf(9, 151936, seed=8)
    assert torch.equal(ops.argmax(logits).cpu(), ref.argmax_lowest(logits.cpu()))
    table = _bf(1000, 256, seed=9)
    ids = torch.tensor([0, 5, 999, 1000, 77], dtype=torch.int32, device=DEV)
    out = ops.embedding(ids, table)
    assert torch.equal(out[:3], table[ids[:3].long()]) and float(out[3].abs().sum()) == 0


@pytest.mark.parametrize("group,pow2", [(128, False), (32, True)])
def test_group_quant_fp8(group, pow2):
    x = _bf(33, 2048, seed=10)
    q, s = ops.group_quant_fp8(x, group, pow2)
    rq, rs = ref.group_quant_fp8(x.cpu(), group, pow2)
    torch.testing.assert_close(s.cpu(), rs, rtol=1e-6, atol=0)
    # round-to-nearest of x/scale may differ by one ulp where the division differs; compare dequantised
    torch.testing.assert_close(ref.group_dequant_fp8(q.cpu(), s.cpu(), group), ref.group_dequant_fp8(rq, rs, group), atol=0.13, rtol=0.07)
    assert (q.cpu().view(torch.uint8) == rq.view(torch.uint8)).float().mean() > 0.995


@pytest.mark.parametrize("Hq,Hkv,D,q_len,page,splits", [
    (32, 4, 128, 1, 16, 1), (32, 4, 128, 1, 16, 3), (64, 4, 128, 1, 16, 2), (32, 2, 256, 1, 16, 2),
    (16, 4, 128, 4, 16, 2), (8, 2, 64, 1, 1, 1), (48, 8, 128, 1, 64, 4),
])
def test_decode_attention(Hq, Hkv, D, q_len, page, splits):
    B = 5
    lens = torch.tensor([1 + q_len, 37, 300, 1025, 513], dtype=torch.int32)[:B]
    max_pages = (int(lens.max()) + page - 1) // page + 1
    n_pages = B * max_pages + 3
    perm = torch.randperm(n_pages)
    pt = perm[:B * max_pages].view(B, max_pages).to(torch.int32)
    kc, vc = _bf(n_pages * page, Hkv, D, seed=11), _bf(n_pages * page, Hkv, D, seed=12)
    q = _bf(B * q_len, Hq, D, seed=13)
    scale = 1 / math.sqrt(D)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    out = ops.decode_attention(q, kc, vc, pt.to(DEV), lens.to(DEV), Hq, Hkv, D, q_len, page, scale, splits=splits, status=status)
    exp = ref.decode_attention(q.cpu(), kc.cpu(), vc.cpu(), pt, lens, Hq, Hkv, D, q_len, page, scale)
    assert int(status) == 0
    torch.testing.assert_close(out.cpu().float(), exp.float(), atol=2e-2, rtol=2e-2)


def test_decode_attention_one_workspace_shared_by_different_shapes():
    """One zeroed workspace serves launches of different (B, splits): the arrival counters sit at a
    fixed place in front of the partial results, so a smaller launch after a larger one still finds
    them at zero and merges its splits."""
    Hq, Hkv, D, page = 32, 4, 128, 16
    scale = 1 / math.sqrt(D)
    ws = ops.decode_attn_workspace(8, Hq, Hkv, 1, D, 8, DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    for i, (B, splits) in enumerate([(8, 8), (4, 8), (8, 4), (3, 2), (2, 5), (1, 3), (8, 8)]):
        lens = torch.tensor([2049, 300, 1025, 513, 1800, 77, 4000, 1234], dtype=torch.int32)[:B]
        max_pages = (int(lens.max()) + page - 1) // page + 1
        n_pages = B * max_pages + 3
        pt = torch.randperm(n_pages)[:B * max_pages].view(B, max_pages).to(torch.int32)
        kc, vc = _bf(n_pages * page, Hkv, D, seed=31 + i), _bf(n_pages * page, Hkv, D, seed=41 + i)
        q = _bf(B, Hq, D, seed=51 + i)
        out = torch.full((B, Hq, D), float("nan"), dtype=torch.bfloat16, device=DEV)
        ops.decode_attention(q, kc, vc, pt.to(DEV), lens.to(DEV), Hq, Hkv, D, 1, page, scale, splits=splits,
                             workspace=ws, out=out, status=status)
        exp = ref.decode_attention(q.cpu(), kc.cpu(), vc.cpu(), pt, lens, Hq, Hkv, D, 1, page, scale)
        assert int(status) == 0
        torch.testing.assert_close(out.cpu().float(), exp.float(), atol=2e-2, rtol=2e-2)


@pytest.mark.parametrize("M,N,K,bt", [(16, 256, 128, 16), (32, 512, 2048, 32), (77, 1536, 2048, 32), (64, 2048, 768, 64), (200, 1024, 512, 128), (5, 128, 64, 16)])
def test_dense_gemm_tcgen05(M, N, K, bt):
    x, w = _bf(M, K, seed=14), _bf(N, K, scale=0.05, seed=15)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    out = ops.dense_gemm(x, w, bt, status=status)
    torch.cuda.synchronize()
    assert int(status) == 0
    exp = (x.float() @ w.float().t())
    torch.testing.assert_close(out.float(), exp, atol=3e-2, rtol=2e-2)


@pytest.mark.parametrize("M,N,K,splits,with_bias", [(64, 5120, 2048, 0, False), (64, 2048, 4096, 8, False), (32, 1024, 2048, 4, True),
                                                     (7, 256, 512, 2, True), (128, 2048, 2048, 0, False), (64, 1280, 2048, 0, True)])
def test_dense_gemm_split_k_and_bias(M, N, K, splits, with_bias):
    """Split-K: several CTAs share one output tile, the last one to arrive sums the fp32 partials.
    Three calls in a row on the same buffers (the counters must come back to zero)."""
    x, w = _bf(M, K, seed=24), _bf(N, K, scale=0.05, seed=25)
    bias = _bf(N, seed=26) if with_bias else None
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    exp = x.float() @ w.float().t() + (bias.float() if with_bias else 0)
    for _ in range(3):
        out = ops.dense_gemm(x, w, status=status, bias=bias, k_splits=splits)
        torch.cuda.synchronize()
        assert int(status) == 0
        torch.testing.assert_close(out.float(), exp, atol=4e-2, rtol=2e-2)


def test_dense_gemm_block_fp8_split_k():
    """Block-FP8 dense projection: e4m3 weights with 128x128 scales, 1x128 activation scales, split-K."""
    M, N, K = 48, 1536, 4096
    x, w = _bf(M, K, seed=27), _bf(N, K, scale=0.05, seed=28)
    wq, wsc = ref.block_quant_fp8(w.cpu().float())
    xq, xs = ops.group_quant_fp8(x, 128)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    out = ops.dense_gemm(xq, wq.to(DEV), status=status, x_scale=xs, w_scale=ops.plain_tile_scales(wsc[None].float()).to(DEV))
    torch.cuda.synchronize()
    assert int(status) == 0
    exp = ref.fp8_gemm_nt(xq.cpu(), xs.cpu(), wq, wsc, torch.float32)
    torch.testing.assert_close(out.cpu().float(), exp, atol=6e-2, rtol=3e-2)


def _tile_schedule(counts, bt):
    info, row = [], 0
    for e, c in enumerate(counts):
        for j in range((c + bt - 1) // bt):
            info.append([e, row + j * bt, min(bt, c - j * bt), 0])
        row += (c + bt - 1) // bt * bt
    return torch.tensor(info, dtype=torch.int32), row


@pytest.mark.parametrize("bt", [16, 32, 64])
def test_grouped_swiglu_bf16(bt):
    E, I, H = 6, 256, 512
    counts = [3, 0, bt, bt + 5, 1, 40]
    info, rows = _tile_schedule(counts, bt)
    x = _bf(rows, H, seed=16)
    wgu = _bf(E, 2 * I, H, scale=0.05, seed=17)
    out = torch.zeros(rows, I, dtype=torch.bfloat16, device=DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    ops.grouped_gemm(w=ops.interleave_gate_up(wgu), x=x, num_experts=E, n_per_expert=2 * I, k=H,
                     tile_info=info.to(DEV), num_tok_tiles=torch.tensor([info.shape[0]], dtype=torch.int32, device=DEV),
                     block_tok=bt, epilogue=ops.EPI_SWIGLU, out=out, out_ld=I, status=status,
                     l2_prefetch_bytes=(8 << 20) if bt == 16 else 0)      # the L2 hint changes no result
    torch.cuda.synchronize()
    assert int(status) == 0
    for t in range(info.shape[0]):
        e, r0, v, _ = info[t].tolist()
        gu = (x[r0:r0 + v].float() @ wgu[e].float().t())
        exp = torch.nn.functional.silu(gu[:, :I]) * gu[:, I:]
        torch.testing.assert_close(out[r0:r0 + v].float(), exp, atol=3e-2, rtol=3e-2)


@pytest.mark.parametrize("bt", [16, 32, 64])
def test_fp8_block_scaled_gemm(bt):
    M, N, K = (50 if bt < 64 else 150), 512, 1024
    x, w = _bf(M, K, seed=18), _bf(N, K, scale=0.05, seed=19)
    xq, xs = ref.group_quant_fp8(x.cpu(), 128)
    wq, ws = ref.block_quant_fp8(w.cpu(), 128)
    exp = ref.fp8_gemm_nt(xq, xs, wq, ws)
    info, n = ops.dense_tile_schedule(M, bt, DEV)
    out = torch.zeros(M, N, dtype=torch.bfloat16, device=DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    ops.grouped_gemm(w=wq.to(DEV), x=xq.to(DEV), num_experts=1, n_per_expert=N, k=K, tile_info=info, num_tok_tiles=n,
                     block_tok=bt, epilogue=ops.EPI_STORE, out=out, out_ld=N, fp8=True, x_scale=xs.to(DEV),
                     w_scale=ops.plain_tile_scales(ws[None].to(DEV)), status=status)
    torch.cuda.synchronize()
    assert int(status) == 0
    torch.testing.assert_close(out.cpu().float(), exp.float(), atol=3e-2, rtol=2e-2)


@pytest.mark.parametrize("hk,hv,dk,dv,merged", [(2, 4, 32, 32, False), (4, 16, 128, 128, False), (4, 16, 128, 128, True)])
def test_gdn_decode_step(hk, hv, dk, dv, merged):
    """`merged`: mixed | z and b | a are column ranges of two wider tensors (the outputs of the merged
    input projections), read in place through their row strides."""
    from fastafd_b200.models.transformer import AttnMeta
    from fastafd_b200.ops import gdn as gdn_ops

    T, slots, W = 5, 9, 4
    Cc = 2 * hk * dk + hv * dv
    mixed, z = _bf(T, Cc, seed=20), _bf(T, hv * dv, seed=21)
    a, b = _bf(T, hv, seed=22), _bf(T, hv, seed=23)
    if merged:
        qkvz, ba = torch.cat([mixed, z], 1).contiguous(), torch.cat([b, a], 1).contiguous()
        mixed, z, b, a = qkvz[:, :Cc], qkvz[:, Cc:], ba[:, :hv], ba[:, hv:]
        assert not z.is_contiguous() and not a.is_contiguous()
    conv_w = _bf(Cc, W, scale=0.5, seed=24)
    A_log = torch.randn(hv, generator=torch.Generator().manual_seed(25)).to(DEV) * 0.5
    dt_bias = torch.randn(hv, generator=torch.Generator().manual_seed(26)).to(DEV) * 0.5
    norm_w = _bf(dv, seed=27) + 1
    conv_state = _bf(slots, W - 1, Cc, seed=28)
    rec_state = torch.randn(slots, hv, dv, dk, generator=torch.Generator().manual_seed(29)).to(DEV) * 0.1
    sl = torch.tensor([3, 0, 8, 5, 1], dtype=torch.int32, device=DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    meta = AttnMeta(positions=None, out_loc=None, page_table=None, seq_lens=None, state_slots=sl, status=status)
    cs_ref, rs_ref = conv_state.cpu().clone(), rec_state.cpu().clone()
    meta_cpu = AttnMeta(positions=None, out_loc=None, page_table=None, seq_lens=None, state_slots=sl.cpu())
    exp = gdn_ops.gdn_block(mixed.cpu(), z.cpu(), a.cpu(), b.cpu(), conv_w.cpu(), A_log.cpu(), dt_bias.cpu(), norm_w.cpu(),
                            cs_ref, rs_ref, meta_cpu, hk, hv, dk, dv, 1e-6)
    got = gdn_ops.gdn_block(mixed, z, a, b, conv_w, A_log, dt_bias, norm_w, conv_state, rec_state, meta, hk, hv, dk, dv, 1e-6)
    torch.cuda.synchronize()
    assert int(status) == 0
    torch.testing.assert_close(conv_state.cpu(), cs_ref)
    torch.testing.assert_close(rec_state.cpu(), rs_ref, atol=2e-3, rtol=2e-3)
    torch.testing.assert_close(got.cpu().float(), exp.float(), atol=4e-2, rtol=4e-2)


@pytest.mark.parametrize("hk,hv,dk,dv", [(2, 4, 32, 32), (2, 8, 128, 128)])
def test_gdn_prefill_matches_token_serial_oracle(hk, hv, dk, dv):
    """Packed prefill of three sequences (one continuing from a stored state, two fresh, plus
    padding rows) against the CPU oracle path of the same block."""
    from fastafd_b200.models.transformer import AttnMeta
    from fastafd_b200.ops import gdn as gdn_ops

    lens, slots, W = [7, 0, 12, 5], 6, 4
    T = sum(lens) + 3                       # 3 padding rows
    Cc = 2 * hk * dk + hv * dv
    mixed, z = _bf(T, Cc, seed=30), _bf(T, hv * dv, seed=31)
    a, b = _bf(T, hv, seed=32), _bf(T, hv, seed=33)
    conv_w = _bf(Cc, W, scale=0.5, seed=34)
    A_log = torch.randn(hv, generator=torch.Generator().manual_seed(35)).to(DEV) * 0.5
    dt_bias = torch.randn(hv, generator=torch.Generator().manual_seed(36)).to(DEV) * 0.5
    norm_w = _bf(dv, seed=37) + 1
    conv_state = _bf(slots, W - 1, Cc, seed=38)
    rec_state = torch.randn(slots, hv, dv, dk, generator=torch.Generator().manual_seed(39)).to(DEV) * 0.1
    sl = torch.tensor([4, 2, 0, 5], dtype=torch.int32, device=DEV)
    # sequence 0 continues (3 tokens already cached), the others start at position 0
    seq_lens = torch.tensor([3 + 7, 0, 12, 5], dtype=torch.int32, device=DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    kw = dict(positions=None, out_loc=None, page_table=None, is_prefill=True, prefill_lens=lens)
    meta = AttnMeta(seq_lens=seq_lens, state_slots=sl, status=status, **kw)
    meta_cpu = AttnMeta(seq_lens=seq_lens.cpu(), state_slots=sl.cpu(), **kw)
    cs_ref, rs_ref = conv_state.cpu().clone(), rec_state.cpu().clone()
    exp = gdn_ops.gdn_block(mixed.cpu(), z.cpu(), a.cpu(), b.cpu(), conv_w.cpu(), A_log.cpu(), dt_bias.cpu(), norm_w.cpu(),
                            cs_ref, rs_ref, meta_cpu, hk, hv, dk, dv, 1e-6)
    got = gdn_ops.gdn_block(mixed, z, a, b, conv_w, A_log, dt_bias, norm_w, conv_state, rec_state, meta, hk, hv, dk, dv, 1e-6)
    torch.cuda.synchronize()
    assert int(status) == 0
    used = [4, 0, 5]
    torch.testing.assert_close(conv_state.cpu()[used], cs_ref[used])
    torch.testing.assert_close(rec_state.cpu()[used], rs_ref[used], atol=3e-3, rtol=3e-3)
    torch.testing.assert_close(got.cpu().float(), exp.float(), atol=5e-2, rtol=5e-2)
    assert float(got[sum(lens):].abs().max()) == 0.0


# ----------------------------------------------------------------------------- sampling
def _kept_set(logits_row, temp, k, tp):
    """Oracle: tokens that survive top-k then top-p (ops_ref.sample semantics) and their
    renormalised probabilities."""
    p = torch.softmax(logits_row.double() / temp, -1)
    V = p.numel()
    if 0 < k < V:
        kth = p.topk(k).values[-1]
        p = torch.where(p < kth, torch.zeros_like(p), p)
    if tp < 1.0:
        sp, si = p.sort(descending=True)
        cum = sp.cumsum(0)
        sp = torch.where((cum - sp) > tp, torch.zeros_like(sp), sp)
        p = torch.zeros_like(p).scatter_(0, si, sp)
    return p / p.sum()


@pytest.mark.gpu
@pytest.mark.parametrize("V,temp,k,tp", [(1000, 1.0, 0, 1.0), (1000, 0.7, 20, 1.0), (1000, 1.3, 0, 0.8),
                                          (5000, 1.0, 50, 0.9), (151936, 0.8, 40, 0.95)])
def test_sample_kernel_distribution(V, temp, k, tp):
    torch.manual_seed(V + k)
    row = (torch.randn(V, device=DEV) * 3).float()
    want = _kept_set(row.cpu(), temp, k, tp)
    N = 20000
    logits = row[None, :].expand(N, V)          # stride-0 rows: every draw sees the same logits
    u = (torch.arange(N, device=DEV, dtype=torch.float32) + 0.5) / N
    toks = ops.sample(logits, torch.full((N,), temp), torch.full((N,), k, dtype=torch.int32),
                      torch.full((N,), tp), uniform=u)
    torch.cuda.synchronize()
    counts = torch.bincount(toks.long().cpu(), minlength=V).double()
    kept = want > 0
    # every draw lies in the oracle's kept set (a token at the top-p border may differ by rounding)
    outside = counts[~kept].sum().item()
    assert outside <= N * 2e-3, outside
    got = counts / N
    # a stratified uniform grid reproduces each probability to about 1/N per token
    err = (got - want).abs()
    assert err.max().item() < 3e-3, err.max().item()
    assert (got[kept] - want[kept]).abs().sum().item() < kept.sum().item() / N + 0.01


@pytest.mark.gpu
def test_sample_kernel_greedy_rows_and_bf16():
    torch.manual_seed(3)
    T, V = 7, 4099
    logits = torch.randn(T, V, device=DEV).to(torch.bfloat16)
    logits[2, 100] = logits[2, 50] = 9.0        # tie: lowest index wins
    temps = torch.tensor([0.0, 1.0, 0.0, 0.5, 0.0, 1.0, 0.0])
    toks = ops.sample(logits, temps, torch.ones(T, dtype=torch.int32), torch.ones(T))   # top_k = 1 -> mode
    torch.cuda.synchronize()
    want = ref.argmax_lowest(logits.float().cpu())
    assert toks.cpu().tolist() == want.tolist()


# ------------------------------------------------------------- model-family kernels
@pytest.mark.parametrize("D,rot,Hq,Hkv,ld_extra", [(128, 64, 6, 2, 0), (128, 128, 4, 1, 0), (64, 32, 8, 4, 256)])
def test_cross_head_norm_rope_store(D, rot, Hq, Hkv, ld_extra):
    """Joint RMSNorm over all q heads / all k heads + RoPE + paged store in one launch, against the
    unfused form (fp32 norm rounded to bf16, then the per-head kernel's oracle without weights)."""
    T, slots = 21, 64
    n = (Hq + 2 * Hkv) * D
    buf = _bf(T, n + ld_extra, seed=61)
    qkv = buf[:, :n] if ld_extra else buf
    qw, kw = _bf(Hq * D, seed=62) * 0.2 + 1, _bf(Hkv * D, seed=63) * 0.2 + 1
    cs = ref.build_cos_sin_cache(512, rot, 5e6).to(DEV)
    pos = torch.randint(0, 512, (T,), dtype=torch.int32, device=DEV)
    loc = torch.randperm(slots, device=DEV)[:T].to(torch.int32)
    loc[5] = -1
    kc = torch.zeros(slots, Hkv, D, dtype=torch.bfloat16, device=DEV)
    vc = torch.zeros_like(kc)
    # oracle
    x = qkv.cpu().clone().contiguous()
    q, k = x[:, :Hq * D].float(), x[:, Hq * D:(Hq + Hkv) * D].float()
    x[:, :Hq * D] = (q * torch.rsqrt(q.pow(2).mean(-1, keepdim=True) + 1e-6) * qw.cpu().float()).to(torch.bfloat16)
    x[:, Hq * D:(Hq + Hkv) * D] = (k * torch.rsqrt(k.pow(2).mean(-1, keepdim=True) + 1e-6) * kw.cpu().float()).to(torch.bfloat16)
    kc_ref, vc_ref = kc.cpu().clone(), vc.cpu().clone()
    ref.qk_norm_rope_store(x, None, None, cs.cpu(), pos.cpu(), loc.cpu(), kc_ref, vc_ref, Hq, Hkv, D, rot, 1e-6)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    ops.cross_head_norm_rope_store(qkv, qw, kw, cs, pos, loc, kc, vc, Hq, Hkv, D, rot, 1e-6, Hq * D, Hkv * D, status=status)
    assert int(status) == 0
    qk_cols = (Hq + Hkv) * D
    torch.testing.assert_close(qkv.cpu().float()[:, :qk_cols], x.float()[:, :qk_cols], atol=6e-2, rtol=3e-2)
    torch.testing.assert_close(kc.cpu().float(), kc_ref.float(), atol=6e-2, rtol=3e-2)
    torch.testing.assert_close(vc.cpu(), vc_ref)
    # TP form: sums of squares given from outside (here: the local ones, i.e. the same result)
    qkv2 = (buf.clone()[:, :n] if ld_extra else _bf(T, n, seed=61))
    sq = ops.qk_square_sums(qkv2, Hq * D, Hkv * D)
    torch.testing.assert_close(sq[:, 0].cpu(), qkv2[:, :Hq * D].float().pow(2).sum(-1).cpu(), rtol=1e-4, atol=1e-3)


@pytest.mark.parametrize("E,K,n_group,topk_group,bf16", [(256, 8, 8, 4, False), (128, 8, 4, 2, True), (160, 6, 5, 3, False), (8, 2, 2, 1, False)])
def test_grouped_topk_route(E, K, n_group, topk_group, bf16):
    T = 37
    g = torch.Generator().manual_seed(9)
    logits = torch.randn(T, E, generator=g)
    if bf16:
        logits = logits.to(torch.bfloat16)
    bias = torch.randn(E, generator=g) * 0.1
    idx, w = ops.grouped_topk_route(logits.to(DEV), bias.to(DEV), K, n_group, topk_group, True, 2.5)
    ridx, rw = ref.grouped_topk_route(logits.float(), bias, K, n_group, topk_group, True, 2.5)
    assert torch.equal(idx.cpu(), ridx)
    torch.testing.assert_close(w.cpu(), rw, atol=1e-5, rtol=1e-4)


def test_shared_gate_and_attention_gate_kernels():
    T, H = 23, 1024
    x, gw, y = _bf(T, H, seed=71), _bf(1, H, scale=0.05, seed=72), _bf(T, H, seed=73)
    g = torch.sigmoid(torch.nn.functional.linear(x, gw).float())
    want = (y.float() * g).to(torch.bfloat16)
    got = ops.shared_gate_mul(x, gw, y.clone())
    torch.testing.assert_close(got.float(), want.float(), atol=2e-2, rtol=2e-2)
    # attention output gate read through a row stride
    n = 512
    merged = _bf(T, 3 * n, seed=74)
    gate = merged[:, 2 * n:]
    o = _bf(T, n, seed=75)
    want = (o.float() * torch.sigmoid(gate.float())).to(torch.bfloat16)
    got = ops.sigmoid_gate_mul(o.clone(), gate)
    torch.testing.assert_close(got.float(), want.float(), atol=1e-2, rtol=1e-2)


def test_prefill_attention_varlen_one_launch():
    """Chunks of different lengths (one of them empty, one continuing an earlier chunk) in one launch
    against the per-request oracle."""
    Hq, Hkv, D, page = 8, 2, 128, 16
    chunk = [37, 0, 5, 64, 1]
    seq = [37, 12, 50, 64, 200]            # KV length including the chunk (requests 2 and 4 continue)
    B = len(chunk)
    max_pages = (max(seq) + page - 1) // page + 1
    n_pages = B * max_pages + 3
    pt = torch.randperm(n_pages)[:B * max_pages].view(B, max_pages).to(torch.int32)
    kc, vc = _bf(n_pages * page, Hkv, D, seed=81), _bf(n_pages * page, Hkv, D, seed=82)
    q = _bf(sum(chunk), Hq, D, seed=83)
    starts = torch.tensor([0] + list(torch.tensor(chunk).cumsum(0)), dtype=torch.int32)
    scale = 1 / math.sqrt(D)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    out = ops.prefill_attention_varlen(q, kc, vc, pt.to(DEV), torch.tensor(seq, dtype=torch.int32, device=DEV),
                                       starts.to(DEV), max(chunk), Hq, Hkv, D, page, scale, status=status)
    torch.cuda.synchronize()
    assert int(status) == 0
    off = 0
    for b, n in enumerate(chunk):
        if n:
            exp = ref.decode_attention(q[off:off + n].cpu(), kc.cpu(), vc.cpu(), pt[b:b + 1], torch.tensor([seq[b]], dtype=torch.int32),
                                       Hq, Hkv, D, n, page, scale)
            torch.testing.assert_close(out[off:off + n].cpu().float(), exp.float(), atol=2e-2, rtol=2e-2)
        off += n
