"""Core-attention disaggregation on a GPU: the hop kernels (put rows + flag, wait + KV store, attention
output straight into the model side's window, o flag, epoch) with the model side and the attention
side in one process on one GPU. Every launch is queued in program order on one stream, so each wait
finds its flag already set; nothing here spins on another launch."""
import pytest
import torch

from fastafd_b200.config import ModelConfig, RopeConfig, RuntimeConfig
from fastafd_b200.engine import AfdEngine, SpmdDriver
from fastafd_b200.protocol import AfdTopology

pytestmark = pytest.mark.gpu

CFGS = {
    "qwen3_moe": ModelConfig(num_layers=3, hidden_size=512, num_q_heads=8, num_kv_heads=2, head_dim=128, vocab_size=2048,
                             num_experts=16, num_experts_per_tok=4, moe_intermediate_size=256),
    "minimax_m2": ModelConfig(architecture="MiniMaxM2ForCausalLM", num_layers=3, hidden_size=512, num_q_heads=8, num_kv_heads=2,
                              head_dim=128, vocab_size=2048, rope=RopeConfig(5e6, 64), qk_norm="cross_head", num_experts=16,
                              num_experts_per_tok=4, moe_intermediate_size=256, scoring="sigmoid", router_bias=True,
                              router_fp32=True),
}


def _engine(cfg, graph):
    rt = RuntimeConfig(num_mb=2, page_size=16, num_pages=128, max_running_requests=16, max_seq_len=256, cuda_graph_max_bs=8,
                       decode_graph_bs=(8,), device="cuda", moe_block_tok=16, use_cuda_graph=graph)
    eng = AfdEngine(cfg, rt, AfdTopology(colocated=True), 0, "cuda:0", seed=0)
    drv = SpmdDriver(eng)
    drv.install_prefilled(12, 40, max_tokens=64)
    return eng, drv


def _tokens(eng, drv, steps):
    out = []
    for _ in range(steps):
        drv.run_decode_steps(1, pipelined=False)
        out.append(torch.cat([b.next_tokens.clone() for b in eng.attn.bufs]).cpu())
    return torch.stack(out)


@pytest.mark.parametrize("graph", [False, True], ids=["eager", "graph"])
@pytest.mark.parametrize("name", list(CFGS))
def test_cad_loopback_equals_local_attention(name, graph):
    from fastafd_b200.cad.gpu import (CadAttentionServer, CadModelHook, attention_window_layout, model_window_layout)
    from fastafd_b200.parallel.fabric import Fabric

    cfg = CFGS[name]
    ref_eng, ref_drv = _engine(cfg, graph)
    want = _tokens(ref_eng, ref_drv, 6)
    ref_eng.close()

    eng, drv = _engine(cfg, graph)
    w = eng.attn
    lanes, cap = w.num_mb, w.cap
    dev = torch.device("cuda:0")
    fabs = Fabric.local([model_window_layout(cfg, 1, lanes, cap).size, attention_window_layout(cfg, lanes, cap).size], dev)
    server = CadAttentionServer(cfg, fabs[1], model_rank=0, index=0, num_attn=1, num_lanes=lanes, max_tokens=cap,
                                num_pages=2, page_size=w.page_size, timeout_ns=int(2e9))
    server.k, server.v = w.kv.k, w.kv.v          # the attention side owns the KV cache (here: the prefilled one)
    hook = CadModelHook(cfg, fabs[0], [1], lanes, cap, servers=[server], timeout_ns=int(2e9))
    for lane in range(lanes):
        b = w.bufs[lane]
        # one attention GPU owns every row; its step metadata are the worker's own device buffers
        hook.set_step(lane, torch.zeros(cap, dtype=torch.int32, device=dev))
        server.n_rows[lane] = cap
        server.out_loc[lane], server.seq_lens[lane], server.page_table[lane] = b.out_loc, b.seq_lens, b.page_table
    w.model.cad = hook
    got = _tokens(eng, drv, 6)
    hook.check()
    assert int(w.status) == 0
    assert torch.equal(got, want)
    eng.close()
    for f in fabs:
        f.close()


def test_cad_wait_times_out_into_the_err_word():
    """A qkv flag that nothing sets: the fused wait + store gives up after its limit, records the
    timeout in the window's err word, stores nothing, and the context stays usable."""
    import ctypes as C

    from fastafd_b200.cad.gpu import _bind
    from fastafd_b200.ops._lib import check, cur_stream, ptr

    L = _bind()
    dev = "cuda:0"
    flag = torch.zeros(1, dtype=torch.int32, device=dev)
    epoch = torch.zeros(1, dtype=torch.int32, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    rows = torch.ones(4, 512, dtype=torch.bfloat16, device=dev)
    loc = torch.arange(4, dtype=torch.int32, device=dev)
    kc = torch.zeros(8, 1, 128, dtype=torch.bfloat16, device=dev)
    vc = torch.zeros_like(kc)
    check(L.afd_cad_wait_store(ptr(flag), ptr(epoch), ptr(rows), ptr(loc), ptr(kc), ptr(vc), 4, 512, 256, 128, 8,
                               C.c_ulonglong(int(0.2e9)), ptr(err), cur_stream()), "cad_wait_store")
    torch.cuda.synchronize()
    assert int(err) == 2 and float(kc.abs().sum()) == 0.0
    err.zero_()
    flag.fill_(1)
    check(L.afd_cad_wait_store(ptr(flag), ptr(epoch), ptr(rows), ptr(loc), ptr(kc), ptr(vc), 4, 512, 256, 128, 8,
                               C.c_ulonglong(int(0.2e9)), ptr(err), cur_stream()), "cad_wait_store")
    torch.cuda.synchronize()
    assert int(err) == 0 and float(kc[:4].float().sum()) == 4 * 128
