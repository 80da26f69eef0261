"""Tiny Qwen3-MoE-shaped AFD decode on CPU/gloo: world 2 (rank 0 attention server, rank 1
MLP server), fp32, 4 requests x 32 prompt tokens, 16 greedy tokens, 2 micro-batches. The
output must match the single-process engine token for token. Also a 2+2 layout."""
import os
import socket
import tempfile

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from fastafd_b200.config import PRESETS, RuntimeConfig
from fastafd_b200.core import SamplingParams
from fastafd_b200.engine import AfdEngine, SpmdDriver
from fastafd_b200.protocol import AfdTopology


def _rt():
    return RuntimeConfig(model_path="tiny-qwen3-moe", num_mb=2, page_size=16, num_pages=64, max_running_requests=8,
                         max_seq_len=128, cuda_graph_max_bs=8, device="cpu", dtype="float32", use_cuda_graph=False)


def _prompts(cfg, n=4, length=32):
    g = torch.Generator().manual_seed(0)
    return [torch.randint(0, cfg.vocab_size, (length,), generator=g).tolist() for _ in range(n)]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, topo_kw, out_path, n_new):
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    torch.set_num_threads(1)
    cfg = PRESETS["tiny-qwen3-moe"]
    topo = AfdTopology(**topo_kw)
    eng = AfdEngine(cfg, _rt(), topo, rank, "cpu", seed=0)
    out = SpmdDriver(eng).generate(_prompts(cfg), SamplingParams(max_tokens=n_new, ignore_eos=True))
    if rank == 0:
        torch.save(out, out_path)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("topo_kw", [dict(attn_dp=1, mlp_ep=1), dict(attn_dp=2, mlp_ep=2),
                                     dict(attn_dp=1, attn_tp=2, mlp_ep=2),
                                     dict(attn_dp=2, mlp_dp=2, mlp_ep=1),           # two expert replicas, one per lane
                                     dict(attn_dp=1, mlp_tp=2, mlp_ep=1)],          # experts sharded along the intermediate dim
                         ids=["1+1", "dp2+ep2", "tp2+ep2", "dp2+mlpdp2", "1+mlptp2"])
def test_gloo_afd_matches_single_process(topo_kw):
    cfg = PRESETS["tiny-qwen3-moe"]
    n_new = 16
    single = AfdEngine(cfg, _rt(), AfdTopology(colocated=True), 0, "cpu", seed=0)
    exp = SpmdDriver(single).generate(_prompts(cfg), SamplingParams(max_tokens=n_new, ignore_eos=True))
    world = AfdTopology(**topo_kw).world
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "out.pt")
        mp.spawn(_worker, args=(world, _free_port(), topo_kw, path, n_new), nprocs=world, join=True)
        got = torch.load(path)
    assert got == exp


def _steps_worker(rank, world, port, topo_kw, out_path):
    """The benchmark's flow: prefilled requests, then decode steps in lock-step and one step ahead."""
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    torch.set_num_threads(1)
    cfg = PRESETS["tiny-qwen3-moe"]
    topo = AfdTopology(**topo_kw)
    eng = AfdEngine(cfg, _rt(), topo, rank, "cpu", seed=0)
    drv = SpmdDriver(eng)
    # 9 tokens each, the first of which the (skipped) prefill already produced: 8 decode steps drain the batch
    drv.install_prefilled(6, 20, max_tokens=9)
    a = drv.run_decode_steps(4, pipelined=False)
    b = drv.run_decode_steps(5, pipelined=True)
    c = drv.run_decode_steps(3, pipelined=False)         # nothing left to decode: empty steps
    res = torch.tensor([a, b, c, max(l.decode_real() for l in drv.lanes)])
    out = [torch.zeros(4, dtype=torch.int64) for _ in range(world)]
    dist.all_gather(out, res)
    if rank == 0:
        torch.save(torch.stack(out), out_path)
    dist.barrier()
    dist.destroy_process_group()


def test_decode_step_driver_keeps_ranks_in_step_with_shadow_lanes():
    """Every rank plans only its own lane and advances the others as shadows; all ranks must agree
    on the bucket of every step (else the gloo exchange would block) and attention ranks must
    produce exactly their lane's tokens, including the steps in which the batch runs dry."""
    topo_kw = dict(attn_dp=2, mlp_ep=2)
    world = 4
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "out.pt")
        mp.spawn(_steps_worker, args=(world, _free_port(), topo_kw, path), nprocs=world, join=True)
        res = torch.load(path)
    for r in range(2):                                   # attention ranks: 6 requests x (4 + 4) tokens, then none
        assert res[r].tolist() == [24, 24, 0, 0]
    for r in range(2, 4):                                # expert ranks produce no tokens but see the same drain
        assert res[r].tolist() == [0, 0, 0, 0]


def _sampling_worker(rank, world, port, out_dir, seed, extra_draw_on):
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    torch.set_num_threads(1)
    cfg = PRESETS["tiny-qwen3-moe"]
    rt = _rt()
    rt.seed = seed
    if rank == extra_draw_on:
        torch.rand(7)                     # an unrelated draw on ONE rank must not desynchronise the lane
    eng = AfdEngine(cfg, rt, AfdTopology(attn_dp=1, attn_tp=2, mlp_ep=2), rank, "cpu", seed=0)
    sp = SamplingParams(max_tokens=10, ignore_eos=True, temperature=0.9, top_k=40, top_p=0.95)
    out = SpmdDriver(eng).generate(_prompts(cfg), sp)
    if eng.attn is not None:
        # what this TP rank itself sampled sits in its token pool: rows of the first request
        torch.save({"out": out, "pool": eng.attn.token_pool[:4, 32:42].clone()}, os.path.join(out_dir, f"r{rank}.pt"))
    dist.barrier()
    dist.destroy_process_group()


def test_sampled_tokens_agree_across_tp_ranks_and_follow_the_seed():
    """Temperature sampling under attention TP: every TP rank of a lane draws from a generator seeded
    by (seed, lane, step, micro-batch), so the ranks pick the same tokens even if one of them consumed
    other random numbers, and the output is a function of --seed."""
    runs = {}
    for seed, extra in ((5, 0), (5, 1), (6, -1)):
        with tempfile.TemporaryDirectory() as d:
            mp.spawn(_sampling_worker, args=(4, _free_port(), d, seed, extra), nprocs=4, join=True)
            r0, r1 = torch.load(os.path.join(d, "r0.pt")), torch.load(os.path.join(d, "r1.pt"))
        assert torch.equal(r0["pool"], r1["pool"])             # both TP ranks wrote the same sampled tokens
        runs[(seed, extra)] = r0["out"]
    assert runs[(5, 0)] == runs[(5, 1)]                        # same seed -> same tokens, whoever drew extra numbers
    assert runs[(5, 0)] != runs[(6, -1)]                       # another seed -> other tokens
