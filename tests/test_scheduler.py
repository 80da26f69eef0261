"""Lane scheduler, page ledgers, buckets: the host-side bookkeeping, with a CPU worker mirror
that applies only the plan's page grants (the worker must end up with the coordinator's
page table)."""
import numpy as np
import pytest

from fastafd_b200.core import SamplingParams
from fastafd_b200.scheduler.buckets import (balanced_split, default_decode_buckets, normalize_buckets, per_mb_real,
                                            select_bucket, split_prefill)
from fastafd_b200.scheduler.cache import NaivePageLedger, OutOfPages, RadixPageCache, mismatch_index
from fastafd_b200.scheduler.lane import AdmissionError, LaneScheduler


def test_bucket_ladder():
    b = default_decode_buckets(320)
    assert b[:4] == [1, 2, 4, 8] and 256 in b and 272 in b and 264 not in b and b[-1] == 320
    assert default_decode_buckets(20)[-1] == 20
    assert normalize_buckets((64, 8, 8), 256) == [8, 64]
    assert select_bucket(5, [1, 2, 4, 8]) == 8
    with pytest.raises(ValueError):
        select_bucket(9, [1, 2, 4, 8])
    assert per_mb_real(5, 2) == 3 and balanced_split(5, 2) == [3, 2] and balanced_split(1, 2) == [1, 0]


def test_prefill_split_at_request_boundaries():
    assert split_prefill([10, 10, 10, 10], 2) == [(0, 2), (2, 4)]
    assert split_prefill([30, 5, 5], 2) == [(0, 1), (1, 3)]
    assert split_prefill([7], 2) in ([(0, 1), (1, 1)], [(0, 0), (0, 1)])
    assert split_prefill([], 2) == [(0, 0), (0, 0)]


def test_naive_ledger():
    l = NaivePageLedger(8, 16)
    a = l.allocate(3)
    assert list(a) == [1, 2, 3] and l.free_pages == 4      # page 0 is reserved
    with pytest.raises(OutOfPages):
        l.allocate(5)
    l.free(a)
    l.check_integrity()
    with pytest.raises(RuntimeError):
        l.free([1])                                          # double free


def test_radix_cache_shares_and_evicts():
    c = RadixPageCache(10, 4)
    ids = list(range(13))
    pages, h = c.match_prefix(ids)
    assert pages == []
    own = list(c.allocate(4))
    c.release(h, ids, own, 13)                               # 3 full pages cached, 1 freed
    assert c.cached_pages == 3 and c.free_pages == 6
    pages, h2 = c.match_prefix(ids[:9] + [99, 98, 97, 96])
    assert pages == own[:2]
    assert mismatch_index(ids, ids[:9] + [99]) == 9
    c.check_integrity()
    # pinned pages cannot be evicted; the unpinned leaf can
    got = c.allocate(7)
    assert len(got) == 7 and c.cached_pages == 2
    with pytest.raises(OutOfPages):
        c.allocate(1)
    c.release(h2, ids[:9] + [99, 98, 97, 96], pages + list(got[:2]), 13)
    c.check_integrity()


class MirrorWorker:
    def __init__(self, rows, max_pages):
        self.table = np.zeros((rows + 1, max_pages), np.int32)

    def apply(self, plan):
        self.table[plan.grant_rows, plan.grant_slots] = plan.grant_pages


def test_page_grants_keep_worker_table_equal_to_ledger():
    s = LaneScheduler(0, num_pages=64, page_size=4, max_running=4, max_seq_len=64, num_mb=2, max_batched_tokens=8,
                      max_comm_tokens=8)
    w = MirrorWorker(4, 16)
    for uid, n in enumerate((11, 6, 3)):
        s.add_req(uid, list(range(n)), SamplingParams(max_tokens=6, ignore_eos=True))
    step = 0
    while not s.idle():
        if s.has_prefill():
            plan = s.schedule_prefill(step)
            assert sum(mb.num_tokens for mb in plan.mbs) <= 8        # chunked by the token budget
        else:
            plan = s.schedule_decode(step, 2)
        w.apply(plan)
        for st in s.states.values():
            pages = st.req.pages
            assert list(w.table[st.req.table_idx, :len(pages)]) == pages
            assert len(pages) == (st.planned_len + 3) // 4
        n = sum(len(mb.rows) for mb in plan.mbs)
        s.complete(step, np.full(n, 5, np.int32))
        s.check_integrity()
        step += 1
    assert s.cache.free_pages == 63 and sorted(s.free_rows) == [0, 1, 2, 3] and s.reserved_pages == 0


def test_padding_is_balanced_over_micro_batches():
    s = LaneScheduler(0, num_pages=64, page_size=16, max_running=8, max_seq_len=64, num_mb=2)
    for uid in range(3):
        s.add_prefilled(uid, 5, SamplingParams(max_tokens=4, ignore_eos=True))
    plan = s.schedule_decode(0, 4)
    assert [mb.num_real for mb in plan.mbs] == [2, 1]
    assert all(len(mb.rows) == 4 for mb in plan.mbs)
    assert (plan.mbs[0].rows[2:] == s.dummy_row).all() and (plan.mbs[1].seq_lens[1:] == 1).all()
    assert len(plan.grant_rows) == 3                         # the pre-admitted requests' first pages travel here


def test_admission_waits_for_pages_then_admits():
    s = LaneScheduler(0, num_pages=6, page_size=4, max_running=4, max_seq_len=32, num_mb=1)
    s.add_req(0, list(range(8)), SamplingParams(max_tokens=4, ignore_eos=True))   # 3 pages
    s.add_req(1, list(range(8)), SamplingParams(max_tokens=4, ignore_eos=True))   # 3 pages: does not fit yet
    assert s.has_prefill() and len(s.states) == 1 and len(s.waiting) == 1
    step = 0
    while not s.idle():
        plan = s.schedule_prefill(step) if s.has_prefill() else s.schedule_decode(step, 1)
        s.complete(step, np.full(sum(len(mb.rows) for mb in plan.mbs), 1, np.int32))
        step += 1
    assert not s.waiting and s.cache.free_pages == 5
    with pytest.raises(AdmissionError):
        s.add_req(2, list(range(30)), SamplingParams(max_tokens=30))


def test_native_mismatch_matches_numpy():
    import numpy as np

    from fastafd_b200.scheduler import cache

    rng = np.random.default_rng(0)
    for dt in (np.int32, np.int64):
        a = rng.integers(0, 1000, 4096).astype(dt)
        for cut in (0, 1, 17, 4095):
            b = a.copy()
            b[cut] += 1
            assert cache.mismatch_index(a, b) == cut
        assert cache.mismatch_index(a, a.copy()) == 4096
        assert cache.mismatch_index(a, a[:100].copy()) == 100
    assert cache._host_lib() is not None, "the host helper library should build with g++"


@pytest.mark.parametrize("cache_type", ["naive", "radix"])
def test_page_audit_runs_every_step_and_catches_a_corrupted_ledger(monkeypatch, cache_type):
    import numpy as np

    from fastafd_b200.core import SamplingParams
    from fastafd_b200.scheduler.lane import LaneScheduler

    monkeypatch.setenv("FASTAFD_PAGE_AUDIT", "1")
    s = LaneScheduler(0, num_pages=64, page_size=4, max_running=4, max_seq_len=64, num_mb=2, cache_type=cache_type)
    assert s.page_audit
    shared = list(range(100, 112))
    for uid in range(3):
        s.add_req(uid, shared + [200 + uid, 300 + uid], SamplingParams(max_tokens=6, ignore_eos=True))
    step = 0
    while not s.idle():
        plan = s.schedule_prefill(step) if s.has_prefill() else s.schedule_decode(step, 4)
        n = sum(len(m.rows) for m in plan.mbs)
        s.complete(step, np.full(n, 7, dtype=np.int32))           # audits inside plan and complete
        step += 1
    s.audit_pages()
    # a page that is free and held at once must be reported
    s.add_req(9, shared + [1, 2, 3], SamplingParams(max_tokens=2, ignore_eos=True))
    s.schedule_prefill(step)
    st = next(iter(s.states.values()))
    s.cache._free[s.cache._n_free] = st.req.pages[-1]
    s.cache._n_free += 1
    with pytest.raises(RuntimeError, match="page audit|corrupted"):
        s.audit_pages()


def test_kv_page_sizing(monkeypatch):
    """Pages from free memory: bytes per page follow the model (full-attention layers only for the
    hybrid family, KV heads per TP rank), an explicit count wins, and the request cap bounds it."""
    import torch

    from fastafd_b200.config import PRESETS, RuntimeConfig
    from fastafd_b200.models.transformer import KVPool
    from fastafd_b200.worker import attention_worker as aw

    cfg = PRESETS["qwen3-235b-a22b-fp8"]
    per_page = KVPool.bytes_per_page(cfg, 16, cfg.num_kv_heads)
    assert per_page == 94 * 2 * 16 * 4 * 128 * 2                    # layers x (K, V) x tokens x heads x dim x bf16
    assert KVPool.bytes_per_page(cfg, 16, 1) * 4 == per_page        # TP-4 rank holds one KV head
    hybrid = PRESETS["qwen3.5-397b-a17b-fp8"]
    full_layers = sum(1 for l in range(hybrid.num_layers) if hybrid.layer_type(l) == "full")
    assert KVPool.bytes_per_page(hybrid, 16, 2) == full_layers * 2 * 16 * 2 * hybrid.head_dim * 2

    rt = RuntimeConfig(page_size=16, max_running_requests=88, max_seq_len=8400, memory_ratio=0.9, device="cuda")
    monkeypatch.setattr(torch.cuda, "mem_get_info", lambda d: (170 << 30, 180 << 30))
    dev = torch.device("cuda", 0)
    want = 88 * (8400 // 16) + 1
    assert aw.determine_num_pages(cfg, rt, dev, cfg.num_kv_heads) == want          # everything fits: the request cap rules
    monkeypatch.setattr(torch.cuda, "mem_get_info", lambda d: (40 << 30, 180 << 30))
    got = aw.determine_num_pages(cfg, rt, dev, cfg.num_kv_heads)
    assert got == (int((40 << 30) * 0.9) - (2 << 30)) // per_page < want          # memory rules
    rt2 = RuntimeConfig(page_size=16, max_running_requests=88, max_seq_len=8400, num_pages=777, device="cuda")
    assert aw.determine_num_pages(cfg, rt2, dev, cfg.num_kv_heads) == 777


def test_decode_out_loc_native_and_bounds():
    import numpy as np

    from fastafd_b200.scheduler import cache

    rng = np.random.default_rng(1)
    pt = rng.integers(1, 50, size=(8, 6)).astype(np.int32)
    rows = np.array([3, 0, 7, 3], np.int32)
    pos = np.array([0, 17, 95, 40], np.int32)
    got = cache.decode_out_loc(pt, rows, pos, 16, 50)
    want = pt[rows, pos // 16] * 16 + pos % 16
    assert got.tolist() == want.tolist()
    pt[7, 5] = -1
    with pytest.raises(IndexError, match="request 2"):
        cache.decode_out_loc(pt, rows, pos, 16, 50)
    with pytest.raises(IndexError, match="request 1"):
        cache.decode_out_loc(pt, rows, np.array([0, 96, 1, 1], np.int32), 16, 50)     # past the last column


def test_attention_split_policy_matches_the_measured_optima():
    """pick_attn_splits is fitted to a sweep on B200 (profiles/decode_attention_paged_gqa.txt): these
    are the cases of that sweep, with the split count that was fastest (or within noise of it)."""
    from fastafd_b200.ops import pick_attn_splits as pick

    assert pick(64, 4, 1, 1040) == 1          # 256 CTAs already: more splits would need a second wave
    assert pick(32, 4, 1, 1040) == 2
    assert pick(16, 4, 1, 4096) == 4
    assert pick(44, 4, 1, 8200) == 2
    assert pick(8, 4, 1, 1040) == 4           # bounded by 256 tokens per split
    assert pick(1, 1, 1, 100) == 1            # never splits below 256 tokens
    assert pick(1, 4, 1, 131072) <= 32        # bounded by the merge table
    for B in (1, 3, 17, 100, 300):
        for kv in (64, 1000, 9000, 70000):
            s = pick(B, 4, 1, kv)
            assert 1 <= s <= 32 and (s == 1 or kv // s >= 256) and (s == 1 or B * 4 * s <= 148 * 3)
    assert pick(8, 2, 1, 16384, D=256) >= 1 and pick(200, 2, 1, 16384, D=256) == 1   # head_dim 256: one CTA per SM


@pytest.mark.parametrize("cache_type,spec_block,seed", [("naive", 0, 1), ("radix", 0, 2), ("naive", 4, 3), ("radix", 0, 4), ("naive", 0, 5)])
def test_randomised_soak_keeps_the_page_ledger_and_request_tables_consistent(monkeypatch, cache_type, spec_block, seed):
    """Random arrivals (shared prefixes, long prompts that need chunked prefill), aborts, EOS and stop tokens,
    steps planned one ahead of their completion (two under speculation) - with the page audit running
    after every planned and every completed step. Every admitted request finishes or is aborted, every
    output respects max_tokens, and at the end nothing is held."""
    import random

    import numpy as np

    from fastafd_b200.core import SamplingParams
    from fastafd_b200.scheduler.buckets import normalize_buckets, per_mb_real, select_bucket
    from fastafd_b200.scheduler.lane import AdmissionError, LaneScheduler

    monkeypatch.setenv("FASTAFD_PAGE_AUDIT", "1")
    rng = random.Random(seed)
    num_mb, max_running = 2, 6
    s = LaneScheduler(0, num_pages=96, page_size=4, max_running=max_running, max_seq_len=96, num_mb=num_mb,
                      max_batched_tokens=24, cache_type=cache_type, eos_token_ids=(3,), spec_block=spec_block, spec_pending=2)
    buckets = normalize_buckets((), 8)
    q = spec_block if spec_block > 1 else 1
    window = 2
    prefixes = [[50 + i for i in range(9)], [70 + i for i in range(5)]]
    next_uid, step, inflight, outputs, limits, aborted, arrivals = 0, 0, [], {}, {}, set(), 40
    for _ in range(3000):
        # arrivals and aborts
        if arrivals and rng.random() < 0.35:
            ids = (rng.choice(prefixes) if rng.random() < 0.5 else []) + [rng.randrange(10, 40) for _ in range(rng.randint(1, 30))]
            sp = SamplingParams(max_tokens=rng.randint(1, 12), ignore_eos=rng.random() < 0.5,
                                stop_token_ids=(5,) if rng.random() < 0.2 else ())
            try:
                s.add_req(next_uid, ids, sp)
                outputs[next_uid], limits[next_uid] = [], sp
            except AdmissionError:
                pass
            next_uid += 1
            arrivals -= 1
        live = [u for u in outputs if u in s.states and u not in aborted]
        if live and rng.random() < 0.05:
            u = rng.choice(live)
            s.abort(u)
            aborted.add(u)
        # plan a step when the window has room
        if len(inflight) < window and not s.idle():
            if s.has_prefill():
                plan = s.schedule_prefill(step)
            elif s.decode_real() > 0:
                bucket = select_bucket(per_mb_real(s.decode_real(), num_mb), buckets)
                plan = s.schedule_decode(step, bucket, q)
            else:
                plan = None
                s.check_admission_stall()
            if plan is not None:
                inflight.append((step, plan))
                step += 1
        # complete the oldest step (always, when the window is full or nothing new can be planned)
        if inflight and (len(inflight) >= window or rng.random() < 0.6 or s.idle()):
            sid, plan = inflight.pop(0)
            rows = sum(len(m.rows) for m in plan.mbs)
            blk = q if plan.phase == "verify" else 1
            toks = np.array([rng.choice([3, 5, 7, 8, 9, 11]) for _ in range(rows * blk)], dtype=np.int32)
            acc = np.array([rng.randint(1, blk) for _ in range(rows)], dtype=np.int32) if blk > 1 else None
            for uid, new, fin in s.complete(sid, toks, acc):
                outputs[uid] += new
                assert len(outputs[uid]) <= limits[uid].max_tokens
                if fin:
                    last = outputs[uid][-1]
                    assert (len(outputs[uid]) == limits[uid].max_tokens or last in limits[uid].stop_token_ids
                            or (last == 3 and not limits[uid].ignore_eos))
        if not arrivals and s.idle() and not inflight:
            break
    else:
        raise AssertionError("the lane did not drain")
    s.audit_pages()
    s.check_integrity()
    assert not s.states and len(s.free_rows) == max_running
    assert sum(1 for u in outputs if outputs[u]) > 10


def test_kv_pages_are_priced_as_the_pool_allocates_them(monkeypatch):
    """Hybrid model (Qwen3.5-397B: 60 layers, every fourth with full attention, 2 KV heads of 256): a page costs
    K and V of the full-attention layers only, the budget is memory_ratio of what is free at that moment minus a
    reserve, the request table caps it, an explicit page count wins; and the worker builds the recurrent-state
    pool (fixed size, tens of GB at this scale) before it sizes the KV pool from what is left."""
    import inspect

    import torch

    from fastafd_b200.config import RuntimeConfig, get_model_config
    from fastafd_b200.models.transformer import KVPool
    from fastafd_b200.worker import attention_worker as aw

    cfg = get_model_config("qwen3.5-397b-a17b-fp8")
    assert cfg.num_full_attn_layers == 15 and cfg.num_linear_layers == 45
    per_page = KVPool.bytes_per_page(cfg, 16, 2, 2)
    assert per_page == 2 * 15 * 16 * 2 * 256 * 2
    GIB = 1 << 30
    free = {"now": 100 * GIB}
    monkeypatch.setattr(torch.cuda, "mem_get_info", lambda dev=None: (free["now"], 180 * GIB))
    dev = torch.device("cuda", 0)
    rt = RuntimeConfig(page_size=16, max_running_requests=256, max_seq_len=262144, memory_ratio=0.9)
    n_before = aw.determine_num_pages(cfg, rt, dev, 2, 2)
    assert n_before == (int(100 * GIB * 0.9) - 2 * GIB) // per_page
    free["now"] -= 46 * GIB                                   # the recurrent state of 257 request slots is resident
    n_after = aw.determine_num_pages(cfg, rt, dev, 2, 2)
    assert n_after == (int(54 * GIB * 0.9) - 2 * GIB) // per_page < n_before
    short = RuntimeConfig(page_size=16, max_running_requests=8, max_seq_len=1024, memory_ratio=0.9)
    assert aw.determine_num_pages(cfg, short, dev, 2, 2) == 8 * 64 + 1            # the request table cannot use more
    assert aw.determine_num_pages(cfg, RuntimeConfig(num_pages=77), dev, 2, 2) == 77
    src = inspect.getsource(aw.AttentionWorker.__init__)
    assert src.index("GDNStatePool(") < src.index("determine_num_pages(") < src.index("KVPool(")
    # the state pool's size at this scale: an fp32 [heads, dv, dk] matrix per linear-attention layer and request slot
    slot_bytes = cfg.num_linear_layers * cfg.gdn_num_v_heads * cfg.gdn_head_v_dim * cfg.gdn_head_k_dim * 4
    assert 40 * GIB < 257 * slot_bytes < 50 * GIB
