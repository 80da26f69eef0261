"""Protocol simulation of one attention TP lane (fused collectives) with its expert GPUs.

The kernels of every stream are modelled as a queue of operations with the blocking behaviour of
the real ones: a flag wait passes when every awaited flag has reached the expected epoch, a flag
release publishes the sender's next epoch, an NCCL collective passes when every member has reached
the same call, `wait_stream` orders one stream after what another has queued. Streams are advanced
in random order. The test checks that (1) every schedule runs to completion (no deadlock), and
(2) buffers are reused safely: a peer never overwrites a gather or reduce-scatter slot before its
previous contents have been consumed. Deliberately broken variants (a lost release; dense layers
with no all-gather between two reduce-scatters) must be caught.

The op sequences mirror worker/attention_worker.py (_pipeline, _compute, _combine),
parallel/tp_fused.py and worker/expert_worker.py.
"""
import random

import pytest


class Deadlock(Exception):
    pass


class Race(Exception):
    pass


class Sim:
    def __init__(self, seed):
        self.rng = random.Random(seed)
        self.streams = {}            # name -> list of ops
        self.pos = {}                # name -> index of next op
        self.flags = {}              # flag key -> epoch
        self.publish = {}            # publisher key -> next epoch to publish
        self.expect = {}             # consumer key -> next epoch to expect
        self.slot_written = {}       # buffer slot -> epoch of the data in it
        self.slot_consumed = {}      # buffer slot -> epoch last read

    def add(self, stream, op):
        self.streams.setdefault(stream, []).append(op)
        self.pos.setdefault(stream, 0)
        return len(self.streams[stream])          # position after this op (for wait_stream)

    def done_upto(self, stream):
        return self.pos.get(stream, 0)

    def step(self, name):
        """Try to run the head op of a stream; True if it ran."""
        ops, i = self.streams[name], self.pos[name]
        if i >= len(ops):
            return False
        op = ops[i]
        kind = op[0]
        if kind == "wait_stream":                  # ordered after op index `upto` of another stream
            _, other, upto = op
            if self.done_upto(other) < upto:
                return False
        elif kind == "wait":                       # flags >= expected epoch; then bump
            _, keys, ekey = op
            e = self.expect.setdefault(ekey, 1)
            if any(self.flags.get(k, 0) < e for k in keys):
                return False
            self.expect[ekey] = e + 1
        elif kind == "write":                      # producer stores into peer slots, then releases flags
            _, pkey, slots, flag_keys = op
            e = self.publish.setdefault(pkey, 1)
            for s in slots:
                if getattr(self, "check_races", True) and self.slot_written.get(s, 0) > self.slot_consumed.get(s, 0):
                    raise Race(f"{name}: slot {s} overwritten (epoch {e}) before epoch {self.slot_written[s]} was read")
                self.slot_written[s] = e
            for k in flag_keys:
                self.flags[k] = e
            self.publish[pkey] = e + 1
        elif kind == "read":                       # consumer reads slots (after its wait)
            _, slots = op
            for s in slots:
                self.slot_consumed[s] = self.slot_written.get(s, 0)
        elif kind == "nccl":                       # passes when every member's head is this call
            _, members, tag = op
            for m in members:
                mo, mi = self.streams[m], self.pos[m]
                if mi >= len(mo) or mo[mi] != ("nccl", members, tag):
                    return False
            for m in members:
                self.pos[m] += 1
            return True
        elif kind == "compute":
            pass
        else:
            raise AssertionError(kind)
        self.pos[name] = i + 1
        return True

    def run(self):
        names = list(self.streams)
        while any(self.pos[n] < len(self.streams[n]) for n in names):
            self.rng.shuffle(names)
            if not any(self.step(n) for n in names):
                stuck = {n: self.streams[n][self.pos[n]] for n in names if self.pos[n] < len(self.streams[n])}
                raise Deadlock(str(stuck)[:600])


def build(sim, tp=4, n_eg=4, lanes=2, layers=3, steps=2, drop_release=None, skip_gather=False, moe=True):
    ag = list(range(tp))
    main = {r: f"ag{r}.main" for r in ag}
    lane_s = {(r, l): f"ag{r}.lane{l}" for r in ag for l in range(lanes)}
    members = tuple(main[r] for r in ag)
    count = {"n": 0}

    def nccl(tag):
        for r in ag:
            sim.add(main[r], ("nccl", members, tag))

    def compute(r, layer, lane, step):
        m = main[r]
        if not (skip_gather and layer >= 1):
            # all-gather: store my rows into every rank's gather slot, then wait for all ranks' rows
            slots = [("ag_buf", p, lane, r) for p in ag]
            flags = [("ag_flag", p, lane, r) for p in ag]
            sim.add(m, ("write", ("ag_pub", r, lane), slots, flags))
            sim.add(m, ("wait", [("ag_flag", r, lane, s) for s in ag], ("ag_exp", r, lane)))
            sim.add(m, ("read", [("ag_buf", r, lane, s) for s in ag]))          # qkv GEMM reads the gathered rows
        sim.add(m, ("compute",))                                                # norm + RoPE, attention
        # o_proj GEMM epilogue: partial rows into every owner's slot of this source, flags by the last CTA
        count["n"] += 1
        rel = [("rs_flag", p, lane, r) for p in ag]
        if drop_release == count["n"]:
            rel = rel[1:]
        sim.add(m, ("write", ("rs_pub", r, lane), [("rs_buf", p, lane, r) for p in ag], rel))
        sim.add(m, ("wait", [("rs_flag", r, lane, s) for s in ag], ("rs_exp", r, lane)))   # one-warp wait
        sim.add(m, ("read", [("rs_buf", r, lane, s) for s in ag]))                          # sum of partials
        if moe:     # route + dispatch: rows into the expert GPUs' receive slots of this source
            sim.add(m, ("write", ("n2m_pub", r, lane), [("recv", e, lane, r) for e in range(n_eg)],
                        [("n2m_flag", e, lane, r) for e in range(n_eg)]))

    def combine(r, lane):
        if not moe:
            return
        ls = lane_s[(r, lane)]
        sim.add(ls, ("wait", [("m2n_flag", r, lane, e) for e in range(n_eg)], ("m2n_exp", r, lane)))
        upto = sim.add(ls, ("read", [("combine", r, lane, e) for e in range(n_eg)]))
        sim.add(main[r], ("wait_stream", ls, upto))                              # _join_lane

    for step in range(steps):
        for lane in range(lanes):                      # embedding + layer 0
            nccl(("embed_rs", step, lane))
            for r in ag:
                compute(r, 0, lane, step)
        for layer in range(layers):
            for lane in range(lanes):
                for r in ag:
                    combine(r, lane)
                    if layer + 1 < layers:
                        compute(r, layer + 1, lane, step)
        for lane in range(lanes):                      # LM head
            nccl(("lm_head_ag", step, lane))
            nccl(("logits_ag", step, lane))
        for e in range(n_eg if moe else 0):            # expert GPU: every layer, lane after lane
            es = f"eg{e}"
            for layer in range(layers):
                for lane in range(lanes):
                    sim.add(es, ("wait", [("n2m_flag", e, lane, r) for r in ag], ("n2m_exp", e, lane)))
                    sim.add(es, ("read", [("recv", e, lane, r) for r in ag]))
                    sim.add(es, ("write", ("m2n_pub", e, lane), [("combine", r, lane, e) for r in ag],
                                 [("m2n_flag", r, lane, e) for r in ag]))


@pytest.mark.parametrize("tp,n_eg,lanes", [(2, 2, 2), (4, 4, 2), (4, 4, 1), (8, 2, 3)])
def test_every_schedule_completes_without_overwriting_unread_slots(tp, n_eg, lanes):
    for seed in range(40):
        sim = Sim(seed)
        build(sim, tp=tp, n_eg=n_eg, lanes=lanes, layers=3, steps=2)
        sim.run()
        assert all(sim.pos[n] == len(sim.streams[n]) for n in sim.streams)


def test_a_lost_flag_release_is_reported_as_a_deadlock():
    sim = Sim(0)
    build(sim, tp=4, n_eg=4, lanes=2, layers=3, steps=1, drop_release=5)
    with pytest.raises(Deadlock):
        sim.run()


def test_reduce_scatter_without_anything_in_between_is_a_race():
    """Something must order a peer's next partial-row store after this rank's read of the previous
    partials: the layer's all-gather does (and, in MoE layers, so does the round trip through the
    expert GPUs, which wait for every source). With neither - dense layers, no gather - some
    schedule overwrites an unread slot, and the simulator has to see it."""
    for seed in range(10):                               # MoE layers alone already give the ordering
        sim = Sim(seed)
        build(sim, tp=4, n_eg=4, lanes=1, layers=3, steps=1, skip_gather=True, moe=True)
        sim.run()
    hit = 0
    for seed in range(60):
        sim = Sim(seed)
        build(sim, tp=4, n_eg=4, lanes=1, layers=3, steps=1, skip_gather=True, moe=False)
        try:
            sim.run()
        except Race:
            hit += 1
    assert hit > 0


def _run_with_timeouts(sim, rank_of):
    """Like Sim.run, with the failure behaviour of the kernels: when nothing can move, every stream
    whose head is an unsatisfied flag wait lets that wait run out (one time limit passes for all of
    them at once, they wait in parallel); the rank's status word is then set, and every later flag
    wait of that rank returns at once (all its communicators share the word). Returns the number of
    time limits that passed and the set of ranks whose status word is set."""
    names = list(sim.streams)
    failed, limits = set(), 0
    while any(sim.pos[n] < len(sim.streams[n]) for n in names):
        sim.rng.shuffle(names)
        moved = False
        for n in names:
            i = sim.pos[n]
            if i < len(sim.streams[n]) and sim.streams[n][i][0] == "wait" and rank_of(n) in failed:
                _, keys, ekey = sim.streams[n][i]          # status already set: the wait gives up at once
                sim.expect[ekey] = sim.expect.setdefault(ekey, 1) + 1
                sim.pos[n] = i + 1
                moved = True
            elif sim.step(n):
                moved = True
        if moved:
            continue
        stuck = [n for n in names if sim.pos[n] < len(sim.streams[n]) and sim.streams[n][sim.pos[n]][0] == "wait"]
        if not stuck:
            raise Deadlock("stuck without a waiting kernel")
        limits += 1
        sim.check_races = False          # a failed step's data is discarded; only termination matters from here
        for n in stuck:
            failed.add(rank_of(n))
        assert limits <= 8, "time-outs keep cascading"
    return limits, failed


@pytest.mark.parametrize("drop", [3, 5, 12])
def test_a_withheld_flag_ends_the_step_on_all_eight_ranks_within_two_time_limits(drop):
    """4 attention TP ranks + 4 expert ranks, one flag release withheld. The ranks that wait for it
    give up after one time limit and set their status word; everything they do afterwards drains
    without waiting (their flags are still released, with garbage behind them), so no rank waits for
    a second full limit in sequence: the whole step ends on all eight ranks after at most two limits,
    and at least one rank carries the error that the step's token exchange then spreads."""
    for seed in range(10):
        sim = Sim(seed)
        build(sim, tp=4, n_eg=4, lanes=2, layers=3, steps=1, drop_release=drop)
        limits, failed = _run_with_timeouts(sim, lambda n: n.split(".")[0])
        assert all(sim.pos[n] == len(sim.streams[n]) for n in sim.streams)       # every rank returned
        assert 1 <= limits <= 2, limits
        assert failed, "nobody noticed the withheld flag"
