"""Benchmark suite: every configuration is well formed; the statistics match hand-computed values."""
import json

import pytest

from fastafd_b200.benchmark import run_stats, suite


def test_every_config_is_well_formed_and_has_a_command():
    cfgs = suite.load_configs()
    assert suite.validate(cfgs) == []
    for name, c in cfgs["configs"].items():
        cmd = suite.command(name, c, steps=4, warmup=3)
        assert "bench.py" in cmd and str(c["batch"]) in cmd
        assert ("torch.distributed.run" in cmd) == (c["gpus"] > 1)


def test_throughput_formula_and_verdict():
    # 4+4 GPUs, 108 requests per attention GPU, 35.008 ms per step -> 1542 tok/s/GPU
    assert run_stats.throughput_per_gpu(108, 35.008, 4, 4) == pytest.approx(1542.5, abs=0.5)
    # 6+2 (3:1), 106 requests, 34.735 ms -> 2289
    assert run_stats.throughput_per_gpu(106, 34.735, 6, 2) == pytest.approx(2288.8, abs=0.5)
    assert run_stats.verdict(35.9, 35.0)[0] == "pass"
    assert run_stats.verdict(36.2, 35.0)[0] == "fail"
    assert run_stats.verdict(36.2, None) == ("unrecorded", None)


def test_decode_window_and_step_mean():
    lines = [f"[afd-step-time] step={i} phase=prefill bucket=0 num_mb=2 ms=50.0 real=8" for i in range(3)]
    lines += [f"[afd-step-time] step={3 + i} phase=decode bucket=8 num_mb=2 ms={10 + (i == 0) * 5:.3f} real=8" for i in range(6)]
    lines += ["[afd-step-time] step=9 phase=decode bucket=8 num_mb=2 ms=7.000 real=[3, 2]"]  # batch draining, per-lane counts
    s = run_stats.parse_step_lines(["noise"] + lines)
    assert len(s) == 10
    w = run_stats.decode_window(s)
    assert [x.step for x in w] == [3, 4, 5, 6, 7, 8]
    assert run_stats.step_mean(w, skip=1) == pytest.approx(10.0)


def test_wall_period_is_inverse_slope():
    ids = list(range(100, 200))
    ts = [5.0 + 0.0125 * (i - 100) for i in ids]
    assert run_stats.wall_period(ids, ts) == pytest.approx(0.0125)


def test_evaluate_bench_line():
    cfgs = suite.load_configs()
    c = cfgs["configs"]["qwen3-235b-8k-1to1"]
    rec = c["recorded"]["step_ms"]
    line = json.dumps({"metric": "m", "value": 4 * c["batch"] / (rec * 1.01 / 1e3), "n_gpus": 8, "ms_per_step": rec * 1.01,
                       "e2e": {"ms_per_step": rec * 1.03}})
    res = suite.evaluate(c, line, 0.03)
    want = 4 * c["batch"] / (rec * 1.01 / 1e3) / 8
    assert res["verdict"] == "pass" and res["tok_s_per_gpu"] == pytest.approx(want, rel=1e-3)
    assert res["vs_published"] == pytest.approx(want / c["published"]["tok_s_per_gpu"], abs=0.002)
    slow = json.dumps({"metric": "m", "value": 1.0, "n_gpus": 8, "ms_per_step": rec * 1.05, "e2e": {"ms_per_step": rec * 1.06}})
    assert suite.evaluate(c, slow, 0.03)["verdict"] == "fail"


def test_trace_reader_and_scaling(tmp_path):
    from fastafd_b200.benchmark.client import read_trace, scale_trace

    p = tmp_path / "trace.jsonl"
    p.write_text("\n".join([
        json.dumps({"timestamp": 5000, "input_length": 100, "output_length": 20, "hash_ids": [1, 2]}),
        json.dumps({"timestamp": 3000, "input_length": 50, "output_length": 10}),
        "not json",
        json.dumps({"timestamp": 9000, "input_length": 0, "output_length": 10}),           # dropped: empty prompt
        json.dumps({"timestamp": 7000, "input_length": 4000, "output_length": 900}),
    ]))
    tr = read_trace(str(p))
    assert [(e.at_s, e.input_length) for e in tr] == [(0.0, 50), (2.0, 100), (4.0, 4000)]
    sc = scale_trace(tr, time_scale=0.5, max_requests=3, max_input=1024, max_output=128)
    assert [(e.at_s, e.input_length, e.output_length) for e in sc] == [(0.0, 50, 10), (1.0, 100, 20), (2.0, 1024, 128)]


def test_record_and_summary(tmp_path):
    import shutil

    cfg_copy = tmp_path / "configs.json"
    shutil.copy(suite.HERE / "configs.json", cfg_copy)
    run_dir = tmp_path / "runs" / "qwen3-235b-8k-1to1-20260101T000000Z"
    run_dir.mkdir(parents=True)
    (run_dir / "config.json").write_text(json.dumps({"name": "qwen3-235b-8k-1to1"}))
    (run_dir / "result.json").write_text(json.dumps({"step_ms": 33.3333, "tok_s_per_gpu": 1320.4, "verdict": "unrecorded"}))
    rec = suite.record("qwen3-235b-8k-1to1", run_dir, cfg_copy)
    assert rec == {"step_ms": 33.333, "tok_s_per_gpu": 1320}
    assert json.loads(cfg_copy.read_text())["configs"]["qwen3-235b-8k-1to1"]["recorded"] == rec
    rows = suite.summary(tmp_path / "runs")
    assert len(rows) == 1 and rows[0]["step_ms"] == 33.3333
    (run_dir / "result.json").write_text(json.dumps({"verdict": "error", "returncode": 1}))
    with pytest.raises(ValueError):
        suite.record("qwen3-235b-8k-1to1", run_dir, cfg_copy)


def test_bench_picks_micro_batches_from_the_layer_model():
    """Two micro-batches only where an expert GPU's weight stream is short next to the attention chain."""
    import importlib.util
    import os

    from fastafd_b200.config import get_model_config
    from fastafd_b200.protocol import AfdTopology

    path = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "bench.py")
    spec = importlib.util.spec_from_file_location("bench_under_test", path)
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    cfg = get_model_config("qwen3-30b-a3b")
    picks = {w: bench.pick_num_mb(cfg, AfdTopology.for_world(w), 64, 1024) for w in (1, 2, 4, 8)}
    assert picks == {1: 1, 2: 1, 4: 1, 8: 2}
    big = get_model_config("qwen3-235b-a22b-fp8")
    assert bench.pick_num_mb(big, AfdTopology.for_world(8), 88, 8192) == 2
    # the 8-GPU default is the named configuration (one TP-4 attention lane + EP-4), data-parallel lanes elsewhere
    assert [bench.default_attn_tp(w) for w in (1, 2, 4, 8)] == [1, 1, 1, 4]
    assert bench.default_attn_tp(8, attn_gpus=6) == 1
    t = AfdTopology.for_world(8, attn_tp=bench.default_attn_tp(8))
    assert (t.attn_dp, t.attn_tp, t.mlp_ep) == (1, 4, 4)


def test_experiment_presets_build_valid_bench_commands(tmp_path):
    """Every preset is a thin wrapper around one runner: with DRY_RUN=1 it prints the bench command
    it would launch; the model must be a known preset and the batch must split over the micro-batches."""
    import glob
    import os
    import subprocess

    from fastafd_b200.config import get_model_config

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    presets = sorted(p for p in glob.glob(os.path.join(root, "fastafd_b200", "benchmark", "experiments", "*.sh"))
                     if not p.endswith("common.sh"))
    assert len(presets) >= 8
    for p in presets:
        env = dict(os.environ, DRY_RUN="1", RUN_DIR=str(tmp_path / os.path.basename(p)))
        out = subprocess.run(["bash", p], env=env, capture_output=True, text=True, timeout=60)
        assert out.returncode == 0, (p, out.stderr)
        cmd = next(ln for ln in out.stdout.splitlines() if ln.startswith("== ")).split(": ", 1)[1].split()
        assert "bench.py" in cmd
        arg = lambda k: cmd[cmd.index(k) + 1]  # noqa: E731
        get_model_config(arg("--model"))
        gpus = int(arg("--gpus"))
        assert gpus in (1, 2, 4, 8) and int(arg("--batch-per-attn-gpu")) > 0 and int(arg("--context")) >= 1024
        if gpus > 1:
            assert f"--nproc-per-node {gpus}" in " ".join(cmd) and "127.0.0.1" in cmd
            assert int(arg("--attn-gpus")) < gpus
        if "--num-mb" in cmd:
            assert int(arg("--batch-per-attn-gpu")) % int(arg("--num-mb")) == 0
        if "SUITE_NAME" in open(p).read():
            from fastafd_b200.benchmark import suite
            name = [ln for ln in open(p).read().splitlines() if "SUITE_NAME" in ln][0].split(":-")[1].rstrip('}"')
            assert name in suite.load_configs()["configs"]


def test_long_prompt_base_is_deterministic_and_sliced_contiguously(tmp_path):
    from fastafd_b200.benchmark import long_prompts as lp

    a = lp.synthetic(6, 300, vocab=5000, seed=7, shared_prefix=64)
    b = lp.synthetic(6, 300, vocab=5000, seed=7, shared_prefix=64)
    assert a == b and all(len(p) == 300 for p in a)
    assert all(p[:64] == a[0][:64] for p in a) and a[0][64:] != a[1][64:]
    assert all(16 <= t < 5000 for p in a for t in p)
    # Zipf-like: the most frequent id is far above the uniform share; phrases repeat inside a prompt
    flat = [t for p in lp.synthetic(4, 4000, vocab=5000, seed=1) for t in p]
    top = max(flat.count(t) for t in set(flat[:200]))
    assert top > 20 * len(flat) / 5000
    lp.save(a, tmp_path / "base.jsonl")
    assert lp.load(str(tmp_path / "base.jsonl")) == a
    assert lp.load(str(tmp_path / "base.jsonl"), max_prompts=2, max_tokens=10) == [p[:10] for p in a[:2]]
    # document slices: contiguous, exact length, round-robin over documents, short documents skipped
    docs = [list(range(1000, 1950)), list(range(5000, 5100)), list(range(9000, 9700))]
    sl = lp.slices_of_documents(docs, 5, 200, seed=3)
    assert len(sl) == 5 and all(len(s) == 200 and s == list(range(s[0], s[0] + 200)) for s in sl)
    assert {s[0] // 1000 for s in sl} == {1, 9}
    import pytest
    with pytest.raises(ValueError):
        lp.slices_of_documents(docs, 50, 200, seed=3)
    assert lp.main(["--count", "3", "--target-tokens", "128", "--vocab", "1024", "--output", str(tmp_path / "o.jsonl")]) == 0
    assert len(lp.load(str(tmp_path / "o.jsonl"))) == 3


def test_clock_samples_are_taken_from_inside_the_timed_region():
    import datetime
    import importlib.util
    import os

    path = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "bench.py")
    spec = importlib.util.spec_from_file_location("bench_under_test2", path)
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)

    base = datetime.datetime(2026, 1, 2, 3, 4, 5).timestamp()

    def line(dt, sm, cap="Not Active", hw="Not Active"):
        ts = datetime.datetime.fromtimestamp(base + dt).strftime("%Y/%m/%d %H:%M:%S.%f")[:-3]
        return f"{ts}, 3, {sm}, 1965, 712.5, 0x0000000000000004, {hw}, Not Active, Not Active, {cap}"

    lines = [line(0.00, 345), line(0.10, 1965), line(0.20, 1905, cap="Active"), line(0.30, 1935), line(0.40, 600, hw="Active")]
    inside = bench.summarize_clock_samples(lines, base + 0.05, base + 0.35)
    assert inside == {"sm_mhz": 1935.0, "sm_max_mhz": 1965.0, "reasons": ["sw_power_cap"], "samples": 3, "in_region": 3}
    # a region between two samples: the neighbours stand in, and the record says so
    short = bench.summarize_clock_samples(lines, base + 0.21, base + 0.29)
    assert short["in_region"] == 0 and short["samples"] == 2 and short["sm_mhz"] == 1920.0
    # no marks (the reference arm): every sample counts, the idle ones and the throttled one included
    whole = bench.summarize_clock_samples(lines)
    assert whole["samples"] == 5 and "hw_slowdown" in whole["reasons"] and "in_region" not in whole
    assert bench.summarize_clock_samples(["garbage", ""]) == {"sm_mhz": None, "sm_max_mhz": None, "reasons": []}


def test_clock_sampler_end_to_end_against_a_fake_nvidia_smi(tmp_path, monkeypatch):
    """The sampler process, its csv and the region marks, with a stand-in for nvidia-smi that prints one
    line every 25 ms in the queried format."""
    import importlib.util
    import os
    import stat
    import time

    fake = tmp_path / "nvidia-smi"
    fake.write_text("#!/usr/bin/env python3\n"
                    "import datetime, sys, time\n"
                    "assert '-i' in sys.argv and any(a.startswith('--query-gpu=timestamp,index,clocks.sm') for a in sys.argv)\n"
                    "while True:\n"
                    "    ts = datetime.datetime.now().strftime('%Y/%m/%d %H:%M:%S.%f')[:-3]\n"
                    "    print(f'{ts}, 0, 1965, 1965, 640.0, 0x0000000000000004, Not Active, Not Active, Not Active, Active', flush=True)\n"
                    "    time.sleep(0.025)\n")
    fake.chmod(fake.stat().st_mode | stat.S_IEXEC)
    monkeypatch.setenv("PATH", str(tmp_path) + os.pathsep + os.environ["PATH"])
    path = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "bench.py")
    spec = importlib.util.spec_from_file_location("bench_under_test3", path)
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    s = bench.ClockSampler(0)
    s.start()
    time.sleep(0.3)
    s.mark_start()
    time.sleep(0.2)
    s.mark_end()
    out = s.stop()
    assert out["sm_mhz"] == 1965.0 and out["sm_max_mhz"] == 1965.0 and out["reasons"] == ["sw_power_cap"]
    assert 3 <= out["in_region"] <= 12 and out["samples"] == out["in_region"]


def test_prompt_pools_are_pinned_by_sha256(tmp_path):
    """A pool is a function of its name and the registry's seed; the builder compares the file's sha256
    with the registered one (the recorded step times belong to exactly these prompts)."""
    import json

    from fastafd_b200.benchmark import long_prompts as lp

    reg = json.loads(lp.POOLS_FILE.read_text())
    assert len(reg["pools"]) >= 8 and all(len(p["sha256"]) == 64 for p in reg["pools"].values())
    res = lp.build_pool("qwen3-30b", 1024, 256, tmp_path)
    assert res["ok"] and res["sha256"] == reg["pools"]["qwen3-30b_isl1024_r256"]["sha256"]
    rows = lp.load(res["path"])
    assert len(rows) == 256 and all(len(r) == 1024 for r in rows)
    tampered = json.loads(json.dumps(reg))
    tampered["pools"]["qwen3-30b_isl1024_r256"]["sha256"] = "0" * 64
    assert not lp.build_pool("qwen3-30b", 1024, 256, tmp_path, tampered)["ok"]
    assert lp.pools_main(["--model", "qwen3-30b", "--out", str(tmp_path), "--pool", "1024:256"]) == 0
    assert lp.build_pool("qwen3-30b", 512, 4, tmp_path)["registered"] is None        # an unregistered pool is only built


def test_model_registry_and_draft_preparation(tmp_path):
    import json

    from fastafd_b200.benchmark import suite
    from fastafd_b200.config import get_model_config

    reg = json.loads((suite.HERE / "models.json").read_text())
    for key, m in reg["models"].items():
        get_model_config(m["preset"])
        assert suite.resolve_model(key, env={}) == m["preset"]
    (tmp_path / "Qwen3-30B-A3B").mkdir()
    assert suite.resolve_model("qwen3-30b", env={"FASTAFD_MODEL_ROOT": str(tmp_path)}) == str(tmp_path / "Qwen3-30B-A3B")
    assert suite.resolve_model("qwen3.5-397b", env={"FASTAFD_MODEL_QWEN3_5_397B": "/x/y"}) == "/x/y"
    src, dst = tmp_path / "draft", tmp_path / "draft-pos262k"
    src.mkdir()
    (src / "config.json").write_text(json.dumps({"max_position_embeddings": 40960, "hidden_size": 4096}))
    (src / "model.safetensors").write_bytes(b"weights")
    out = suite.prepare_draft("eagle3-qwen3-235b", src, dst)
    cfg = json.loads((dst / "config.json").read_text())
    assert cfg == {"max_position_embeddings": 262144, "hidden_size": 4096} and out["changed"] == {"max_position_embeddings": [40960, 262144]}
    assert (dst / "model.safetensors").read_bytes() == b"weights"
    assert json.loads((src / "config.json").read_text())["max_position_embeddings"] == 40960       # the source is untouched
