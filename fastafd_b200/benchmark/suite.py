"""Benchmark suite: named configurations, one run each, verdict against the recorded value.

    python -m fastafd_b200.benchmark.suite list
    python -m fastafd_b200.benchmark.suite command qwen3-235b-8k-1to1
    python -m fastafd_b200.benchmark.suite run qwen3-235b-8k-1to1 --out runs/
    python -m fastafd_b200.benchmark.suite summary runs/
    python -m fastafd_b200.benchmark.suite record qwen3-235b-8k-1to1 runs/qwen3-235b-8k-1to1-<UTC>

``run`` launches ``bench.py`` of the repository root (one process per GPU through
``torch.distributed.run``), stores ``result.json`` (measured step time, throughput, the verdict
against ``recorded`` and the ratio to the reference's published number) plus the raw output in a
directory named after the configuration and the UTC time.
Reference: scripts/benchmark/benchmark.py (list / run / summary over configs.json).
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import time
from pathlib import Path
from typing import Dict, List

from . import run_stats

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent


def load_configs(path: Path = HERE / "configs.json") -> Dict:
    return json.loads(path.read_text())


def validate(cfgs: Dict) -> List[str]:
    """Static checks of every configuration; returns a list of problems (empty = fine)."""
    from ..config import PRESETS

    bad = []
    for name, c in cfgs["configs"].items():
        for key in ("kind", "model", "context", "batch", "gpus", "attn_gpus", "num_mb"):
            if key not in c:
                bad.append(f"{name}: missing {key}")
        if c.get("model") not in PRESETS:
            bad.append(f"{name}: unknown model {c.get('model')}")
            continue
        m = PRESETS[c["model"]]
        gpus, ag = c.get("gpus", 0), c.get("attn_gpus", 0)
        tp = c.get("attn_tp", 1)
        if gpus == 1:
            if ag != 1:
                bad.append(f"{name}: a 1-GPU run is colocated (attn_gpus 1)")
        else:
            if not 0 < ag < gpus:
                bad.append(f"{name}: attn_gpus {ag} out of range for {gpus} GPUs")
            elif m.num_experts % (gpus - ag) != 0:
                bad.append(f"{name}: {m.num_experts} experts do not split over {gpus - ag} expert GPUs")
            if ag % tp != 0 or m.num_kv_heads % tp != 0:
                bad.append(f"{name}: attention TP {tp} does not divide {ag} GPUs / {m.num_kv_heads} KV heads")
        if not 1 <= c.get("num_mb", 0) <= 4:
            bad.append(f"{name}: num_mb must be 1..4")
        if c.get("kind") not in ("decode", "spec", "cad", "variant"):
            bad.append(f"{name}: unknown kind {c.get('kind')}")
    return bad


def command(name: str, c: Dict, steps: int, warmup: int, port: int = 29531) -> List[str]:
    args = ["bench.py", "--gpus", str(c["gpus"]), "--steps", str(steps), "--warmup", str(warmup), "--model", c["model"],
            "--batch-per-attn-gpu", str(c["batch"]), "--context", str(c["context"]), "--num-mb", str(c["num_mb"])]
    if c["gpus"] > 1:
        args += ["--attn-gpus", str(c["attn_gpus"]), "--attn-tp", str(c.get("attn_tp", 1))]
        return [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={c['gpus']}",
                "--master-addr", "127.0.0.1", "--master-port", str(port)] + args
    return [sys.executable] + args


def evaluate(c: Dict, bench_line: str, tolerance: float) -> Dict:
    st = run_stats.from_bench_json(bench_line)
    ag = c["attn_gpus"]
    eg = c["gpus"] - ag if c["gpus"] > 1 else 0
    per_gpu = run_stats.throughput_per_gpu(c["batch"], st["step_ms"], ag, eg)
    rec = (c.get("recorded") or {}).get("step_ms")
    v, dev = run_stats.verdict(st["step_ms"], rec, tolerance)
    pub = c.get("published") or {}
    return {"step_ms": st["step_ms"], "e2e_step_ms": st["e2e_step_ms"], "tok_s_per_gpu": round(per_gpu, 1),
            "recorded_step_ms": rec, "verdict": v, "deviation": dev,
            "published_tok_s_per_gpu": pub.get("tok_s_per_gpu"),
            "vs_published": (round(per_gpu / pub["tok_s_per_gpu"], 3) if pub.get("tok_s_per_gpu") else None)}


def run(name: str, out_root: Path, steps: int, warmup: int) -> Dict:
    cfgs = load_configs()
    c = cfgs["configs"][name]
    run_dir = out_root / f"{name}-{time.strftime('%Y%m%dT%H%M%SZ', time.gmtime())}"
    run_dir.mkdir(parents=True, exist_ok=True)
    cmd = command(name, c, steps, warmup)
    (run_dir / "config.json").write_text(json.dumps({"name": name, **c, "command": cmd}, indent=1))
    p = subprocess.run(cmd, cwd=REPO, capture_output=True, text=True, env=dict(os.environ))
    (run_dir / "stdout.log").write_text(p.stdout)
    (run_dir / "stderr.log").write_text(p.stderr)
    lines = [ln for ln in p.stdout.splitlines() if ln.startswith("{") and '"metric"' in ln]
    if p.returncode != 0 or not lines:
        res = {"verdict": "error", "returncode": p.returncode}
    else:
        res = evaluate(c, lines[-1], c.get("tolerance", cfgs.get("tolerance", 0.03)))
    (run_dir / "result.json").write_text(json.dumps(res, indent=1))
    return res


def resolve_model(key: str, env=None, path: Path = HERE / "models.json") -> str:
    """Where a benchmark model key comes from: FASTAFD_MODEL_<KEY>, else $FASTAFD_MODEL_ROOT/<dir> when it
    exists, else the preset name (random-init weights of the same architecture)."""
    env = os.environ if env is None else env
    m = json.loads(path.read_text())["models"][key]
    override = env.get("FASTAFD_MODEL_" + key.upper().replace("-", "_").replace(".", "_"))
    if override:
        return override
    root = env.get("FASTAFD_MODEL_ROOT")
    if root and (Path(root) / m["dir"]).is_dir():
        return str(Path(root) / m["dir"])
    return m["preset"]


def prepare_draft(name: str, src: Path, dst: Path, path: Path = HERE / "models.json") -> Dict:
    """Copy a downloaded draft-head directory to `dst` with the registry's changes to its config.json
    (the Qwen3 EAGLE-3 head needs max_position_embeddings raised for 32K contexts). Weights are linked, not
    copied, where the file system allows."""
    import shutil

    spec = json.loads(path.read_text())["drafts"][name]
    dst.mkdir(parents=True, exist_ok=True)
    for f in sorted(src.iterdir()):
        if f.name == "config.json" or not f.is_file():
            continue
        target = dst / f.name
        if target.exists():
            target.unlink()
        try:
            os.link(f, target)
        except OSError:
            shutil.copy2(f, target)
    cfg = json.loads((src / "config.json").read_text())
    changed = {}
    if "max_position_embeddings" in spec and cfg.get("max_position_embeddings") != spec["max_position_embeddings"]:
        changed["max_position_embeddings"] = [cfg.get("max_position_embeddings"), spec["max_position_embeddings"]]
        cfg["max_position_embeddings"] = spec["max_position_embeddings"]
    (dst / "config.json").write_text(json.dumps(cfg, indent=1))
    return {"draft": name, "dst": str(dst), "changed": changed}


def summary(root: Path) -> List[Dict]:
    rows = []
    for d in sorted(root.iterdir()):
        r, c = d / "result.json", d / "config.json"
        if r.exists() and c.exists():
            rows.append({"run": d.name, **json.loads(r.read_text())})
    return rows


def record(name: str, run_dir: Path, path: Path = HERE / "configs.json") -> Dict:
    """Make the result of a finished run the recorded value of its configuration."""
    res = json.loads((run_dir / "result.json").read_text())
    if "step_ms" not in res:
        raise ValueError(f"{run_dir} holds no measured step time (verdict {res.get('verdict')})")
    cfgs = json.loads(path.read_text())
    if name not in cfgs["configs"]:
        raise KeyError(name)
    cfgs["configs"][name]["recorded"] = {"step_ms": round(res["step_ms"], 3), "tok_s_per_gpu": round(res["tok_s_per_gpu"])}
    path.write_text(json.dumps(cfgs, indent=1))
    return cfgs["configs"][name]["recorded"]


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="fastafd_b200.benchmark.suite")
    sub = ap.add_subparsers(dest="cmd", required=True)
    sub.add_parser("list")
    for n in ("command", "run"):
        sp = sub.add_parser(n)
        sp.add_argument("name")
        sp.add_argument("--steps", type=int, default=64)
        sp.add_argument("--warmup", type=int, default=8)
        sp.add_argument("--out", default="benchmark-runs")
    sp = sub.add_parser("summary")
    sp.add_argument("root")
    sp = sub.add_parser("record")
    sp.add_argument("name")
    sp.add_argument("run_dir")
    sp = sub.add_parser("prepare-draft")
    sp.add_argument("name")
    sp.add_argument("src")
    sp.add_argument("dst")
    sp = sub.add_parser("resolve-model")
    sp.add_argument("key")
    a = ap.parse_args(argv)
    cfgs = load_configs()
    if a.cmd == "list":
        problems = validate(cfgs)
        for name, c in cfgs["configs"].items():
            ratio = "colocated" if c["gpus"] == 1 else f"{c['attn_gpus']}+{c['gpus'] - c['attn_gpus']}"
            print(f"{name:34s} {c['kind']:8s} {c['model']:24s} ctx {c['context']:6d} b {c['batch']:4d} {ratio:9s} mb {c['num_mb']}")
        for p in problems:
            print("PROBLEM:", p)
        return 1 if problems else 0
    if a.cmd == "command":
        print(" ".join(command(a.name, cfgs["configs"][a.name], a.steps, a.warmup)))
        return 0
    if a.cmd == "run":
        res = run(a.name, Path(a.out), a.steps, a.warmup)
        print(json.dumps(res))
        return 0 if res.get("verdict") in ("pass", "unrecorded") else 1
    if a.cmd == "record":
        print(json.dumps(record(a.name, Path(a.run_dir))))
        return 0
    if a.cmd == "prepare-draft":
        print(json.dumps(prepare_draft(a.name, Path(a.src), Path(a.dst))))
        return 0
    if a.cmd == "resolve-model":
        print(resolve_model(a.key))
        return 0
    for row in summary(Path(a.root)):
        print(json.dumps(row))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
