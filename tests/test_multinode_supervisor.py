"""Multi-node launch planning on fake node reports: placement, forwarded environment, version
guard, and the refusal where Ray is missing."""
import pytest

from fastafd_b200.protocol import AfdTopology
from fastafd_b200.server import supervisor_ray as sr


def _nodes(*gpus, head=0):
    return [sr.NodeReport(address=f"10.0.0.{i + 1}", gpus=g, is_head=(i == head),
                          versions={"torch": "2.11", "cuda": "12.8", "package": "0.1.0"}) for i, g in enumerate(gpus)]


def test_placement_fills_head_first_and_keeps_tp_groups_on_one_node():
    topo = AfdTopology(attn_dp=2, attn_tp=2, mlp_ep=4)          # 4 attention + 4 expert ranks
    plan = sr.plan_placement(_nodes(4, 4, head=1), topo)
    assert [s.rank for s in plan] == list(range(8))
    assert [s.role for s in plan] == ["attention"] * 4 + ["expert"] * 4
    assert {s.node for s in plan[:4]} == {"10.0.0.2"}           # the head node is taken first
    assert {s.node for s in plan[4:]} == {"10.0.0.1"}
    assert sorted(s.gpu for s in plan[:4]) == [0, 1, 2, 3]
    # a TP group does not straddle nodes: 3 + 3 GPUs cannot hold two TP-2 lanes + 2 experts on the
    # first node, so the second lane moves to the next node as a whole
    plan = sr.plan_placement(_nodes(3, 3), AfdTopology(attn_dp=2, attn_tp=2, mlp_ep=2))
    lanes = [{s.node for s in plan if s.rank in (0, 1)}, {s.node for s in plan if s.rank in (2, 3)}]
    assert all(len(l) == 1 for l in lanes) and lanes[0] != lanes[1]
    assert len({(s.node, s.gpu) for s in plan}) == 6


def test_placement_refuses_what_does_not_fit():
    with pytest.raises(ValueError, match="need 8 GPUs"):
        sr.plan_placement(_nodes(4, 2), AfdTopology(attn_dp=4, attn_tp=1, mlp_ep=4))
    with pytest.raises(ValueError, match="tensor-parallel group"):
        sr.plan_placement(_nodes(2, 2, 2, 2, 2), AfdTopology(attn_dp=1, attn_tp=4, mlp_ep=4))


def test_actor_env_forwards_knobs_but_not_node_scoped_keys():
    env = {"FASTAFD_NUM_MB": "2", "MINISGL_AFD_MODE": "cad", "NCCL_DEBUG": "INFO", "CUDA_VISIBLE_DEVICES": "3",
           "TMPDIR": "/scratch", "HOME": "/root", "PYTHONPATH": "/x", "FASTAFD_LOG_DIR": "/logs", "MY_FLAG": "1"}
    out = sr.actor_env(env, extra_keys=("MY_FLAG",))
    assert out == {"FASTAFD_NUM_MB": "2", "MINISGL_AFD_MODE": "cad", "NCCL_DEBUG": "INFO", "PYTHONPATH": "/x", "MY_FLAG": "1"}


def test_version_guard_names_the_node_that_differs():
    nodes = _nodes(4, 4)
    assert sr.check_runtime_versions(nodes) == []
    odd = sr.NodeReport(address="10.0.0.9", gpus=4, versions={"torch": "2.10", "cuda": "12.8", "package": "0.1.0"})
    problems = sr.check_runtime_versions(nodes + [odd])
    assert len(problems) == 1 and "10.0.0.9" in problems[0] and "torch" in problems[0]


def test_ray_backend_is_refused_where_ray_is_missing():
    try:
        import ray  # noqa: F401
        pytest.skip("ray is installed here")
    except ImportError:
        pass
    from fastafd_b200.server.args import parse_args

    with pytest.raises(ValueError, match="ray"):                  # refused when the flags are parsed
        parse_args(["--mode", "afd-serve", "--model-path", "tiny-qwen3-moe", "--device", "cpu", "--launch-backend", "ray"])
    with pytest.raises(sr.RayUnavailable):                        # and by the supervisor itself
        sr.RaySupervisor(server_args=None)


def _sleep_forever(path):
    import os
    import time
    with open(path, "w") as f:
        f.write(str(os.getpid()))
    time.sleep(600)


def _parent_that_dies(path):
    """Starts a backend-style child through the supervisor's entry, then dies without any clean-up."""
    import multiprocessing as mp
    import os
    import time

    from fastafd_b200.server.supervisor import _child_entry
    p = mp.get_context("spawn").Process(target=_child_entry, args=(_sleep_forever, (path,)), daemon=False)
    p.start()
    for _ in range(200):
        if os.path.exists(path) and os.path.getsize(path) > 0:
            break
        time.sleep(0.05)
    os._exit(0)            # no atexit, no join: the child is orphaned


def test_backend_process_leaves_when_its_parent_is_gone(tmp_path):
    import multiprocessing as mp
    import os
    import time

    path = str(tmp_path / "child.pid")
    parent = mp.get_context("spawn").Process(target=_parent_that_dies, args=(path,))
    parent.start()
    parent.join(60)
    assert os.path.exists(path)
    pid = int(open(path).read())
    deadline = time.time() + 20
    alive = True
    while time.time() < deadline:
        try:
            os.kill(pid, 0)
        except ProcessLookupError:
            alive = False
            break
        time.sleep(0.2)
    if alive:
        os.kill(pid, 9)        # exact PID of the child this test started
    assert not alive, "the child outlived its parent"


def test_ray_flags_parse_and_the_nsys_preflight_refuses_a_node_without_nsys(monkeypatch):
    """The reference's `--ray-*` and `--control-host` flags are accepted; `--ray-nsys` is checked when the
    flags are parsed (backend and the nsys binary), not when a rank starts."""
    import shutil

    from fastafd_b200.server import args as sa

    p = sa.build_parser()
    a = p.parse_args(["--ray-address", "10.0.0.7:6379", "--ray-log-dir", "/var/log/afd", "--ray-nsys-output-prefix", "x",
                      "--ray-node-scoped-cache", "--control-host", "10.0.0.7"])
    assert (a.ray_address, a.ray_log_dir, a.ray_nsys_output_prefix, a.ray_node_scoped_cache, a.control_host, a.ray_nsys) == \
        ("10.0.0.7:6379", "/var/log/afd", "x", True, "10.0.0.7", False)
    with pytest.raises(ValueError, match="launch-backend ray"):
        sa.parse_args(["--mode", "afd-serve", "--model-path", "tiny-qwen3-moe", "--device", "cpu", "--ray-nsys"])
    monkeypatch.setattr(shutil, "which", lambda name: None)
    with pytest.raises(ValueError, match="nsys"):
        sa.parse_args(["--mode", "afd-serve", "--model-path", "tiny-qwen3-moe", "--device", "cpu", "--ray-nsys",
                       "--launch-backend", "ray"])


def test_actor_options_carry_logs_profile_and_cache_scope():
    slot = sr.Slot(3, "expert", "10.0.0.8", 1)
    env = {"FASTAFD_DIRECT": "1", "TVM_FFI_CACHE_DIR": "/driver/cache", "NCCL_DEBUG": "WARN"}
    plain = sr.actor_options(slot, env)
    assert plain["resources"] == {"node:10.0.0.8": 0.001} and plain["runtime_env"] == {"env_vars": env}
    full = sr.actor_options(slot, env, ray_log_dir="/logs", ray_nsys=True, node_scoped_cache=True)
    ev = full["runtime_env"]["env_vars"]
    assert "TVM_FFI_CACHE_DIR" not in ev and ev["FASTAFD_DIRECT"] == "1"           # the node builds its own cache
    assert ev["FASTAFD_RANK_LOG"] == "/logs/rank3.log" and ev["FASTAFD_LOG_DIR"] == "/logs"
    assert full["runtime_env"]["nsight"]["o"] == "/logs/nsys/fastafd-rank3"
    assert sr.actor_options(slot, env, ray_nsys=True, nsys_output_prefix="/p/run")["runtime_env"]["nsight"]["o"] == "/p/run-rank3"
    assert env == {"FASTAFD_DIRECT": "1", "TVM_FFI_CACHE_DIR": "/driver/cache", "NCCL_DEBUG": "WARN"}    # not modified


def test_stop_ends_exactly_the_recorded_processes(tmp_path):
    """The pid file names processes by pid and start time: the recorded sleeper is ended, an entry whose
    start time does not match (a pid that was reused) and an entry whose process is gone are skipped."""
    import subprocess
    import sys

    from fastafd_b200.server import stop

    path = str(tmp_path / "run" / "server.pids.json")
    sleeper = subprocess.Popen([sys.executable, "-c", "import time; time.sleep(600)"])
    bystander = subprocess.Popen([sys.executable, "-c", "import time; time.sleep(600)"])
    try:
        stop.record_process(path, sleeper.pid, "worker0")
        entries = stop.load(path)
        assert entries[0]["role"] == "worker0" and entries[0]["start_ticks"] == stop.process_start_ticks(sleeper.pid)
        # a reused pid: same number, another start time
        entries.append({"pid": bystander.pid, "role": "worker1", "start_ticks": stop.process_start_ticks(bystander.pid) + 1})
        entries.append({"pid": 2 ** 22 + 12345, "role": "gone", "start_ticks": 1})
        import json as _json
        open(path, "w").write(_json.dumps(entries))
        res = stop.stop_recorded(path, grace_s=5.0)
        assert res["terminated"] + res["killed"] == [sleeper.pid]
        assert sorted(res["skipped"]) == sorted([bystander.pid, 2 ** 22 + 12345])
        assert sleeper.wait(timeout=5) is not None and bystander.poll() is None
        assert stop.main([path, "--grace", "0.5"]) == 0          # a second run finds nothing left to end
    finally:
        for p in (sleeper, bystander):
            if p.poll() is None:
                p.kill()
            p.wait()


def test_supervisor_records_its_processes_when_asked(tmp_path, monkeypatch):
    from fastafd_b200.server import stop
    from fastafd_b200.server.args import parse_args
    from fastafd_b200.server.supervisor import LocalSupervisor

    path = str(tmp_path / "pids.json")
    args = parse_args(["--mode", "serve", "--model-path", "tiny-qwen3-moe", "--device", "cpu", "--pid-file", path])
    sup = LocalSupervisor(args)

    sup._spawn("worker0", __import__("time").sleep, (60,))
    try:
        e = stop.load(path)
        assert [x["role"] for x in e] == ["server", "worker0"] and all(stop.same_process(x) for x in e)
        assert e[0]["pid"] == __import__("os").getpid()            # the front end is on record too (and `stop` never signals itself)
    finally:
        for p in sup.procs:
            p.terminate()
            p.join(5)


def test_the_distributed_timeout_reaches_the_workers_process_group():
    import ast
    import datetime
    import inspect

    from fastafd_b200.server.args import parse_args
    from fastafd_b200.worker import main as wm

    base = ["--mode", "afd-serve", "--model-path", "tiny-qwen3-moe", "--device", "cpu"]
    assert wm.host_group_options(parse_args(base)) == {}
    assert wm.host_group_options(parse_args(base + ["--distributed-timeout", "90"])) == {"timeout": datetime.timedelta(seconds=90)}
    tree = ast.parse(inspect.getsource(wm.worker_main))
    calls = [n for n in ast.walk(tree) if isinstance(n, ast.Call) and getattr(n.func, "attr", "") == "init_process_group"]
    assert len(calls) == 1 and any(k.arg is None and getattr(k.value.func, "id", "") == "host_group_options" for k in calls[0].keywords)
