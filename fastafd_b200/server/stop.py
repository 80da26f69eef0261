"""End the processes of one server, and only those.

A supervisor started with ``--pid-file FILE`` records every process it spawns: pid, role and the start time
the kernel reports for that pid. ``python -m fastafd_b200.server.stop FILE`` sends SIGTERM (then SIGKILL after
``--grace`` seconds) to the recorded processes that are still the same processes: an entry whose pid is gone,
or whose pid now belongs to a process with another start time, is skipped. Nothing is looked up by name or
command line, so no other job on a shared machine can be hit.

Reference: scripts/kill_afd_ray_tasks.sh (ends leftover workers by command-line pattern on every node; its
header warns that it also ends other people's jobs on a shared cluster, which is what this form avoids).
"""
from __future__ import annotations

import argparse
import json
import os
import signal
import time
from typing import Dict, List, Optional, Sequence


def process_start_ticks(pid: int) -> Optional[int]:
    """Start time of `pid` in clock ticks since boot (field 22 of /proc/<pid>/stat), None if there is no such
    process. Together with the pid it names one process for the lifetime of the machine."""
    try:
        with open(f"/proc/{pid}/stat", "rb") as f:
            data = f.read().decode("ascii", "replace")
    except OSError:
        return None
    tail = data[data.rfind(")") + 2:].split()          # the command name may contain spaces and parentheses
    return int(tail[19]) if len(tail) > 19 else None


def record_process(path: str, pid: int, role: str) -> None:
    entries = load(path)
    entries.append({"pid": int(pid), "role": role, "start_ticks": process_start_ticks(pid), "recorded_by": os.getpid()})
    tmp = f"{path}.{os.getpid()}.tmp"
    os.makedirs(os.path.dirname(os.path.abspath(path)), exist_ok=True)
    with open(tmp, "w") as f:
        json.dump(entries, f)
    os.replace(tmp, path)


def load(path: str) -> List[Dict[str, object]]:
    try:
        with open(path) as f:
            return list(json.load(f))
    except (OSError, ValueError):
        return []


def same_process(entry: Dict[str, object]) -> bool:
    ticks = process_start_ticks(int(entry["pid"]))
    return ticks is not None and entry.get("start_ticks") is not None and ticks == int(entry["start_ticks"])


def stop_recorded(path: str, grace_s: float = 5.0) -> Dict[str, List[int]]:
    """Returns {"terminated": [...], "killed": [...], "skipped": [...]} (pids)."""
    out: Dict[str, List[int]] = {"terminated": [], "killed": [], "skipped": []}
    live = []
    entries = load(path)
    entries.sort(key=lambda e: e.get("role") == "server")      # the front end after the processes it started
    for e in entries:
        pid = int(e["pid"])
        if pid == os.getpid() or not same_process(e):
            out["skipped"].append(pid)
            continue
        try:
            os.kill(pid, signal.SIGTERM)
            live.append(e)
        except OSError:
            out["skipped"].append(pid)
    deadline = time.monotonic() + grace_s
    while live and time.monotonic() < deadline:
        live = [e for e in live if _still_there(e, out)]
        time.sleep(0.05)
    for e in live:
        if _still_there(e, out):
            try:
                os.kill(int(e["pid"]), signal.SIGKILL)
                out["killed"].append(int(e["pid"]))
            except OSError:
                out["terminated"].append(int(e["pid"]))
    return out


def _still_there(e: Dict[str, object], out: Dict[str, List[int]]) -> bool:
    pid = int(e["pid"])
    try:                                    # a child of this process stays a zombie until it is reaped
        if os.waitpid(pid, os.WNOHANG)[0] == pid:
            out["terminated"].append(pid)
            return False
    except ChildProcessError:
        pass
    if same_process(e) and _state(pid) != "Z":
        return True
    out["terminated"].append(pid)
    return False


def _state(pid: int) -> str:
    try:
        with open(f"/proc/{pid}/stat", "rb") as f:
            data = f.read().decode("ascii", "replace")
        return data[data.rfind(")") + 2:].split()[0]
    except OSError:
        return ""


def main(argv: Optional[Sequence[str]] = None) -> int:
    ap = argparse.ArgumentParser(prog="fastafd_b200.server.stop")
    ap.add_argument("pid_file")
    ap.add_argument("--grace", type=float, default=5.0, help="seconds between SIGTERM and SIGKILL")
    a = ap.parse_args(argv)
    res = stop_recorded(a.pid_file, a.grace)
    print(json.dumps(res))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
