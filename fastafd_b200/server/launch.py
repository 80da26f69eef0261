"""``launch_server``: parse flags, start the backend processes, then serve HTTP - or, when runtime
prompts were given (``--afd-prompt`` / ``--afd-prompt-file``), replay them once through the started
backend and write the sample bundle that the alignment scripts score, or (``--shell-mode``) run an
interactive shell on it.
Reference: python/minisgl/server/launch.py:6-23; the runtime replay flags of
python/minisgl/server/args.py (``--afd-prompt*``, ``--afd-report-dir``, ``--afd-sample-json``) and
scripts/validate/check_alignment_report.py (the bundle's ``samples[].generated_token_ids``)."""
from __future__ import annotations

import contextlib
import json
import os
import socket
import sys
import threading
import time
from typing import Iterator, List, Optional, Sequence, Tuple


def runtime_prompts(args) -> List[str]:
    """Prompts of a runtime replay: the ``--afd-prompt`` texts, then the lines of ``--afd-prompt-file``
    (empty lines skipped), the whole list repeated ``--afd-prompt-repeat`` times."""
    prompts = list(args.afd_prompt)
    if args.afd_prompt_file:
        with open(args.afd_prompt_file, encoding="utf-8") as f:
            prompts += [ln.rstrip("\n") for ln in f if ln.strip()]
    return prompts * max(args.afd_prompt_repeat, 1)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@contextlib.contextmanager
def local_endpoint(args, supervisor) -> Iterator[str]:
    """The backend of `supervisor` behind the HTTP app on a private port of this process; yields the
    base URL. The same FastAPI app as the server, so a replay takes the served path end to end."""
    import requests
    import uvicorn

    from .api_server import FrontendManager, create_app

    addrs = supervisor.start()
    server = None
    try:
        app = create_app(FrontendManager(addrs.to_tokenizer, addrs.from_tokenizer), args.model_path)
        port = _free_port()
        server = uvicorn.Server(uvicorn.Config(app, host="127.0.0.1", port=port, log_level="warning"))
        threading.Thread(target=server.run, daemon=True).start()
        base = f"http://127.0.0.1:{port}"
        for _ in range(600):
            try:
                if requests.get(base + "/v1/models", timeout=1).ok:
                    break
            except Exception:
                time.sleep(0.1)
        yield base
    finally:
        if server is not None:
            server.should_exit = True
        supervisor.shutdown()


def run_runtime_replay(args, supervisor) -> dict:
    """Send the runtime prompts as one batch request (greedy, `--afd-max-new-tokens` tokens each), write
    the sample bundle and a short report, return the bundle."""
    import requests

    prompts = runtime_prompts(args)
    if not prompts:
        raise ValueError("runtime replay without prompts")
    t0 = time.time()
    with local_endpoint(args, supervisor) as base:
        r = requests.post(base + "/v1/chat/completions/batch",
                          json={"prompts": prompts, "max_tokens": args.afd_max_new_tokens, "temperature": 0,
                                "return_token_ids": True}, timeout=3600)
        body = r.json()
        failures = supervisor.get_failures() if hasattr(supervisor, "get_failures") else []
    if "choices" not in body:
        raise RuntimeError(f"runtime replay failed: {json.dumps(body)[:500]}")
    samples = []
    for p, c in zip(prompts, sorted(body["choices"], key=lambda c: c["index"])):
        ids = [int(t) for t in c.get("token_ids") or []]
        samples.append({"prompt": p, "generated_token_ids": ids, "num_generated_tokens": len(ids),
                        "text": c.get("message", {}).get("content", "")})
    bundle = {"model": args.model_path, "mode": args.mode, "topology": str(args.topology) if args.mode == "afd-serve" else "colocated",
              "sampling": {"temperature": 0, "max_tokens": args.afd_max_new_tokens}, "samples": samples}
    report = {"prompts": len(prompts), "generated_tokens": sum(s["num_generated_tokens"] for s in samples),
              "elapsed_s": round(time.time() - t0, 3), "worker_failures": [str(f) for f in failures]}
    out = args.afd_sample_json or (os.path.join(args.afd_report_dir, "samples.json") if args.afd_report_dir else "")
    if out:
        os.makedirs(os.path.dirname(os.path.abspath(out)), exist_ok=True)
        with open(out, "w") as f:
            json.dump(bundle, f)
    if args.afd_report_dir:
        os.makedirs(args.afd_report_dir, exist_ok=True)
        with open(os.path.join(args.afd_report_dir, "runtime_report.json"), "w") as f:
            json.dump(report, f)
    print(json.dumps(report))
    return bundle


class _HttpLlm:
    """What `shell.run_shell` needs of an LLM (tokenizer, rt, generate), answered by a served backend."""

    def __init__(self, args, base: str):
        from ..tokenizer import load_tokenizer

        self.base, self.rt, self.tokenizer = base, args.runtime_config(), load_tokenizer(args.model_path)

    def generate(self, prompts: Sequence[Sequence[int]], sp) -> List[dict]:
        import requests

        out = []
        for ids in prompts:
            body = requests.post(self.base + "/v1/chat/completions",
                                 json={"input_ids": [int(t) for t in ids], "max_tokens": sp.max_tokens,
                                       "temperature": sp.temperature, "return_token_ids": True, "stream": False},
                                 timeout=3600).json()
            if "choices" not in body:
                raise RuntimeError(json.dumps(body)[:300])
            toks = body["choices"][0].get("token_ids") or []
            out.append({"token_ids": toks, "text": self.tokenizer.decode(toks)})
        return out


def launch_server(argv: Optional[Sequence[str]] = None) -> None:
    from .api_server import run_api_server
    from .args import parse_args
    from .supervisor import create_backend_supervisor

    args = parse_args(argv)
    supervisor = create_backend_supervisor(args)
    if args.afd_prompt or args.afd_prompt_file:
        run_runtime_replay(args, supervisor)
        return
    if args.shell_mode:
        from ..shell import run_shell

        with local_endpoint(args, supervisor) as base:
            run_shell(_HttpLlm(args, base), max_tokens=min(args.afd_max_new_tokens, 256), inp=sys.stdin, out=sys.stdout)
        return
    run_api_server(args, supervisor.start, stop_backend=supervisor.shutdown)
