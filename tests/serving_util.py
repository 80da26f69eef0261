"""Helpers shared by the serving tests: start a supervisor + HTTP frontend in this process
and talk to it."""
import contextlib
import json
import socket
import threading
import time


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@contextlib.contextmanager
def running_server(args):
    """Workers (processes) + tokenizer + coordinator of `args`, and the FastAPI app on a free
    port. Yields (base_url, supervisor)."""
    import requests
    import uvicorn

    from fastafd_b200.server.api_server import FrontendManager, create_app
    from fastafd_b200.server.supervisor import LocalSupervisor

    sup = LocalSupervisor(args)
    addrs = sup.start()
    port = free_port()
    server = None
    try:
        app = create_app(FrontendManager(addrs.to_tokenizer, addrs.from_tokenizer), args.model_path)
        server = uvicorn.Server(uvicorn.Config(app, host="127.0.0.1", port=port, log_level="warning"))
        threading.Thread(target=server.run, daemon=True).start()
        base = f"http://127.0.0.1:{port}"
        for _ in range(200):
            try:
                if requests.get(base + "/v1/models", timeout=1).ok:
                    break
            except Exception:
                time.sleep(0.1)
        yield base, sup
    finally:
        if server is not None:
            server.should_exit = True
        sup.shutdown()


def greedy_tokens(base, prompt_ids, max_tokens, timeout=300):
    """Token ids of one greedy, ignore-EOS completion (non-streaming)."""
    import requests

    r = requests.post(base + "/v1/chat/completions",
                      json={"input_ids": list(prompt_ids), "max_tokens": max_tokens, "temperature": 0, "ignore_eos": True,
                            "return_token_ids": True, "stream": False}, timeout=timeout)
    body = r.json()
    assert "choices" in body, json.dumps(body)[:500]
    return body["choices"][0]["token_ids"]
