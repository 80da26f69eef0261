"""The serving shell on CPU: flag parsing, message codec, tokenizer worker logic, the offline
LLM API, and a full HTTP round trip against a 1+1 CPU/gloo deployment (processes, ZeroMQ)."""
import json
import socket
import threading
import time

import pytest

from fastafd_b200.core import SamplingParams
from fastafd_b200.message import DetokenizeMsg, TokenizeMsg, UserMsg, deserialize, serialize
from fastafd_b200.server.args import parse_args
from fastafd_b200.server.prompt_ids import validate_prompt_ids
from fastafd_b200.tokenizer import ByteTokenizer, DetokenizeManager


def test_parse_args_and_validation():
    a = parse_args(["--mode", "afd-serve", "--model-path", "tiny-qwen3-moe", "--afd-attn-dp-size", "2",
                    "--afd-mlp-ep-size", "2", "--afd-num-mb", "2", "--afd-decode-graph-bs", "4,8", "--device", "cpu"])
    assert a.topology.world == 4 and a.afd_decode_graph_bs == (4, 8)
    rt = a.runtime_config()
    assert rt.num_mb == 2 and rt.dtype == "float32" and not rt.use_cuda_graph
    with pytest.raises(ValueError):
        parse_args(["--afd-num-mb", "9"])
    with pytest.raises(ValueError):
        parse_args(["--afd-attn-tp-size", "3"])          # 4 query heads
    with pytest.raises(ValueError):
        parse_args(["--launch-backend", "ray"])          # ray is not installed here
    with pytest.raises(ValueError):
        parse_args(["--spec-block", "4", "--cache-type", "radix"])


def test_message_codec_roundtrip():
    m = TokenizeMsg(uid=3, input_ids=[1, 2], sampling=SamplingParams(temperature=0.5, max_tokens=7, stop_token_ids=(9,)))
    r = deserialize(serialize(m))
    assert r == m and isinstance(r.sampling, SamplingParams) and r.sampling.stop_token_ids == (9,)
    assert deserialize(serialize(UserMsg(uid=1, input_ids=[5], sampling=SamplingParams()))).input_ids == [5]


def test_prompt_ids_validation():
    assert validate_prompt_ids([1, 2, 3], 10, 8) == [1, 2, 3]
    for bad in ([], [1, 10], [-1], [1.5], [True], list(range(8))):
        with pytest.raises(ValueError):
            validate_prompt_ids(bad, 10, 8)


def test_incremental_detokenize_holds_back_partial_characters():
    tok = ByteTokenizer()
    d = DetokenizeManager(tok)
    ids = tok.encode("hé!")                      # é is two bytes
    pieces = [d.step(DetokenizeMsg(uid=0, token_ids=[i], finished=(k == len(ids) - 1))).text for k, i in enumerate(ids)]
    assert "".join(pieces) == "hé!" and pieces[1] == ""      # first byte of é alone prints nothing
    assert 0 not in d.state


def test_offline_llm_api_cpu():
    from fastafd_b200.llm import LLM

    llm = LLM("tiny-qwen3-moe", device="cpu", num_pages=64, max_seq_len=128, max_running_requests=8, cuda_graph_max_bs=8)
    out = llm.generate([[1, 2, 3, 4], "hi"], SamplingParams(max_tokens=3, ignore_eos=True))
    assert len(out) == 2 and all(len(o["token_ids"]) == 3 for o in out)
    again = llm.generate([[1, 2, 3, 4]], SamplingParams(max_tokens=3, ignore_eos=True))
    assert again[0]["token_ids"] == out[0]["token_ids"]      # deterministic, state cleaned up between calls
    llm.shutdown()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.timeout(300)
@pytest.mark.parametrize("mode,cache", [("afd-serve", "naive"), ("serve", "radix")],
                         ids=["afd-two-roles", "colocated-serve-radix"])
def test_http_round_trip_cpu_afd(mode, cache):
    """HTTP -> tokenizer -> coordinator -> workers and back, in AFD mode (attention and expert
    processes) and in the colocated `serve` mode with the radix prefix cache."""
    import requests
    import uvicorn

    from fastafd_b200.server.api_server import FrontendManager, create_app
    from fastafd_b200.server.supervisor import LocalSupervisor

    args = parse_args(["--mode", mode, "--model-path", "tiny-qwen3-moe", "--device", "cpu", "--afd-num-mb", "2",
                       "--num-pages", "64", "--max-seq-len-override", "128", "--afd-max-running-requests", "8",
                       "--cuda-graph-max-bs", "8", "--cache-type", cache])
    sup = LocalSupervisor(args)
    addrs = sup.start()
    port = _free_port()
    server = None
    try:
        manager = FrontendManager(addrs.to_tokenizer, addrs.from_tokenizer)
        app = create_app(manager, args.model_path)
        server = uvicorn.Server(uvicorn.Config(app, host="127.0.0.1", port=port, log_level="warning"))
        th = threading.Thread(target=server.run, daemon=True)
        th.start()
        for _ in range(100):
            try:
                if requests.get(f"http://127.0.0.1:{port}/v1/models", timeout=1).ok:
                    break
            except Exception:
                time.sleep(0.1)
        base = f"http://127.0.0.1:{port}"
        assert requests.get(base + "/v1/models").json()["data"][0]["id"] == "tiny-qwen3-moe"
        r = requests.post(base + "/v1/chat/completions", json={"input_ids": [1, 2, 3, 4, 5], "max_tokens": 4,
                                                               "temperature": 0, "ignore_eos": True,
                                                               "return_token_ids": True}, stream=True, timeout=120)
        toks, done = [], False
        for line in r.iter_lines():
            if not line:
                continue
            payload = line.decode()[len("data: "):]
            if payload == "[DONE]":
                done = True
                break
            toks += json.loads(payload)["choices"][0].get("token_ids") or []
        assert done and len(toks) == 4
        rb = requests.post(base + "/v1/chat/completions/batch", json={"prompts": ["ab", "cde"], "max_tokens": 3,
                                                                      "temperature": 0, "ignore_eos": True,
                                                                      "return_token_ids": True}, timeout=120).json()
        assert [len(c["token_ids"]) for c in rb["choices"]] == [3, 3]
        whole = requests.post(base + "/v1/chat/completions", json={"input_ids": [1, 2, 3, 4, 5], "max_tokens": 4, "temperature": 0,
                                                                   "ignore_eos": True, "return_token_ids": True,
                                                                   "stream": False}, timeout=120).json()
        assert whole["object"] == "chat.completion" and whole["choices"][0]["token_ids"] == toks      # same greedy tokens
        assert whole["usage"]["completion_tokens"] == 4 and whole["choices"][0]["finish_reason"] == "stop"
        assert requests.get(base + "/health").json() == {"status": "ok"}
        legacy = requests.post(base + "/v1/completions", json={"prompt": "ab", "max_tokens": 3, "temperature": 0, "ignore_eos": True,
                                                               "return_token_ids": True, "stream": False}, timeout=120).json()
        assert len(legacy["choices"][0]["token_ids"]) == 3
        bad = requests.post(base + "/v1/chat/completions", json={"input_ids": [99999], "max_tokens": 2}, stream=True, timeout=60)
        assert "outside the vocabulary" in bad.text
        assert sup.get_failures() == []
    finally:
        if server is not None:
            server.should_exit = True
        sup.shutdown()
        sup.shutdown()          # idempotent


def test_step_profiler_window_and_client_summary():
    from fastafd_b200.benchmark.client import RequestTrace, summarize
    from fastafd_b200.worker.profiler import StepProfiler

    class Fake:
        calls = []
        def start(self): self.calls.append("start")
        def stop(self): self.calls.append("stop")
    f = Fake()
    p = StepProfiler(start_step=3, stop_step=5, backend=f)
    for s in range(8):
        p.on_step(s)
    assert f.calls == ["start", "stop"]
    p2 = StepProfiler(start_step=-1, backend=f)
    p2.on_step(0)
    assert f.calls == ["start", "stop"]
    tr = RequestTrace(start=0.0, ticks=[0.5, 0.6, 0.7], tokens=3)
    assert abs(tr.ttft - 0.5) < 1e-9 and abs(tr.tpot - 0.1) < 1e-9
    s = summarize([tr, RequestTrace(start=0.0, error="x")], 1.0)
    assert s["failed"] == 1 and s["output_tokens"] == 3 and s["tpot_ms_p50"] == 100.0


def test_interactive_shell_keeps_context_and_resets():
    import io

    from fastafd_b200.llm import LLM
    from fastafd_b200.shell import run_shell

    llm = LLM("tiny-qwen3-moe", device="cpu", max_seq_len=128, num_pages=64, max_running_requests=4, cuda_graph_max_bs=4)
    out = io.StringIO()
    turns = run_shell(llm, max_tokens=4, inp=io.StringIO("hello there\n\nagain\n/reset\nthird\n/exit\nnot read\n"), out=out)
    assert turns == 3
    assert "(conversation cleared)" in out.getvalue()
    assert out.getvalue().count(">>> ") == 6


def test_load_client_against_cpu_server_closed_batch_and_trace_replay():
    """The benchmark client (closed batch and open-loop trace replay) against a colocated CPU
    server: every request streams its tokens, TTFT / TPOT come out finite."""
    import asyncio

    import requests
    import uvicorn

    from fastafd_b200.benchmark import client
    from fastafd_b200.server.api_server import FrontendManager, create_app
    from fastafd_b200.server.supervisor import LocalSupervisor

    args = parse_args(["--mode", "serve", "--model-path", "tiny-qwen3-moe", "--device", "cpu", "--num-pages", "64",
                       "--max-seq-len-override", "128", "--afd-max-running-requests", "8", "--cuda-graph-max-bs", "8"])
    sup = LocalSupervisor(args)
    addrs = sup.start()
    port = _free_port()
    server = None
    try:
        app = create_app(FrontendManager(addrs.to_tokenizer, addrs.from_tokenizer), args.model_path)
        server = uvicorn.Server(uvicorn.Config(app, host="127.0.0.1", port=port, log_level="warning"))
        threading.Thread(target=server.run, daemon=True).start()
        for _ in range(100):
            try:
                if requests.get(f"http://127.0.0.1:{port}/v1/models", timeout=1).ok:
                    break
            except Exception:
                time.sleep(0.1)
        res = asyncio.run(client.run("127.0.0.1", port, num=3, prompt_len=12, max_tokens=4, vocab=1024))
        assert res["requests"] == 3 and res["failed"] == 0 and res["output_tokens"] == 12
        assert res["ttft_ms_p50"] > 0 and res["tpot_ms_p50"] > 0
        entries = [client.TraceEntry(0.0, 8, 3), client.TraceEntry(0.2, 10, 2)]
        rep = asyncio.run(client.replay("127.0.0.1", port, entries, vocab=1024))
        assert rep["requests"] == 2 and rep["failed"] == 0 and rep["output_tokens"] == 5
    finally:
        if server is not None:
            server.should_exit = True
        sup.shutdown()


def test_cpu_trace_mirrors_ranges_and_parses_step_ids(tmp_path):
    import json as _json

    from fastafd_b200.utils import trace

    trace.CPU_TRACE.clear()
    old = trace.CPU_TRACE.enabled
    trace.CPU_TRACE.enabled = True
    try:
        class Worker:
            @trace.nvtx_annotate("AFD_AG_Attn_L{}_mb{}")
            def attn(self, layer, mb):
                return layer * 10 + mb

        with trace.nvtx_range("decode step=17"):
            assert Worker().attn(3, 1) == 31
        names = [e["name"] for e in trace.CPU_TRACE.events]
        assert names == ["AFD_AG_Attn_L3_mb1", "decode step=17"]        # inner range closes first
        assert trace.CPU_TRACE.events[1]["step"] == 17 and trace.CPU_TRACE.events[0]["step"] is None
        assert all(e["dur_us"] >= 0 for e in trace.CPU_TRACE.events)
        path = trace.CPU_TRACE.dump(str(tmp_path / "run"))
        assert len(_json.load(open(path))["traceEvents"]) == 2
    finally:
        trace.CPU_TRACE.enabled = old
        trace.CPU_TRACE.clear()
    with trace.nvtx_range("off"):                                        # disabled: no event, no error
        pass
    assert trace.CPU_TRACE.events == []


def test_env_knobs_answer_to_all_prefixes_and_reject_bad_values(monkeypatch):
    from fastafd_b200.env import ENV, afd_env

    for n in ENV.FLAG_TIMEOUT_S.names():
        monkeypatch.delenv(n, raising=False)
    assert ENV.FLAG_TIMEOUT_S.value == 20.0
    monkeypatch.setenv("MINISGL_FLAG_TIMEOUT_S", "3")           # least specific name
    assert ENV.FLAG_TIMEOUT_S.value == 3.0
    monkeypatch.setenv("MINISGL_AFD_FLAG_TIMEOUT_S", "5")       # the reference's AFD prefix wins over it
    assert ENV.FLAG_TIMEOUT_S.value == 5.0
    monkeypatch.setenv("FASTAFD_FLAG_TIMEOUT_S", "7.5")         # this framework's own name wins over both
    assert ENV.FLAG_TIMEOUT_S.value == 7.5
    monkeypatch.setenv("FASTAFD_FLAG_TIMEOUT_S", "soon")
    with pytest.raises(ValueError, match="FASTAFD_FLAG_TIMEOUT_S"):
        ENV.FLAG_TIMEOUT_S.value
    monkeypatch.setenv("MINISGL_AFD_MODE", "cad")
    monkeypatch.delenv("FASTAFD_MODE", raising=False)
    assert afd_env("MODE") == "cad" and afd_env("NO_SUCH_KNOB", "x") == "x"


def test_buffered_log_file_flushes_by_count_and_on_demand(tmp_path):
    from fastafd_b200.utils.logger import BufferedLogFile

    path = tmp_path / "logs" / "w.log"
    log = BufferedLogFile(str(path), interval_s=3600.0, max_lines=3)
    log.line("a")
    log.line("b")
    assert not path.exists() or path.read_text() == ""          # still buffered
    log.line("c")                                               # third line reaches max_lines
    assert [ln.split(" ", 1)[1] for ln in path.read_text().splitlines()] == ["a", "b", "c"]
    log.line("d")
    log.flush()
    assert path.read_text().splitlines()[-1].endswith(" d")


@pytest.mark.timeout(300)
def test_runtime_replay_writes_the_sample_bundle(tmp_path):
    """`--afd-prompt` / `--afd-prompt-file`: the prompts run once through the started backend (attention
    and expert processes, the HTTP app on a private port) and the continuations land in the sample
    bundle; the same prompt gives the same tokens, a repeat factor repeats the list."""
    from fastafd_b200.server.launch import run_runtime_replay, runtime_prompts
    from fastafd_b200.server.supervisor import create_backend_supervisor

    pf = tmp_path / "prompts.txt"
    pf.write_text("ab\n\ncde\n", encoding="utf-8")
    out = tmp_path / "report" / "bundle.json"
    args = parse_args(["--mode", "afd-serve", "--model-path", "tiny-qwen3-moe", "--device", "cpu", "--afd-num-mb", "2",
                       "--num-pages", "64", "--max-seq-len-override", "128", "--max-running-requests", "8", "--graph", "8",
                       "--afd-prompt", "hello", "--afd-prompt-file", str(pf), "--afd-prompt-repeat", "2",
                       "--afd-max-new-tokens", "5", "--afd-sample-json", str(out), "--afd-report-dir", str(tmp_path / "report")])
    assert runtime_prompts(args) == ["hello", "ab", "cde"] * 2
    bundle = run_runtime_replay(args, create_backend_supervisor(args))
    on_disk = json.loads(out.read_text())
    assert on_disk == bundle and bundle["model"] == "tiny-qwen3-moe" and len(bundle["samples"]) == 6
    for s in bundle["samples"]:
        assert s["num_generated_tokens"] == len(s["generated_token_ids"]) and 1 <= s["num_generated_tokens"] <= 5
    first, second = bundle["samples"][:3], bundle["samples"][3:]
    assert [s["prompt"] for s in first] == ["hello", "ab", "cde"]
    assert [s["generated_token_ids"] for s in first] == [s["generated_token_ids"] for s in second]     # greedy
    report = json.loads((tmp_path / "report" / "runtime_report.json").read_text())
    assert report["prompts"] == 6 and report["worker_failures"] == []


@pytest.mark.timeout(300)
def test_shell_mode_talks_to_the_started_backend():
    import io

    from fastafd_b200.server.launch import _HttpLlm, local_endpoint
    from fastafd_b200.server.supervisor import create_backend_supervisor
    from fastafd_b200.shell import run_shell

    args = parse_args(["--mode", "serve", "--model-path", "tiny-qwen3-moe", "--device", "cpu", "--num-pages", "64",
                       "--max-seq-len-override", "128", "--max-running-requests", "4", "--graph", "4", "--shell-mode"])
    assert args.shell_mode
    out = io.StringIO()
    with local_endpoint(args, create_backend_supervisor(args)) as base:
        turns = run_shell(_HttpLlm(args, base), max_tokens=4, inp=io.StringIO("hi\n/reset\nagain\n/exit\n"), out=out)
    assert turns == 2 and "(conversation cleared)" in out.getvalue()


def test_serve_script_takes_the_reference_scripts_options(tmp_path):
    """`fastafd_server.sh --model PATH --port P <CLI flags> --extra-args "..."`: the printed command parses,
    and a flag given by the caller replaces the script's default (argparse keeps the last occurrence)."""
    import os
    import shlex
    import subprocess

    script = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "fastafd_b200", "server", "fastafd_server.sh")
    out = subprocess.run(["bash", script, "--model", "tiny-qwen3-moe", "--port", "19193", "--afd-attn-tp-size", "2",
                          "--afd-attn-dp-size", "1", "--afd-mlp-ep-size", "2", "--launch-backend", "mp", "--extra-args",
                          "--afd-max-new-tokens 1 --device cpu"], env=dict(os.environ, DRY_RUN="1"),
                         capture_output=True, text=True, timeout=60)
    assert out.returncode == 0, out.stderr
    words = shlex.split(out.stdout.strip())
    assert words[:3] == ["python", "-m", "fastafd_b200"]
    a = parse_args(words[3:])
    assert (a.model_path, a.port, a.afd_attn_tp_size, a.afd_attn_dp_size, a.afd_mlp_ep_size, a.afd_max_new_tokens) == \
        ("tiny-qwen3-moe", 19193, 2, 1, 2, 1)
    bad = subprocess.run(["bash", script, "--env", "not-this-env", "--model", "x"],
                         env={k: v for k, v in os.environ.items() if k != "CONDA_DEFAULT_ENV"}, capture_output=True, text=True)
    assert bad.returncode == 2 and "not-this-env" in bad.stderr


def test_offline_api_takes_the_reference_keywords_and_per_prompt_sampling():
    """`LLM(path, dtype, use_dummy_weight=..., max_running_req=..., max_seq_len_override=..., ...)` and
    `generate(prompts, [params per prompt])`, as a program written for the reference calls them."""
    import torch

    from fastafd_b200.llm import LLM, translate_kwargs

    assert translate_kwargs({"use_dummy_weight": True, "max_running_req": 8, "max_seq_len_override": None,
                             "cuda_graph_bs": [2, 4], "attention_backend": "auto", "page_size": 16}) == \
        {"dummy_weights": True, "max_running_requests": 8, "decode_graph_bs": (2, 4), "page_size": 16}
    llm = LLM("tiny-qwen3-moe", torch.float32, device="cpu", use_dummy_weight=True, max_running_req=4, cuda_graph_max_bs=4,
              max_seq_len_override=128, num_page_override=64, max_extend_tokens=256, memory_ratio=0.9, cache_type="naive")
    try:
        assert (llm.rt.max_running_requests, llm.rt.max_seq_len, llm.rt.num_pages, llm.rt.max_batched_tokens, llm.rt.dtype) == \
            (4, 128, 64, 256, "float32")
        out = llm.generate([[5, 6, 7, 8], "ab"], [SamplingParams(max_tokens=3, ignore_eos=True),
                                                  SamplingParams(max_tokens=5, ignore_eos=True)])
        assert [len(o["token_ids"]) for o in out] == [3, 5] and all(isinstance(o["text"], str) for o in out)
        with pytest.raises(ValueError):
            llm.generate([[1, 2]], [SamplingParams(), SamplingParams()])
    finally:
        llm.shutdown()


def test_hugging_face_tokenizer_directory_chat_template_and_incremental_detokenise(tmp_path):
    """A tokenizer directory as `transformers` saves it (byte-level BPE, a chat template): requests with
    `messages` go through the template, and text streamed token by token equals the text decoded at once, also
    where one character spans several tokens."""
    tokenizers = pytest.importorskip("tokenizers")
    from tokenizers import Tokenizer, decoders, models, pre_tokenizers, trainers
    from transformers import PreTrainedTokenizerFast

    from fastafd_b200.message import DetokenizeMsg, TokenizeMsg
    from fastafd_b200.tokenizer import DetokenizeManager, load_tokenizer, tokenize_request

    tk = Tokenizer(models.BPE(unk_token=None))
    tk.pre_tokenizer = pre_tokenizers.ByteLevel(add_prefix_space=False)
    tk.decoder = decoders.ByteLevel()
    trainer = trainers.BpeTrainer(vocab_size=300, special_tokens=["<|im_start|>", "<|im_end|>"],
                                  initial_alphabet=pre_tokenizers.ByteLevel.alphabet())
    tk.train_from_iterator(["hello world, how are you today?", "the quick brown fox jumps over the lazy dog"] * 20, trainer)
    template = ("{% for m in messages %}<|im_start|>{{ m['role'] }}\n{{ m['content'] }}<|im_end|>\n{% endfor %}"
                "{% if add_generation_prompt %}<|im_start|>assistant\n{% endif %}")
    PreTrainedTokenizerFast(tokenizer_object=tk, eos_token="<|im_end|>", chat_template=template).save_pretrained(str(tmp_path))
    tok = load_tokenizer(str(tmp_path))
    assert type(tok).__name__ != "ByteTokenizer"
    ids = tokenize_request(tok, TokenizeMsg(uid=1, messages=[{"role": "user", "content": "hello world"}]), 300, 256)
    text = tok.decode(ids)
    assert text == "<|im_start|>user\nhello world<|im_end|>\n<|im_start|>assistant\n"
    assert ids[0] == tok.convert_tokens_to_ids("<|im_start|>") and ids.count(ids[0]) == 2      # special tokens are single ids
    plain = tokenize_request(tok, TokenizeMsg(uid=2, text="the lazy dog"), 300, 256)
    assert tok.decode(plain) == "the lazy dog"
    # streaming: characters outside the training text fall back to bytes, several tokens per character
    sample = "hello wörld ✓ 你好, the fox"
    out_ids = tok.encode(sample)
    assert len(out_ids) > len(sample.split())
    dm = DetokenizeManager(tok)
    streamed = "".join(dm.step(DetokenizeMsg(uid=7, token_ids=[t], finished=(i == len(out_ids) - 1))).text
                       for i, t in enumerate(out_ids))
    assert streamed == sample and "�" not in streamed


def test_stop_strings_cut_the_output_and_hold_back_partial_matches():
    from fastafd_b200.server.api_server import StopFilter

    f = StopFilter(["</s>", "\n\n"])
    out = []
    for piece in ["Hello", " wor", "ld<", "/", "s", ">ignored"]:
        text, hit = f.feed(piece, False)
        out.append(text)
        if hit:
            break
    assert "".join(out) == "Hello world" and hit                 # the stop string itself is not part of the output
    assert all("<" not in t for t in out)                        # a possible beginning of a stop string is held back
    g = StopFilter(["END"])
    assert g.feed("abcE", False) == ("ab", False)                 # two characters held: they could start "END"
    assert g.feed("Nx", False) == ("cE", False)
    assert g.feed("y", True) == ("Nxy", False)                    # final piece: everything held is released
    h = StopFilter(["a", "abc"])
    assert h.feed("xxabc", False) == ("xx", True)                 # the earliest match wins


def test_stop_strings_end_the_stream_and_abort_the_backend_request():
    """The frontend's reply stream with a stop list: pieces are passed on up to the stop string, the reply that
    reaches it is marked finished, an abort goes to the backend, and nothing later is delivered."""
    import asyncio

    from fastafd_b200.message import AbortMsg, UserReply
    from fastafd_b200.server.api_server import FrontendManager, StopFilter

    class Push:
        def __init__(self):
            self.sent = []

        async def put(self, m):
            self.sent.append(m)

    async def run():
        man = FrontendManager.__new__(FrontendManager)
        man.queues, man.stops, man.push = {5: asyncio.Queue()}, {5: StopFilter(["STOP"])}, Push()
        for i, piece in enumerate(["one ", "two S", "TO", "P three", " four"]):
            man.queues[5].put_nowait(UserReply(uid=5, text=piece, token_ids=[i], finished=False))
        got = [m async for m in man.stream(5)]
        return man, got

    man, got = asyncio.run(run())
    assert "".join(m.text for m in got) == "one two " and got[-1].finished and not any(m.finished for m in got[:-1])
    assert [type(m) for m in man.push.sent] == [AbortMsg] and man.push.sent[0].uid == 5
    assert 5 not in man.queues and 5 not in man.stops
