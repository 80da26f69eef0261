"""HTTP frontend: FastAPI + uvicorn, OpenAI-style endpoints with server-sent events.

    POST /generate                     {prompt, max_tokens, ignore_eos}             -> SSE text pieces
    POST /v1/chat/completions          prompt | messages | input_ids (+ sampling)   -> SSE chunks
    POST /v1/chat/completions/batch    prompts[] | messages_batch[][]               -> one JSON
    GET  /v1/models ; GET/POST/HEAD/OPTIONS /v1

``input_ids`` is an extension: the ids are used verbatim after validation against the
vocabulary and the maximum sequence length. A client that disconnects aborts its request.

Reference: python/minisgl/server/api_server.py (FrontendManager :123-263, endpoints
:282-419, run_api_server :525-580).
"""
from __future__ import annotations

import asyncio
import json
import time
from typing import Any, AsyncIterator, Callable, Dict, List, Optional

from fastapi import FastAPI, Request
from fastapi.responses import JSONResponse, StreamingResponse
from pydantic import BaseModel

from ..core import SamplingParams
from ..message import AbortMsg, TokenizeMsg, UserReply
from ..utils.logger import init_logger

logger = init_logger("api")


class GenerateRequest(BaseModel):
    prompt: str
    max_tokens: int = 16
    ignore_eos: bool = False


class Message(BaseModel):
    role: str
    content: str


class CompletionRequest(BaseModel):
    model: str = ""
    prompt: Optional[str] = None
    messages: Optional[List[Message]] = None
    input_ids: Optional[List[int]] = None
    max_tokens: int = 16
    temperature: float = 1.0
    top_k: int = -1
    top_p: float = 1.0
    n: int = 1
    stream: bool = True
    return_token_ids: bool = False
    stop: Optional[Any] = None
    presence_penalty: float = 0.0
    frequency_penalty: float = 0.0
    ignore_eos: bool = False


class BatchCompletionRequest(BaseModel):
    model: str = ""
    prompts: Optional[List[str]] = None
    messages_batch: Optional[List[List[Message]]] = None
    max_tokens: int = 16
    temperature: float = 1.0
    top_k: int = -1
    top_p: float = 1.0
    return_token_ids: bool = False
    ignore_eos: bool = False


def _sampling(req) -> SamplingParams:
    return SamplingParams(temperature=getattr(req, "temperature", 0.0), top_k=getattr(req, "top_k", -1),
                          top_p=getattr(req, "top_p", 1.0), ignore_eos=req.ignore_eos, max_tokens=req.max_tokens)


class StopFilter:
    """Stop strings of a request (`stop` of the OpenAI request body): text is passed on up to the first stop string,
    which is not part of the output; the last characters are held back while they could still be the beginning of
    a stop string that continues in the next piece."""

    def __init__(self, stops: List[str]):
        self.stops = [s for s in stops if s]
        self.hold = max(len(s) for s in self.stops) - 1
        self.buf = ""

    def feed(self, text: str, final: bool):
        """-> (text to emit now, whether a stop string was reached)."""
        self.buf += text
        cut = min((i for i in (self.buf.find(s) for s in self.stops) if i >= 0), default=-1)
        if cut >= 0:
            out, self.buf = self.buf[:cut], ""
            return out, True
        keep = 0 if final else min(self.hold, len(self.buf))
        out, self.buf = self.buf[:len(self.buf) - keep], self.buf[len(self.buf) - keep:]
        return out, False


class FrontendManager:
    """uid allocation, per-request reply queues, and the reader task that routes
    ``UserReply`` messages from the detokenizer to the waiting HTTP handlers."""

    def __init__(self, to_tokenizer_addr: str, from_tokenizer_addr: str):
        from ..utils.mp import ZmqAsyncPullQueue, ZmqAsyncPushQueue

        self.push = ZmqAsyncPushQueue(to_tokenizer_addr, bind=False)
        self.pull = ZmqAsyncPullQueue(from_tokenizer_addr, bind=True)
        self.next_uid = 0
        self.queues: Dict[int, asyncio.Queue] = {}
        self.stops: Dict[int, StopFilter] = {}
        self._reader: Optional[asyncio.Task] = None

    def start(self) -> None:
        if self._reader is None:
            self._reader = asyncio.get_event_loop().create_task(self._read_loop())

    async def _read_loop(self) -> None:
        while True:
            msg = await self.pull.get()
            if isinstance(msg, UserReply):
                q = self.queues.get(msg.uid)
                if q is not None:
                    q.put_nowait(msg)

    async def submit(self, *, text=None, messages=None, input_ids=None, sampling: SamplingParams, stop=None) -> int:
        self.start()
        uid = self.next_uid
        self.next_uid += 1
        self.queues[uid] = asyncio.Queue()
        stops = [stop] if isinstance(stop, str) else [s for s in (stop or []) if isinstance(s, str)]
        if any(stops):
            self.stops[uid] = StopFilter(stops)
        await self.push.put(TokenizeMsg(uid=uid, text=text, messages=messages, input_ids=input_ids, sampling=sampling))
        return uid

    async def stream(self, uid: int) -> AsyncIterator[UserReply]:
        q = self.queues[uid]
        stop = self.stops.pop(uid, None)
        try:
            while True:
                msg: UserReply = await q.get()
                if stop is not None and not msg.error:
                    text, hit = stop.feed(msg.text, msg.finished)
                    msg = UserReply(uid=msg.uid, text=text, token_ids=msg.token_ids, finished=msg.finished or hit, error=msg.error)
                    if hit and not msg.error:
                        yield msg
                        await self.push.put(AbortMsg(uid=uid))          # the backend stops generating for this request
                        return
                yield msg
                if msg.finished:
                    return
        finally:
            self.queues.pop(uid, None)

    async def abort(self, uid: int) -> None:
        self.queues.pop(uid, None)
        self.stops.pop(uid, None)
        await self.push.put(AbortMsg(uid=uid))

    async def collect(self, uid: int) -> UserReply:
        text, ids, err = "", [], None
        async for m in self.stream(uid):
            text += m.text
            ids += m.token_ids
            err = err or m.error
        return UserReply(uid=uid, text=text, token_ids=ids, finished=True, error=err)


def create_app(manager: FrontendManager, model_name: str) -> FastAPI:
    app = FastAPI(title="fastafd_b200")
    created = int(time.time())

    async def sse_with_abort(request: Request, uid: int, fmt: Callable[[UserReply], List[str]], tail: List[str]):
        try:
            async for msg in manager.stream(uid):
                if await request.is_disconnected():
                    await manager.abort(uid)
                    return
                for line in fmt(msg):
                    yield line
            for line in tail:
                yield line
        except asyncio.CancelledError:
            await manager.abort(uid)
            raise

    @app.post("/generate")
    async def generate(req: GenerateRequest, request: Request):
        sp = SamplingParams(max_tokens=req.max_tokens, ignore_eos=req.ignore_eos)
        uid = await manager.submit(text=req.prompt, sampling=sp)

        def fmt(m: UserReply):
            if m.error:
                return [f"data: [ERROR] {m.error}\n"]
            return [f"data: {m.text}\n"] if m.text else []
        return StreamingResponse(sse_with_abort(request, uid, fmt, ["data: [DONE]\n"]), media_type="text/event-stream")

    @app.api_route("/v1", methods=["GET", "POST", "HEAD", "OPTIONS"])
    async def v1_root():
        return {"status": "ok"}

    @app.post("/v1/chat/completions")
    async def chat(req: CompletionRequest, request: Request):
        given = [x is not None for x in (req.prompt, req.messages, req.input_ids)]
        if sum(given) != 1:
            return JSONResponse({"error": "give exactly one of prompt, messages, input_ids"}, status_code=400)
        msgs = [m.model_dump() for m in req.messages] if req.messages else None
        uid = await manager.submit(text=req.prompt, messages=msgs, input_ids=req.input_ids, sampling=_sampling(req), stop=req.stop)
        if not req.stream:
            # one JSON body once the request has finished (OpenAI "stream": false)
            r = await manager.collect(uid)
            choice: Dict[str, Any] = {"index": 0, "message": {"role": "assistant", "content": r.text},
                                      "finish_reason": "error" if r.error else "stop"}
            if req.return_token_ids:
                choice["token_ids"] = r.token_ids
            body: Dict[str, Any] = {"id": f"cmpl-{uid}", "object": "chat.completion", "created": created,
                                    "model": model_name, "choices": [choice],
                                    "usage": {"completion_tokens": len(r.token_ids or [])}}
            if r.error:
                body["error"] = r.error
            return JSONResponse(body, status_code=400 if r.error else 200)
        first = {"sent_role": False}

        def chunk(delta: Dict[str, Any], finish=None, token_ids=None) -> str:
            choice = {"delta": delta, "index": 0, "finish_reason": finish}
            if token_ids is not None:
                choice["token_ids"] = token_ids
            return "data: " + json.dumps({"id": f"cmpl-{uid}", "object": "text_completion.chunk", "choices": [choice]}) + "\n\n"

        def fmt(m: UserReply):
            if m.error:
                return [chunk({"content": ""}, finish="error"), "data: " + json.dumps({"error": m.error}) + "\n\n"]
            delta: Dict[str, Any] = {}
            if not first["sent_role"]:
                delta["role"] = "assistant"
                first["sent_role"] = True
            delta["content"] = m.text
            return [chunk(delta, token_ids=m.token_ids if req.return_token_ids else None)]
        tail = [chunk({}, finish="stop"), "data: [DONE]\n\n"]
        return StreamingResponse(sse_with_abort(request, uid, fmt, tail), media_type="text/event-stream")

    # text-completion clients post {"prompt": ...} to /v1/completions: same request model and replies
    app.post("/v1/completions")(chat)

    @app.get("/health")
    async def health():
        return {"status": "ok"}

    @app.post("/v1/chat/completions/batch")
    async def chat_batch(req: BatchCompletionRequest):
        if (req.prompts is None) == (req.messages_batch is None):
            return JSONResponse({"error": "give exactly one of prompts, messages_batch"}, status_code=400)
        sp = _sampling(req)
        uids = []
        if req.prompts is not None:
            for p in req.prompts:
                uids.append(await manager.submit(text=p, sampling=sp))
        else:
            for ms in req.messages_batch:
                uids.append(await manager.submit(messages=[m.model_dump() for m in ms], sampling=sp))
        results = await asyncio.gather(*[manager.collect(u) for u in uids])
        choices = []
        for i, r in enumerate(results):
            c = {"index": i, "message": {"role": "assistant", "content": r.text},
                 "finish_reason": "error" if r.error else "stop"}
            if req.return_token_ids:
                c["token_ids"] = r.token_ids
            if r.error:
                c["error"] = r.error
            choices.append(c)
        return {"id": f"batchcmpl-{uids[0]}-{uids[-1]}", "object": "chat.completion.batch", "choices": choices}

    @app.get("/v1/models")
    async def models():
        return {"object": "list", "data": [{"id": model_name, "object": "model", "created": created,
                                            "owned_by": "fastafd_b200", "root": model_name}]}

    return app


def run_api_server(args, start_backend: Callable[[], Any], stop_backend: Callable[[], None]) -> None:
    """Start the backend, then serve HTTP until interrupted; always stops the backend."""
    import uvicorn

    addrs = start_backend()
    manager = FrontendManager(addrs.to_tokenizer, addrs.from_tokenizer)
    app = create_app(manager, args.model_path)
    # uvicorn re-raises the signal that stopped it once its loop has ended, which ends the
    # process before a `finally` here could run: stop the backend from the shutdown hook too.
    app.add_event_handler("shutdown", stop_backend)
    try:
        uvicorn.run(app, host=args.host, port=args.port, log_level=args.log_level.lower())
    finally:
        stop_backend()
