"""Tokenizer / detokenizer worker process.

It sits between the HTTP frontend and the coordinator: tokenises incoming requests (chat
template for message lists, verbatim ids for the ``input_ids`` extension) and turns the
coordinator's token stream back into printable text increments, holding back bytes that do
not yet form a complete character.

Without a Hugging Face tokenizer on disk (synthetic presets) a byte-level tokenizer is used
so that the serving path stays testable end to end.

Reference: python/minisgl/tokenizer/{server,tokenize,detokenize}.py.
"""
from __future__ import annotations

import os
from typing import Dict, List, Optional, Sequence

from ..message import (AbortMsg, BatchDetokenizeMsg, DetokenizeMsg, ExitMsg, TokenizeMsg, UserMsg, UserReply)


class ByteTokenizer:
    """ids 0..255 are bytes; 256 = BOS, 257 = EOS. Vocabulary ids above that decode to ''."""
    eos_token_id = 257
    bos_token_id = 256

    def encode(self, text: str) -> List[int]:
        return list(text.encode("utf-8"))

    def decode(self, ids: Sequence[int]) -> str:
        return bytes(i for i in ids if 0 <= i < 256).decode("utf-8", errors="replace")

    def apply_chat_template(self, messages, tokenize=False, add_generation_prompt=True):
        text = "".join(f"<|{m['role']}|>{m['content']}\n" for m in messages)
        if add_generation_prompt:
            text += "<|assistant|>"
        return self.encode(text) if tokenize else text


def load_tokenizer(model_path: str):
    """A Hugging Face tokenizer when the path holds one (offline), else the byte tokenizer."""
    if os.path.isdir(model_path) and any(os.path.exists(os.path.join(model_path, f))
                                         for f in ("tokenizer.json", "tokenizer.model", "tokenizer_config.json")):
        os.environ.setdefault("HF_HUB_OFFLINE", "1")
        from transformers import AutoTokenizer

        return AutoTokenizer.from_pretrained(model_path, local_files_only=True)
    return ByteTokenizer()


def tokenize_request(tok, msg: TokenizeMsg, vocab_size: int, max_seq_len: int) -> List[int]:
    if msg.input_ids is not None:
        from ..server.prompt_ids import validate_prompt_ids

        return validate_prompt_ids(msg.input_ids, vocab_size, max_seq_len)
    if msg.messages is not None:
        text = tok.apply_chat_template(msg.messages, tokenize=False, add_generation_prompt=True)
        return list(tok.encode(text))
    return list(tok.encode(msg.text or ""))


class DetokenizeManager:
    """Incremental detokenisation per request: decode the tail of the id sequence and emit
    only text that can no longer change (no dangling replacement character at the end)."""

    def __init__(self, tok):
        self.tok = tok
        self.state: Dict[int, dict] = {}

    def step(self, msg: DetokenizeMsg) -> UserReply:
        st = self.state.setdefault(msg.uid, {"ids": [], "sent": 0, "read": 0})
        st["ids"].extend(msg.token_ids)
        ids = st["ids"]
        # decode from a few tokens back so that merges across the boundary come out right
        start = max(st["read"] - 6, 0)
        prefix = self.tok.decode(ids[start:st["read"]]) if st["read"] > start else ""
        full = self.tok.decode(ids[start:])
        piece = full[len(prefix):] if full.startswith(prefix) else full
        if piece.endswith("�") and not msg.finished:
            piece = ""                      # incomplete multi-byte character: wait for more tokens
        else:
            st["read"] = len(ids)
        if msg.finished or msg.error:
            self.state.pop(msg.uid, None)
        return UserReply(uid=msg.uid, text=piece, token_ids=list(msg.token_ids), finished=msg.finished, error=msg.error)


def tokenize_worker(model_path: str, vocab_size: int, max_seq_len: int, addr_from_frontend: str,
                    addr_to_backend: str, addr_from_backend: str, addr_to_frontend: str, ready=None) -> None:
    """Process entry point. Two inbound queues (frontend requests, backend tokens), two outbound."""
    import zmq

    from ..utils.mp import ZmqPullQueue, ZmqPushQueue

    tok = load_tokenizer(model_path)
    detok = DetokenizeManager(tok)
    q_req = ZmqPullQueue(addr_from_frontend, bind=True)
    q_tok = ZmqPullQueue(addr_from_backend, bind=True)
    to_backend = ZmqPushQueue(addr_to_backend, bind=False)
    to_frontend = ZmqPushQueue(addr_to_frontend, bind=False)
    if ready is not None:
        ready.set()
    poller = zmq.Poller()
    poller.register(q_req.sock, zmq.POLLIN)
    poller.register(q_tok.sock, zmq.POLLIN)
    while True:
        for sock, _ in poller.poll(1000):
            msg = (q_req if sock is q_req.sock else q_tok).get()
            if isinstance(msg, ExitMsg):
                to_backend.put(msg)
                return
            if isinstance(msg, TokenizeMsg):
                try:
                    ids = tokenize_request(tok, msg, vocab_size, max_seq_len)
                    to_backend.put(UserMsg(uid=msg.uid, input_ids=ids, sampling=msg.sampling))
                except Exception as e:  # bad request: answer the client, do not kill the worker
                    to_frontend.put(UserReply(uid=msg.uid, text="", finished=True, error=str(e)))
            elif isinstance(msg, AbortMsg):
                to_backend.put(msg)
                detok.state.pop(msg.uid, None)
            elif isinstance(msg, BatchDetokenizeMsg):
                for item in msg.items:
                    to_frontend.put(detok.step(item))
            elif isinstance(msg, DetokenizeMsg):
                to_frontend.put(detok.step(msg))
