"""Messages between the HTTP frontend, the tokenizer / detokenizer workers and the
coordinator, with a msgpack codec (dataclasses are tagged by type name).

Reference: python/minisgl/message/{backend,frontend,tokenizer,utils}.py.
"""
from __future__ import annotations

from dataclasses import dataclass, field, fields, is_dataclass
from typing import Any, Dict, List, Optional

import msgpack

from ..core import SamplingParams


@dataclass
class TokenizeMsg:
    """frontend -> tokenizer: text, chat messages or ready token ids of one request."""
    uid: int
    text: Optional[str] = None
    messages: Optional[List[Dict[str, str]]] = None
    input_ids: Optional[List[int]] = None
    sampling: SamplingParams = field(default_factory=SamplingParams)


@dataclass
class UserMsg:
    """tokenizer -> coordinator: an admitted request."""
    uid: int
    input_ids: List[int]
    sampling: SamplingParams


@dataclass
class AbortMsg:
    """frontend -> tokenizer -> coordinator: the client went away."""
    uid: int


@dataclass
class DetokenizeMsg:
    """coordinator -> detokenizer: newly generated token(s) of one request."""
    uid: int
    token_ids: List[int]
    finished: bool = False
    error: Optional[str] = None


@dataclass
class BatchDetokenizeMsg:
    items: List[DetokenizeMsg] = field(default_factory=list)


@dataclass
class UserReply:
    """detokenizer -> frontend: printable text increment."""
    uid: int
    text: str
    token_ids: List[int] = field(default_factory=list)
    finished: bool = False
    error: Optional[str] = None


@dataclass
class ExitMsg:
    reason: str = ""


_TYPES = {c.__name__: c for c in (TokenizeMsg, UserMsg, AbortMsg, DetokenizeMsg, BatchDetokenizeMsg, UserReply,
                                  ExitMsg, SamplingParams)}


def _enc(o: Any) -> Any:
    if is_dataclass(o) and type(o).__name__ in _TYPES:
        return {"__t__": type(o).__name__, "f": {f.name: _enc(getattr(o, f.name)) for f in fields(o)}}
    if isinstance(o, (list, tuple)):
        return [_enc(v) for v in o]
    if isinstance(o, dict):
        return {k: _enc(v) for k, v in o.items()}
    return o


def _dec(o: Any) -> Any:
    if isinstance(o, dict):
        if "__t__" in o:
            cls = _TYPES[o["__t__"]]
            kw = {k: _dec(v) for k, v in o["f"].items()}
            if cls is SamplingParams and isinstance(kw.get("stop_token_ids"), list):
                kw["stop_token_ids"] = tuple(kw["stop_token_ids"])
            return cls(**kw)
        return {k: _dec(v) for k, v in o.items()}
    if isinstance(o, list):
        return [_dec(v) for v in o]
    return o


def serialize(msg: Any) -> bytes:
    return msgpack.packb(_enc(msg), use_bin_type=True)


def deserialize(data: bytes) -> Any:
    return _dec(msgpack.unpackb(data, raw=False))
