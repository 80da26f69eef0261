"""ZeroMQ queues between processes: PUSH/PULL and PUB/SUB, sync and asyncio flavours, with a
pluggable codec (the message codec by default).

Reference: python/minisgl/utils/mp.py:68-237.
"""
from __future__ import annotations

import socket
from typing import Any, Callable, List, Optional

import zmq
import zmq.asyncio


def pick_free_ports(n: int, host: str = "127.0.0.1") -> List[int]:
    """n distinct free TCP ports (held open together while probing so they do not collide)."""
    socks, ports = [], []
    for _ in range(n):
        s = socket.socket(socket.AF_INET, socket.SOCK_STREAM)
        s.bind((host, 0))
        socks.append(s)
        ports.append(s.getsockname()[1])
    for s in socks:
        s.close()
    return ports


def _default_codec():
    from ..message import deserialize, serialize

    return serialize, deserialize


class _Base:
    def __init__(self, addr: str, kind: int, bind: bool, encode=None, decode=None, asyncio_mode: bool = False):
        enc, dec = _default_codec()
        self.encode: Callable[[Any], bytes] = encode or enc
        self.decode: Callable[[bytes], Any] = decode or dec
        self.ctx = zmq.asyncio.Context.instance() if asyncio_mode else zmq.Context.instance()
        self.sock = self.ctx.socket(kind)
        self.sock.setsockopt(zmq.LINGER, 0)
        if kind == zmq.SUB:
            self.sock.setsockopt(zmq.SUBSCRIBE, b"")
        (self.sock.bind if bind else self.sock.connect)(addr)
        self.addr = addr

    def close(self) -> None:
        self.sock.close(0)


class ZmqPushQueue(_Base):
    def __init__(self, addr: str, bind: bool = False, **kw):
        super().__init__(addr, zmq.PUSH, bind, **kw)

    def put(self, msg: Any) -> None:
        self.sock.send(self.encode(msg))


class ZmqPullQueue(_Base):
    def __init__(self, addr: str, bind: bool = True, **kw):
        super().__init__(addr, zmq.PULL, bind, **kw)

    def get(self, timeout_ms: Optional[int] = None) -> Any:
        """Blocking receive; with a timeout returns None when nothing arrived."""
        if timeout_ms is not None and not self.sock.poll(timeout_ms):
            return None
        return self.decode(self.sock.recv())

    def get_nowait(self) -> Any:
        try:
            return self.decode(self.sock.recv(zmq.NOBLOCK))
        except zmq.Again:
            return None

    def empty(self) -> bool:
        return not self.sock.poll(0)


class ZmqPubQueue(_Base):
    def __init__(self, addr: str, bind: bool = True, **kw):
        super().__init__(addr, zmq.PUB, bind, **kw)

    def put(self, msg: Any) -> None:
        self.sock.send(self.encode(msg))


class ZmqSubQueue(_Base):
    def __init__(self, addr: str, bind: bool = False, **kw):
        super().__init__(addr, zmq.SUB, bind, **kw)

    def get(self, timeout_ms: Optional[int] = None) -> Any:
        if timeout_ms is not None and not self.sock.poll(timeout_ms):
            return None
        return self.decode(self.sock.recv())


class ZmqAsyncPushQueue(_Base):
    def __init__(self, addr: str, bind: bool = False, **kw):
        super().__init__(addr, zmq.PUSH, bind, asyncio_mode=True, **kw)

    async def put(self, msg: Any) -> None:
        await self.sock.send(self.encode(msg))


class ZmqAsyncPullQueue(_Base):
    def __init__(self, addr: str, bind: bool = True, **kw):
        super().__init__(addr, zmq.PULL, bind, asyncio_mode=True, **kw)

    async def get(self) -> Any:
        return self.decode(await self.sock.recv())
