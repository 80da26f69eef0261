"""``launch_server``: parse flags, start the backend processes, serve HTTP.
Reference: python/minisgl/server/launch.py:6-23."""
from __future__ import annotations

from typing import Optional, Sequence


def launch_server(argv: Optional[Sequence[str]] = None) -> None:
    from .api_server import run_api_server
    from .args import parse_args
    from .supervisor import create_backend_supervisor

    args = parse_args(argv)
    supervisor = create_backend_supervisor(args)
    run_api_server(args, supervisor.start, stop_backend=supervisor.shutdown)
