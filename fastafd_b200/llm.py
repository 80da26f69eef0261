"""Offline API: ``LLM(model).generate(prompts | token-id lists, sampling_params)``.

Runs the engine in this process (colocated on one device) under the coordinator, with the
same scheduler, paging and pipeline as the server. Reference: python/minisgl/llm/llm.py:28-98.
"""
from __future__ import annotations

from typing import Dict, List, Optional, Sequence, Union

import torch

from .config import RuntimeConfig, get_model_config
from .coordinator import AfdCoordinator, InProcTransport
from .core import SamplingParams
from .engine import AfdEngine
from .protocol import AfdTopology
from .tokenizer import load_tokenizer


class LLM:
    def __init__(self, model_path: str, device: Optional[str] = None, **runtime_kw):
        device = device or ("cuda" if torch.cuda.is_available() else "cpu")
        self.cfg = get_model_config(model_path)
        kw = dict(model_path=model_path, num_mb=1, max_running_requests=64, cuda_graph_max_bs=64,
                  max_seq_len=min(self.cfg.max_position, 4096), device=device,
                  dtype="bfloat16" if device.startswith("cuda") else "float32",
                  use_cuda_graph=device.startswith("cuda"))
        kw.update(runtime_kw)
        self.rt = RuntimeConfig(**kw)
        self.topo = AfdTopology(colocated=True)
        self.engine = AfdEngine(self.cfg, self.rt, self.topo, 0, device if ":" in device or device == "cpu" else device + ":0",
                                seed=self.rt.seed, fast_init=device.startswith("cuda"))
        self.tokenizer = load_tokenizer(model_path)
        self._out: Dict[int, List[int]] = {}
        self.coordinator = AfdCoordinator(self.cfg, self.rt, self.topo, InProcTransport({0: self.engine}),
                                          num_pages=self.engine.attn.num_pages,
                                          max_comm_tokens=self.engine.max_comm_tokens, on_tokens=self._on_tokens)
        self._uid = 0

    def _on_tokens(self, items) -> None:
        for uid, toks, _fin in items:
            self._out.setdefault(uid, []).extend(toks)

    def generate(self, prompts: Sequence[Union[str, Sequence[int]]],
                 sampling_params: Optional[SamplingParams] = None) -> List[Dict[str, object]]:
        sp = sampling_params or SamplingParams(max_tokens=16)
        uids = []
        for p in prompts:
            ids = list(self.tokenizer.encode(p)) if isinstance(p, str) else [int(t) for t in p]
            uid = self._uid
            self._uid += 1
            self.coordinator.add_request(uid, ids, sp)
            uids.append(uid)
        self.coordinator.run_until_idle()
        out = []
        for u in uids:
            toks = self._out.pop(u, [])
            out.append({"token_ids": toks, "text": self.tokenizer.decode(toks)})
        return out

    def shutdown(self) -> None:
        self.coordinator.shutdown()
        self.engine.close()
