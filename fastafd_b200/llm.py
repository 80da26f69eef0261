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


# The reference's keyword names for the same settings (python/minisgl/engine/config.py:20-37,
# python/minisgl/scheduler/config.py:16-18) -> RuntimeConfig fields; None = accepted, nothing to set here.
REFERENCE_KWARGS = {
    "use_dummy_weight": "dummy_weights", "max_running_req": "max_running_requests",
    "max_seq_len_override": "max_seq_len", "max_extend_tokens": "max_batched_tokens",
    "num_page_override": "num_pages", "cuda_graph_bs": "decode_graph_bs",
    "attention_backend": None, "moe_backend": None, "distributed_timeout": None, "use_pynccl": None,
    "offline_mode": None, "ep_size": None, "dp_size": None, "dp_rank": None,
}


def translate_kwargs(kw: Dict[str, object]) -> Dict[str, object]:
    """Keyword arguments of the reference's `LLM(...)` under this package's names. A value of None for a
    size override means "not given" there and is dropped."""
    out: Dict[str, object] = {}
    for k, v in kw.items():
        if k in REFERENCE_KWARGS:
            new = REFERENCE_KWARGS[k]
            if new is None or v is None:
                continue
            if k == "cuda_graph_bs":
                v = tuple(int(x) for x in v)
            out[new] = v
        else:
            out[k] = v
    return out


class LLM:
    def __init__(self, model_path: str, dtype=None, device: Optional[str] = None, **runtime_kw):
        """`dtype`: a torch dtype or its name (default bfloat16 on CUDA, float32 on CPU). Keyword arguments are
        RuntimeConfig fields; the reference's names (`use_dummy_weight`, `max_running_req`,
        `max_seq_len_override`, `max_extend_tokens`, ...) are accepted too."""
        if isinstance(dtype, str) and device is None and (dtype == "cpu" or dtype.startswith("cuda")):
            dtype, device = None, dtype            # LLM(path, "cpu"): the device given positionally
        device = device or ("cuda" if torch.cuda.is_available() else "cpu")
        self.cfg = get_model_config(model_path)
        kw = dict(model_path=model_path, num_mb=1, max_running_requests=64, cuda_graph_max_bs=64,
                  max_seq_len=min(self.cfg.max_position, 4096), device=device,
                  dtype="bfloat16" if device.startswith("cuda") else "float32",
                  use_cuda_graph=device.startswith("cuda"))
        if dtype is not None:
            kw["dtype"] = str(dtype).replace("torch.", "")
        kw.update(translate_kwargs(runtime_kw))
        self.rt = RuntimeConfig(**kw)
        self.tokenizer = load_tokenizer(model_path)
        self._out: Dict[int, List[int]] = {}
        self._uid = 0
        from .cad.config import CadConfig

        cad = CadConfig.from_env()
        if cad.enabled:
            return self._init_cad(cad, device)
        self.topo = AfdTopology(colocated=True)
        self.engine = AfdEngine(self.cfg, self.rt, self.topo, 0, device if ":" in device or device == "cpu" else device + ":0",
                                seed=self.rt.seed, fast_init=device.startswith("cuda"))
        self.coordinator = AfdCoordinator(self.cfg, self.rt, self.topo, InProcTransport({0: self.engine}),
                                          num_pages=self.engine.attn.num_pages,
                                          max_comm_tokens=self.engine.max_comm_tokens, on_tokens=self._on_tokens)

    def _init_cad(self, cad, device: str) -> None:
        """``FASTAFD_MODE=cad`` (the reference's ``MINISGL_AFD_MODE=cad``): core-attention disaggregation with
        one model rank and ``FASTAFD_CAD_ATTN_PER_MODEL`` attention ranks, every rank an object of this process.
        CPU only: between GPU processes the hop kernels and the two sides' hooks exist (cad/gpu.py), the worker
        loops that take CAD commands from the coordinator do not."""
        if device != "cpu":
            raise NotImplementedError("CAD through the offline API runs on CPU (device='cpu')")
        from .cad.coordinator import CadCoordinator
        from .cad.deploy import CadLocalWorkers

        self.engine = None
        self.topo = AfdTopology(attn_dp=cad.attn_per_model, mlp_ep=1)
        workers = CadLocalWorkers(self.cfg, self.rt, self.topo, seed=self.rt.seed, device=device)
        comm = max(self.rt.cuda_graph_max_bs, min(2048, self.rt.max_batched_tokens // max(self.rt.num_mb, 1)))
        self.coordinator = CadCoordinator(self.cfg, self.rt, self.topo, workers, num_pages=workers.num_pages,
                                          max_comm_tokens=comm, on_tokens=self._on_tokens)

    def _on_tokens(self, items) -> None:
        for uid, toks, _fin in items:
            self._out.setdefault(uid, []).extend(toks)

    def generate(self, prompts: Sequence[Union[str, Sequence[int]]],
                 sampling_params: Union[None, SamplingParams, Sequence[SamplingParams]] = None) -> List[Dict[str, object]]:
        sp = sampling_params or SamplingParams(max_tokens=16)
        sps = list(sp) if isinstance(sp, (list, tuple)) else [sp] * len(prompts)      # one for all, or one per prompt
        if len(sps) != len(prompts):
            raise ValueError(f"{len(prompts)} prompts but {len(sps)} sampling parameter sets")
        uids = []
        for p, one in zip(prompts, sps):
            ids = list(self.tokenizer.encode(p)) if isinstance(p, str) else [int(t) for t in p]
            uid = self._uid
            self._uid += 1
            self.coordinator.add_request(uid, ids, one)
            uids.append(uid)
        self.coordinator.run_until_idle()
        out = []
        for u in uids:
            toks = self._out.pop(u, [])
            out.append({"token_ids": toks, "text": self.tokenizer.decode(toks)})
        return out

    def shutdown(self) -> None:
        self.coordinator.shutdown()
        if self.engine is not None:
            self.engine.close()
