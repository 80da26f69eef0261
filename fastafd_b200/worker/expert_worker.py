"""Expert-GPU (MLP server) worker: serves every MoE layer of every lane of a step.

A step is `for layer in moe_layers: for lane in lanes: serve(lane, layer, T_lane)`, in the
same order in which the attention ranks dispatch. On CUDA the whole step for a decode bucket
is one CUDA graph (all kernels on one stream; the grouping kernel of each layer waits,
bounded, for the attention ranks' flags), so a decode step costs one graph launch.

Reference: python/minisgl/afd_expert_worker.py:214-400,421-532 (_run_eg_megamoe_pipeline_body,
AfdEgDecodeGraphRunner, _run_afd_eg_step).
"""
from __future__ import annotations

import time
from typing import Dict, List, Optional

import torch

from ..config import ModelConfig, RuntimeConfig
from ..models.transformer import ExpertStage
from ..protocol import EgStepPlan, EgStepReply
from ..utils.trace import nvtx_range
from .moe_client import MoeServer


class ExpertWorker:
    def __init__(self, cfg: ModelConfig, rt: RuntimeConfig, device, stage: ExpertStage, server: MoeServer,
                 rank: int = 0, status: Optional[torch.Tensor] = None):
        self.cfg, self.rt, self.device, self.stage, self.server, self.rank = cfg, rt, torch.device(device), stage, server, rank
        self.cuda = self.device.type == "cuda"
        self.status = status
        self.graphs: Dict[tuple, "torch.cuda.CUDAGraph"] = {}
        self.kernels_per_step = 0
        if self.cuda:
            self.stream = torch.cuda.Stream(self.device)

    def _body(self, tokens_per_mb: List[int]) -> None:
        for layer in self.stage.moe_layers:
            for lane, T in enumerate(tokens_per_mb):
                with nvtx_range(f"AFD_EG_L{layer}_mb{lane}"):
                    self.server.serve(lane, layer, T)

    def run_step(self, plan: EgStepPlan) -> EgStepReply:
        t0 = time.perf_counter()
        key = tuple(plan.tokens_per_mb)
        if self.cuda:
            with torch.cuda.stream(self.stream):
                if plan.phase != "prefill" and self.rt.use_cuda_graph:
                    if key not in self.graphs:
                        self._body(list(key))                    # eager pass: pairs with the peers' warm-up
                        torch.cuda.synchronize(self.device)
                        from ..ops._lib import LAUNCHES

                        g = torch.cuda.CUDAGraph()
                        c0 = LAUNCHES["count"]
                        with torch.cuda.graph(g, stream=self.stream, capture_error_mode="thread_local"):
                            self._body(list(key))
                        self.kernels_per_step = LAUNCHES["count"] - c0
                        self.graphs[key] = g
                    self.graphs[key].replay()
                else:
                    self._body(list(key))
        else:
            self._body(list(key))
        return EgStepReply(step_id=plan.step_id, rank=self.rank, step_ms=(time.perf_counter() - t0) * 1e3)

    def finish(self) -> int:
        if self.cuda:
            self.stream.synchronize()
            return int(self.status.item()) if self.status is not None else 0
        return 0
