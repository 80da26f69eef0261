"""How an attention rank reaches the experts, and how an expert rank serves them.

Three transports behind one pair of interfaces (:class:`MoeClient` on the attention side,
:class:`MoeServer` on the expert side):

* fabric  - CUDA: fused push / grouped GEMM / combine kernels over NVLink peer memory
            (:mod:`fastafd_b200.moe.afd_moe`). In a colocated single-GPU run the client also
            drives the expert endpoint on the same stream.
* gloo    - CPU processes: tensors travel by ``torch.distributed`` point-to-point messages
            (the plumbing slice; numerics identical to the single-process oracle).
* local   - one CPU process holds both stages (the oracle).

Reference roles: python/minisgl/moe/megamoe_m2n_afd.py (ag_moe / eg_moe),
python/minisgl/moe/deepep_m2n_adapter.py (dispatch / combine).
"""
from __future__ import annotations

from typing import Dict, List, Optional, Sequence

import torch
import torch.distributed as dist

from .. import ops
from ..models.transformer import ExpertStage, combine_rows


class MoeClient:
    """Attention-side interface. `combine` fuses: y = scale * sum_k w_k * rows_k (+ extra);
    residual += y; returns rmsnorm(residual) * norm_w (written into `normed_out` if given)."""

    def dispatch(self, lane: int, layer: int, x, topk_idx, topk_w) -> None:
        raise NotImplementedError

    def combine(self, lane: int, layer: int, T: int, topk_w, topk_idx, residual, norm_w, eps: float, *,
                extra=None, scale: float = 1.0, offset1: bool = False, normed_out=None):
        raise NotImplementedError

    def status_tensors(self) -> List[torch.Tensor]:
        return []

    # Optional fast path: one launch for post-attention norm + router + dispatch. Clients that
    # have it return True from `can_fuse_route`.
    def can_fuse_route(self, T: int, num_experts: int, hidden: int) -> bool:
        return False


def _finish_combine(y, residual, norm_w, eps, offset1, normed_out):
    normed = ops.add_rmsnorm(y, residual, norm_w, eps, offset1)
    if normed_out is not None:
        normed_out.copy_(normed)
        return normed_out
    return normed


class LocalMoeClient(MoeClient):
    """Single process, CPU: experts are called directly (all expert ranks emulated in turn)."""

    def __init__(self, stages: Sequence[ExpertStage]):
        self.stages = list(stages)
        self._pending: Dict[int, torch.Tensor] = {}

    def dispatch(self, lane, layer, x, topk_idx, topk_w):
        rows = None
        for st in self.stages:
            r = st.run_experts_dense(layer, x, topk_idx)
            rows = r if rows is None else rows + r
        self._pending[lane] = rows

    def combine(self, lane, layer, T, topk_w, topk_idx, residual, norm_w, eps, *, extra=None, scale=1.0,
                offset1=False, normed_out=None):
        y = combine_rows(self._pending.pop(lane), topk_w, topk_idx, scale)
        if extra is not None:
            y = (y.float() + extra.float()).to(y.dtype)
        return _finish_combine(y, residual, norm_w, eps, offset1, normed_out)


class NullMoeClient(MoeClient):
    """No experts at all: the MoE output is taken to be zero. Only for measuring the
    attention side in isolation."""

    def dispatch(self, lane, layer, x, topk_idx, topk_w):
        pass

    def combine(self, lane, layer, T, topk_w, topk_idx, residual, norm_w, eps, *, extra=None, scale=1.0,
                offset1=False, normed_out=None):
        return ops.rmsnorm(residual, norm_w, eps, offset1, out=normed_out)


class GlooMoeClient(MoeClient):
    """CPU multi-process: send (x, idx) to every expert rank, receive per-(k, token) rows."""

    def __init__(self, expert_ranks: Sequence[int], hidden: int, topk: int, group=None):
        self.expert_ranks, self.hidden, self.topk, self.group = list(expert_ranks), hidden, topk, group
        self._reqs: Dict[int, list] = {}

    def dispatch(self, lane, layer, x, topk_idx, topk_w):
        reqs = []
        hdr = torch.tensor([x.shape[0]], dtype=torch.int64)
        xc, ic = x.contiguous(), topk_idx.contiguous()
        for r in self.expert_ranks:
            reqs.append(dist.isend(hdr, r, group=self.group, tag=lane))
            reqs.append(dist.isend(xc, r, group=self.group, tag=lane))
            reqs.append(dist.isend(ic, r, group=self.group, tag=lane))
        self._reqs[lane] = reqs + [hdr, xc, ic]

    def combine(self, lane, layer, T, topk_w, topk_idx, residual, norm_w, eps, *, extra=None, scale=1.0,
                offset1=False, normed_out=None):
        for q in self._reqs.pop(lane, []):
            if hasattr(q, "wait"):
                q.wait()
        rows = torch.zeros(self.topk, T, self.hidden, dtype=residual.dtype)
        buf = torch.empty_like(rows)
        for r in self.expert_ranks:
            dist.recv(buf, r, group=self.group, tag=lane)
            rows += buf          # supports are disjoint: every (k, token) row comes from one rank
        y = combine_rows(rows, topk_w, topk_idx, scale)
        if extra is not None:
            y = (y.float() + extra.float()).to(y.dtype)
        return _finish_combine(y, residual, norm_w, eps, offset1, normed_out)


class FabricMoeClient(MoeClient):
    """CUDA: the fused kernels. `colocated` is an expert server living in the same process
    and GPU (single-GPU runs): its layer is launched right after the push on the same stream."""

    def __init__(self, endpoint, colocated: Optional["FabricMoeServer"] = None, tp_expand: int = 1, base_experts: int = 0):
        self.ep, self.colocated = endpoint, colocated
        # MLP tensor parallelism: expert e's slice r is virtual expert r * base_experts + e on expert
        # rank r; every routing entry is repeated for the tp slices (same weight).
        self.tp_expand, self.base_experts = tp_expand, base_experts
        self._expanded = {}

    def _expand(self, lane, topk_idx, topk_w):
        n, E = self.tp_expand, self.base_experts
        idx = torch.cat([torch.where(topk_idx >= 0, topk_idx + r * E, topk_idx) for r in range(n)], dim=1).contiguous()
        w = torch.cat([topk_w] * n, dim=1).contiguous()
        self._expanded[lane] = (idx, w)
        return idx, w

    def dispatch(self, lane, layer, x, topk_idx, topk_w):
        if self.tp_expand > 1:
            topk_idx, topk_w = self._expand(lane, topk_idx, topk_w)
        self.ep.dispatch(lane, x, topk_idx)
        if self.colocated is not None:
            self.colocated.serve(lane, layer, x.shape[0])

    def can_fuse_route(self, T, num_experts, hidden):
        return self.tp_expand == 1 and T <= 256 and num_experts <= 512 and hidden % 256 == 0 and hidden <= 4096

    def route_dispatch(self, lane, layer, attn_out, residual, norm_w, gate_w, gate_bias, x_out, topk_idx, topk_w, *,
                       scoring, renorm, eps, offset1=False):
        local = None
        if self.colocated is not None and self.ep.cfg.use_direct(attn_out.shape[0]):
            local = self.colocated.ep.schedule_desc(lane)
        self._scheduled = self.ep.route_dispatch(lane, attn_out, residual, norm_w, gate_w, gate_bias, x_out, topk_idx, topk_w,
                                                 scoring=scoring, renorm=renorm, eps=eps, offset1=offset1,
                                                 local_schedule=local)

    def after_dispatch(self, lane, layer, T):
        """Work that follows a push in the same process (colocated expert stage)."""
        if self.colocated is not None:
            self.colocated.serve(lane, layer, T, scheduled=bool(getattr(self, "_scheduled", False)))
            self._scheduled = False

    def combine(self, lane, layer, T, topk_w, topk_idx, residual, norm_w, eps, *, extra=None, scale=1.0,
                offset1=False, normed_out=None):
        if normed_out is None:
            normed_out = torch.empty_like(residual)
        if self.tp_expand > 1:
            topk_idx, topk_w = self._expanded.pop(lane)
        return self.ep.combine_reduce(lane, topk_w, topk_idx, T, scale=scale, extra=extra, residual=residual,
                                      norm_w=norm_w, normed=normed_out, eps=eps, offset1=offset1)

    def status_tensors(self):
        out = [self.ep.status]
        if self.colocated is not None:
            out.append(self.colocated.ep.status)
        return out


class MoeServer:
    def serve(self, lane: int, layer: int, T: int, scheduled: bool = False) -> None:
        raise NotImplementedError


class FabricMoeServer(MoeServer):
    def __init__(self, endpoint, stage: ExpertStage):
        self.ep, self.stage = endpoint, stage

    def serve(self, lane, layer, T, scheduled=False):
        s = self.stage
        self.ep.run_layer(lane, T, s.w13[layer], s.w2[layer], s.w13_scale[layer], s.w2_scale[layer], scheduled=scheduled)


class GlooMoeServer(MoeServer):
    def __init__(self, stage: ExpertStage, source_ranks: Sequence[int], hidden: int, topk: int, dtype, group=None):
        self.stage, self.sources, self.hidden, self.topk, self.dtype, self.group = stage, list(source_ranks), hidden, topk, dtype, group

    def serve(self, lane, layer, T, scheduled=False):
        """T is ignored: each source announces its own token count."""
        outs = []
        for r in self.sources:
            hdr = torch.zeros(1, dtype=torch.int64)
            dist.recv(hdr, r, group=self.group, tag=lane)
            t = int(hdr[0])
            x = torch.empty(t, self.hidden, dtype=self.dtype)
            idx = torch.empty(t, self.topk, dtype=torch.int32)
            dist.recv(x, r, group=self.group, tag=lane)
            dist.recv(idx, r, group=self.group, tag=lane)
            outs.append((r, self.stage.run_experts_dense(layer, x, idx).contiguous()))
        for r, rows in outs:
            dist.send(rows, r, group=self.group, tag=lane)
