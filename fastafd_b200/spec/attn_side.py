"""Attention-side speculative decoding (EAGLE-3 style): verify step + draft proposal.

One verify step per request processes ``block`` tokens: the last committed token followed
by ``block - 1`` draft tokens. The target model runs the normal micro-batch pipeline with
``block`` tokens per request (paged attention in multi-token mode, causal inside the block);
the LM head gives the target's own choice at each of the positions; the longest draft prefix
that equals those choices is accepted and the target's next token is appended (greedy
verification is lossless: the output equals plain greedy decoding). The draft head then
writes its KV context for the accepted positions and proposes the next ``block - 1`` tokens,
all into the device-side token pool.

The expert GPUs just see a wider decode bucket (bucket * block tokens per micro-batch).

Reference: python/minisgl/spec/attn_side.py (verify :91-136, greedy head :375-383, propose
:228-244,361-371), python/minisgl/spec/config.py:85-124 (acceptance rule, reply packing),
python/minisgl/afd_scheduler.py:516-552 (verify scheduled as a block-token extend).
"""
from __future__ import annotations

from typing import List, Optional

import numpy as np
import torch

from .. import ops
from ..models.transformer import AttnMeta
from ..protocol import AgStepPlan, AgStepReply
from ..reference import ops_ref as ref
from .eagle3 import Eagle3Config, Eagle3Draft


def simulated_accept(n_rows: int, block: int, mean_accept: float, rng: np.random.Generator) -> np.ndarray:
    """Emitted-token counts with a fixed mean in [1, block] (timing runs with a fixed acceptance
    instead of a trained draft head): each row emits floor(mean) or ceil(mean) tokens."""
    mean = min(max(mean_accept, 1.0), float(block))
    lo = int(np.floor(mean))
    p_hi = mean - lo
    n = lo + (rng.random(n_rows) < p_hi).astype(np.int32)
    return np.clip(n, 1, block).astype(np.int32)


class SpecRunner:
    """Bound to an AttentionWorker; owns the draft head and the verify step."""

    def __init__(self, worker, block: int, draft_path: str = "", seed: int = 0, sim_accept: float = 0.0):
        self.w, self.block, self.sim_accept = worker, block, sim_accept
        self.rng = np.random.default_rng(seed)
        cfg = worker.cfg
        self.dcfg = Eagle3Config.for_target(cfg)
        slots = worker.kv.num_pages * worker.kv.page_size
        self.draft = Eagle3Draft(self.dcfg, worker.device, worker.dtype, slots)
        if draft_path:
            self.draft.load(draft_path)
        else:
            self.draft.init_random(seed, share_embedding=worker.model.w["model.embed_tokens.weight"])
        self.capture_layers = list(self.dcfg.target_layers)
        self.accept_hist = np.zeros(block + 1, np.int64)

    # ------------------------------------------------------------------ helpers
    def _meta(self, rows: torch.Tensor, first_pos: torch.Tensor, q_len: int) -> AttnMeta:
        w, ps = self.w, self.w.page_size
        B = rows.shape[0]
        pos = (first_pos[:, None] + torch.arange(q_len, device=rows.device, dtype=first_pos.dtype)[None]).reshape(-1)
        pt = w.page_table_all[rows]
        page = torch.gather(pt, 1, (pos.view(B, q_len) // ps).long()).reshape(-1)
        loc = (page * ps + pos % ps).to(torch.int32)
        return AttnMeta(positions=pos.to(torch.int32), out_loc=loc, page_table=pt, seq_lens=(first_pos + q_len).to(torch.int32),
                        q_len=q_len, state_slots=rows.to(torch.int32), status=w.status)

    def write_prefill_context(self, rows: torch.Tensor, starts: List[int], lens: List[int], ids: torch.Tensor,
                              aux: List[torch.Tensor], first_tokens: Optional[torch.Tensor], sample_mask) -> None:
        """Draft KV for the prompt chunk just prefilled: position p gets (token p+1, feature p).
        The chunk's last position needs the token after the chunk: the sampled first token when
        the prompt ended here, else it is left for the next chunk (only acceptance can suffer)."""
        feat = self.draft.fuse_features(aux)
        off, si = 0, 0
        for b, n in enumerate(lens):
            if n == 0:
                continue
            nxt = ids[off + 1:off + n]
            use = n - 1
            if sample_mask[b]:
                nxt = torch.cat([nxt, first_tokens[si:si + 1].to(ids.dtype)])
                use = n
                si += 1
            if use > 0:
                meta = self._meta(rows[b:b + 1], torch.tensor([starts[b]], device=rows.device, dtype=torch.int32), use)
                self.draft.layer(nxt[:use].contiguous(), feat[off:off + use].contiguous(), meta, self.w.page_size)
            off += n

    # ------------------------------------------------------------------ verify step
    def run_verify(self, plan: AgStepPlan) -> AgStepReply:
        w, k = self.w, self.block
        dev = w.device
        mbs, rows_l, L_l = [], [], []
        w.apply_grants(plan)
        for lane, mbp in enumerate(plan.mbs):
            rows = torch.from_numpy(mbp.rows.astype(np.int64)).to(dev)
            L = torch.from_numpy((mbp.seq_lens - k).astype(np.int32)).to(dev)       # committed KV length
            meta = self._meta(rows, L, k)
            ids = w.token_pool[rows[:, None], (L[:, None] + torch.arange(k, device=dev)[None]).long()].reshape(-1).contiguous()
            mb = w.make_ctx(lane, ids, meta)
            mb.capture = {}
            mbs.append(mb)
            rows_l.append(rows)
            L_l.append(L)
        w.pipeline(mbs, capture_layers=self.capture_layers)
        out_tokens, out_n = [], []
        for lane, (mb, mbp) in enumerate(zip(mbs, plan.mbs)):
            B = len(mbp.rows)
            rows, L = rows_l[lane], L_l[lane]
            logits = w.model.lm_head(mb.normed)
            target = ops.argmax(logits).view(B, k).to(torch.int64)
            drafts = mb.ids.view(B, k)[:, 1:].to(torch.int64)
            n, emitted = ref.greedy_accept(drafts, target)
            if self.sim_accept > 0:
                n = torch.from_numpy(simulated_accept(B, k, self.sim_accept, self.rng)).to(dev)
                emitted = torch.where(torch.arange(k, device=dev)[None] < n[:, None], target, torch.full_like(target, -1))
            n = n.to(torch.int64)
            # commit: pool[row, L+1+j] = emitted[j] for j < n
            j = torch.arange(k, device=dev)[None]
            valid = j < n[:, None]
            r_idx = rows[:, None].expand(B, k)[valid]
            p_idx = (L[:, None].long() + 1 + j).expand(B, k)[valid]
            w.token_pool[r_idx, p_idx] = emitted[valid].to(torch.int32)
            # draft: context for positions L..L+k-1 (the ones past L+n-1 are overwritten later), then chain
            feat = self.draft.fuse_features([mb.capture[l] for l in self.capture_layers])
            nxt = torch.where(valid, emitted, torch.zeros_like(emitted)).to(torch.int32).reshape(-1).contiguous()
            h = self.draft.layer(nxt, feat, self._meta(rows, L, k), w.page_size).view(B, k, -1)
            last = h[torch.arange(B, device=dev), (n - 1).clamp(0, k - 1)]            # output at position L' - 1
            newL = L.long() + n                                                        # L' (bonus token sits at L')
            for i in range(k - 1):
                tok = self.draft.logits_to_tokens(last)                               # draft i+1 -> position L'+1+i
                w.token_pool[rows, newL + 1 + i] = tok
                if i + 1 < k - 1:
                    meta1 = self._meta(rows, (newL + i).to(torch.int32), 1)
                    last = self.draft.layer(tok.contiguous(), last.contiguous(), meta1, w.page_size)
            out_tokens.append(emitted.to(torch.int32).cpu().numpy().reshape(-1))
            nn = n.to(torch.int32).cpu().numpy()
            out_n.append(nn)
            for v in nn[:mbp.num_real]:
                self.accept_hist[int(v)] += 1
        if w.cuda:
            torch.cuda.current_stream().synchronize()
        return AgStepReply(step_id=plan.step_id, rank=w.rank, next_tokens=np.concatenate(out_tokens),
                           accepted=np.concatenate(out_n), status=w.read_status())

    def mean_accept(self) -> float:
        tot = self.accept_hist.sum()
        return float((self.accept_hist * np.arange(len(self.accept_hist))).sum() / tot) if tot else 0.0
