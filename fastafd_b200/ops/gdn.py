"""Gated DeltaNet block of the Qwen3.5 hybrid layers: causal depthwise conv + SiLU, the
gated delta rule (single-token recurrent update for decode, token loop for prefill), and
the per-head gated RMSNorm.

CUDA tensors go to the kernels in csrc/gdn.cu; CPU tensors to the oracle.
Reference: python/minisgl/kernel/qwen35_gdn.py:21-98,235-336,565-652 and
python/minisgl/kernel/qwen35_gated_norm.py:28.
"""
from __future__ import annotations

import ctypes as C

import torch

from ..reference import ops_ref as ref


def _split_qkv(mixed, hk, hv, dk, dv):
    T = mixed.shape[0]
    q = mixed[:, :hk * dk].reshape(T, hk, dk)
    k = mixed[:, hk * dk:2 * hk * dk].reshape(T, hk, dk)
    v = mixed[:, 2 * hk * dk:].reshape(T, hv, dv)
    return q, k, v


def gdn_block(mixed, z, a, b, conv_w, A_log, dt_bias, norm_w, conv_state, rec_state, meta, hk, hv, dk, dv, eps):
    """mixed [T, 2*hk*dk + hv*dv] (q|k|v pre-conv), z [T, hv*dv], a/b [T, hv].
    conv_state [slots, taps-1, C]; rec_state [slots, hv, dv, dk] fp32. Returns [T, hv*dv]."""
    if mixed.is_cuda and not meta.is_prefill:
        return _gdn_decode_cuda(mixed, z, a, b, conv_w, A_log, dt_bias, norm_w, conv_state, rec_state, meta,
                                hk, hv, dk, dv, eps)
    if mixed.is_cuda:
        return _gdn_prefill_cuda(mixed, z, a, b, conv_w, A_log, dt_bias, norm_w, conv_state, rec_state, meta,
                                 hk, hv, dk, dv, eps)
    T = mixed.shape[0]
    slots = meta.state_slots.long()
    out = torch.empty(T, hv * dv, dtype=mixed.dtype, device=mixed.device)
    if not meta.is_prefill:
        cs = conv_state[slots]
        y = ref.causal_conv1d_step(mixed, cs, conv_w)
        conv_state[slots] = cs
        q, k, v = _split_qkv(y, hk, hv, dk, dv)
        st = rec_state[slots]
        o = ref.gdn_recurrent_step(q, k, v, a, b, A_log, dt_bias, st)
        rec_state[slots] = st
        out = ref.gated_rmsnorm(o, z.view(T, hv, dv), norm_w, eps).reshape(T, hv * dv)
        return out
    off = 0
    starts = (meta.seq_lens.cpu() - torch.tensor(meta.prefill_lens, dtype=torch.int32)).tolist()
    for r, n in enumerate(meta.prefill_lens):
        if n == 0:
            continue
        s = int(slots[r])
        if starts[r] == 0:                       # fresh request: reset its state
            conv_state[s] = 0
            rec_state[s] = 0
        cs = conv_state[s:s + 1].clone()
        ys = []
        for t in range(n):
            ys.append(ref.causal_conv1d_step(mixed[off + t:off + t + 1], cs, conv_w))
        conv_state[s] = cs[0]
        y = torch.cat(ys, 0)
        q, k, v = _split_qkv(y, hk, hv, dk, dv)
        st = rec_state[s].clone()
        o = ref.gdn_prefill(q, k, v, a[off:off + n], b[off:off + n], A_log, dt_bias, st)
        rec_state[s] = st
        out[off:off + n] = ref.gated_rmsnorm(o, z[off:off + n].view(n, hv, dv), norm_w, eps).reshape(n, hv * dv)
        off += n
    if off < T:
        out[off:] = 0
    return out


def _gdn_decode_cuda(mixed, z, a, b, conv_w, A_log, dt_bias, norm_w, conv_state, rec_state, meta, hk, hv, dk, dv, eps):
    from ._lib import check, cur_stream, lib, ptr

    T = mixed.shape[0]
    dev = mixed.device
    out = torch.empty(T, hv * dv, dtype=mixed.dtype, device=dev)
    scratch = torch.empty(T, mixed.shape[1], dtype=mixed.dtype, device=dev)
    fn = lib().afd_gdn_decode_ld
    fn.restype = C.c_int
    vp = C.c_void_p
    bf = lambda t: t if t.dtype == torch.bfloat16 else t.to(torch.bfloat16)  # noqa: E731

    def rows(t):        # bf16 with unit column stride; the row stride is passed on (column ranges of one
        t = bf(t)       # merged projection output are read in place)
        return t if t.stride(1) == 1 else t.contiguous()

    mixed, z, a, b = rows(mixed), rows(z), rows(a), rows(b)
    args = [mixed, z, a, b, bf(conv_w.contiguous()),
            A_log.float().contiguous(), dt_bias.float().contiguous(), bf(norm_w.contiguous())]
    check(fn(*[vp(ptr(t)) for t in args], vp(ptr(conv_state)), vp(ptr(rec_state)), vp(ptr(meta.state_slots)),
             vp(ptr(out)), vp(ptr(scratch)), C.c_int(T), C.c_int(hk), C.c_int(hv), C.c_int(dk), C.c_int(dv),
             C.c_int(conv_w.shape[1]), C.c_int(conv_state.shape[0]), C.c_float(eps), vp(ptr(meta.status)),
             vp(cur_stream()), C.c_long(mixed.stride(0)), C.c_long(z.stride(0)), C.c_long(a.stride(0)),
             C.c_long(b.stride(0))), "gdn_decode")
    return out


def _gdn_prefill_cuda(mixed, z, a, b, conv_w, A_log, dt_bias, norm_w, conv_state, rec_state, meta, hk, hv, dk, dv, eps):
    """Packed sequences of a prefill chunk through csrc/gdn.cu (conv, token-serial delta rule with
    the state rows in registers, gated norm). A sequence whose chunk starts at position 0 starts
    from zero state."""
    import numpy as np

    from ._lib import check, cur_stream, lib, ptr

    T = mixed.shape[0]
    dev = mixed.device
    lens = np.asarray(meta.prefill_lens, dtype=np.int64)
    n = len(lens)
    cu = np.zeros(n + 1, dtype=np.int32)
    cu[1:] = np.cumsum(lens)
    starts = meta.seq_lens[:n].cpu().numpy().astype(np.int64) - lens
    host = torch.from_numpy(np.concatenate([cu, (starts == 0).astype(np.int32)]))
    meta_dev = host.to(dev, non_blocking=False)
    cu_d, fresh_d = meta_dev[:n + 1], meta_dev[n + 1:]
    out = torch.empty(T, hv * dv, dtype=torch.bfloat16, device=dev)
    C_ = mixed.shape[1]
    scratch = torch.empty(T * (C_ + hv * dv), dtype=torch.bfloat16, device=dev)
    fn = lib().afd_gdn_prefill
    fn.restype = C.c_int
    vp = C.c_void_p
    bf = lambda t: t if t.dtype == torch.bfloat16 else t.to(torch.bfloat16)  # noqa: E731
    args = [bf(mixed.contiguous()), bf(z.contiguous()), bf(a.contiguous()), bf(b.contiguous()), bf(conv_w.contiguous()),
            A_log.float().contiguous(), dt_bias.float().contiguous(), bf(norm_w.contiguous())]
    check(fn(*[vp(ptr(t)) for t in args], vp(ptr(conv_state)), vp(ptr(rec_state)), vp(ptr(meta.state_slots)),
             vp(ptr(cu_d)), vp(ptr(fresh_d)), vp(ptr(out)), vp(ptr(scratch)), C.c_int(T), C.c_int(int(cu[-1])),
             C.c_int(n), C.c_int(hk), C.c_int(hv), C.c_int(dk), C.c_int(dv), C.c_int(conv_w.shape[1]),
             C.c_int(conv_state.shape[0]), C.c_float(eps), vp(ptr(meta.status)), vp(cur_stream())), "gdn_prefill")
    return out.to(mixed.dtype)
