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
    out = torch.empty(T, hv * dv, dtype=mixed.dtype, device=mixed.device)
    fn = getattr(lib(), "afd_gdn_decode", None)
    if fn is None:
        raise RuntimeError("kernel library has no afd_gdn_decode; rebuild with fastafd_b200.build")
    fn.restype = C.c_int
    check(fn(C.c_void_p(ptr(mixed)), C.c_void_p(ptr(z)), C.c_void_p(ptr(a)), C.c_void_p(ptr(b)),
             C.c_void_p(ptr(conv_w)), C.c_void_p(ptr(A_log)), C.c_void_p(ptr(dt_bias)), C.c_void_p(ptr(norm_w)),
             C.c_void_p(ptr(conv_state)), C.c_void_p(ptr(rec_state)), C.c_void_p(ptr(meta.state_slots)),
             C.c_void_p(ptr(out)), C.c_int(T), C.c_int(hk), C.c_int(hv), C.c_int(dk), C.c_int(dv),
             C.c_int(conv_w.shape[1]), C.c_int(conv_state.shape[0]), C.c_float(eps), C.c_void_p(cur_stream())),
          "gdn_decode")
    return out
