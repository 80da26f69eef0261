"""ctypes binding of ``libfastafd_kernels.so`` (the sm_100a kernel library).

The library is built ahead of time by :mod:`fastafd_b200.build`. On a machine with
a GPU a missing library is an error, never a silent fallback: the CUDA path is the
product and the PyTorch implementations in :mod:`fastafd_b200.reference` exist for
CPU runs and as test oracles only.
"""
from __future__ import annotations

import ctypes as C
from functools import lru_cache

from ..build import build_extension, lib_path

MAX_PEERS = 16
VP = C.c_void_p


class GroupedGemmDesc(C.Structure):
    _fields_ = [
        ("w", VP), ("x", VP),
        ("num_experts", C.c_int), ("n_per_expert", C.c_int), ("k", C.c_int), ("pool_rows", C.c_int),
        ("block_tok", C.c_int), ("fp8", C.c_int), ("epilogue", C.c_int), ("grid", C.c_int),
        ("tile_info", VP), ("num_tok_tiles", VP),
        ("max_tok_tiles", C.c_int),
        ("out", VP), ("out_ld", C.c_int),
        ("x_scale", VP), ("w_scale", VP), ("out_q", VP), ("out_scale", VP),
        ("row_meta", VP),
        ("peer_combine", VP * MAX_PEERS), ("peer_flag", VP * MAX_PEERS),
        ("num_peers", C.c_int), ("combine_tokens", C.c_int), ("hidden", C.c_int),
        ("epoch", VP), ("done_counter", VP), ("status", VP), ("trace", VP),
        ("k_splits", C.c_int), ("splitk_ws", VP), ("splitk_cnt", VP), ("bias", VP),
        ("w_tile_major", C.c_int),
        ("l2_prefetch_bytes", C.c_int),
    ]


class DispatchDesc(C.Structure):
    _fields_ = [
        ("x", VP), ("topk_idx", VP),
        ("T", C.c_int), ("H", C.c_int), ("K", C.c_int), ("src_rank", C.c_int),
        ("num_eg", C.c_int), ("experts_per_eg", C.c_int), ("fp8", C.c_int), ("recv_tokens", C.c_int),
        ("peer_recv_x", VP * MAX_PEERS), ("peer_recv_scale", VP * MAX_PEERS),
        ("peer_recv_idx", VP * MAX_PEERS), ("peer_flag", VP * MAX_PEERS),
        ("epoch", VP), ("done_counter", VP), ("status", VP), ("trace", VP),
    ]


class RouteDispatchDesc(C.Structure):
    _fields_ = [
        ("attn_out", VP), ("residual", VP), ("norm_w", VP), ("gate_w", VP), ("gate_bias", VP),
        ("x_out", VP), ("topk_idx_out", VP), ("topk_w_out", VP),
        ("E", C.c_int), ("gate_fp32", C.c_int), ("scoring", C.c_int), ("renorm", C.c_int), ("offset1", C.c_int),
        ("eps", C.c_float), ("route_scale", C.c_float),
        ("d", DispatchDesc),
    ]


class DirectDesc(C.Structure):
    _fields_ = [
        ("peer_pool", VP * MAX_PEERS), ("peer_scale", VP * MAX_PEERS), ("peer_meta", VP * MAX_PEERS),
        ("peer_count", VP * MAX_PEERS), ("peer_flag", VP * MAX_PEERS),
        ("num_eg", C.c_int), ("experts_per_eg", C.c_int), ("cap", C.c_int), ("fp8", C.c_int),
        ("T", C.c_int), ("H", C.c_int), ("K", C.c_int), ("src_rank", C.c_int),
        ("epoch", VP), ("done_counter", VP), ("status", VP), ("trace", VP),
    ]


class ScheduleDesc(C.Structure):
    _fields_ = [
        ("n2m_flag", VP), ("A", C.c_int), ("epoch", VP), ("counts", VP),
        ("experts_local", C.c_int), ("cap", C.c_int), ("block_tok", C.c_int), ("max_tok_tiles", C.c_int),
        ("tile_info", VP), ("counters", VP), ("expert_counts", VP),
        ("timeout_ns", C.c_ulonglong),
        ("status", VP), ("trace", VP),
    ]


class RouteDirectDesc(C.Structure):
    _fields_ = [
        ("attn_out", VP), ("residual", VP), ("norm_w", VP), ("gate_w", VP), ("gate_bias", VP),
        ("x_out", VP), ("topk_idx_out", VP), ("topk_w_out", VP),
        ("E", C.c_int), ("gate_fp32", C.c_int), ("scoring", C.c_int), ("renorm", C.c_int), ("offset1", C.c_int),
        ("eps", C.c_float), ("route_scale", C.c_float),
        ("tokens_per_cta", C.c_int), ("cluster", C.c_int),
        ("d", DirectDesc),
        ("fuse_schedule", C.c_int), ("sched", ScheduleDesc),
    ]


class GroupDesc(C.Structure):
    _fields_ = [
        ("recv_idx", VP), ("n2m_flag", VP), ("epoch", VP),
        ("A", C.c_int), ("T", C.c_int), ("K", C.c_int), ("recv_tokens", C.c_int),
        ("expert_base", C.c_int), ("experts_local", C.c_int), ("block_tok", C.c_int),
        ("pool_rows", C.c_int), ("max_tok_tiles", C.c_int),
        ("row_meta", VP), ("tile_info", VP), ("counters", VP), ("expert_counts", VP),
        ("timeout_ns", C.c_ulonglong),
        ("status", VP),
        ("recv_x", VP), ("recv_scale", VP), ("pool_x", VP), ("pool_scale", VP),
        ("row_bytes", C.c_int), ("scale_per_row", C.c_int),
        ("trace", VP), ("done_counter", VP),
    ]


class CombineDesc(C.Structure):
    _fields_ = [
        ("combine", VP), ("topk_w", VP), ("topk_idx", VP), ("m2n_flag", VP),
        ("epoch", VP), ("done_counter", VP),
        ("T", C.c_int), ("H", C.c_int), ("K", C.c_int), ("combine_tokens", C.c_int), ("num_eg", C.c_int),
        ("scale", C.c_float),
        ("extra", VP), ("y", VP), ("residual", VP), ("norm_w", VP), ("normed", VP),
        ("eps", C.c_float), ("offset1", C.c_int),
        ("timeout_ns", C.c_ulonglong),
        ("status", VP),
        ("trace", VP),
    ]


_SIGNATURES = {
    "afd_grouped_gemm": (C.c_int, [C.POINTER(GroupedGemmDesc), VP]),
    "afd_rmsnorm": (C.c_int, [VP, VP, VP, VP, C.c_long, C.c_int, C.c_float, C.c_int, VP]),
    "afd_qk_norm_rope_store": (C.c_int, [VP, C.c_long, VP, VP, VP, VP, VP, VP, VP, C.c_int, C.c_int, C.c_int,
                                         C.c_int, C.c_int, C.c_float, C.c_int, C.c_long, VP, VP]),
    "afd_embedding": (C.c_int, [VP, VP, VP, C.c_int, C.c_int, C.c_int, C.c_int, VP]),
    "afd_silu_mul": (C.c_int, [VP, VP, C.c_long, C.c_int, VP]),
    "afd_cross_head_norm_rope_store": (C.c_int, [VP, C.c_long, VP, VP, VP, C.c_float, C.c_float, VP, VP, VP, VP, VP,
                                                 C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_float, C.c_int,
                                                 C.c_long, VP, VP]),
    "afd_qk_square_sums": (C.c_int, [VP, C.c_long, VP, C.c_int, C.c_int, C.c_int, VP]),
    "afd_grouped_topk_route": (C.c_int, [VP, VP, VP, VP, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                         C.c_float, C.c_int, VP]),
    "afd_shared_gate_mul": (C.c_int, [VP, VP, VP, C.c_int, C.c_int, VP]),
    "afd_sigmoid_gate_mul": (C.c_int, [VP, VP, C.c_long, C.c_long, C.c_int, VP]),
    "afd_topk_route": (C.c_int, [VP, VP, VP, VP, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                 C.c_float, C.c_int, VP]),
    "afd_decode_attention_strided": (C.c_int, [VP, C.c_long, VP, VP, VP, VP, VP, VP, C.c_int, C.c_int, C.c_int,
                                               C.c_int, C.c_int, C.c_int, C.c_int, C.c_long, C.c_int, C.c_float,
                                               VP, VP]),
    "afd_prefill_attention_varlen": (C.c_int, [VP, C.c_long, VP, VP, VP, VP, VP, VP, C.c_int, C.c_int, C.c_int, C.c_int,
                                               C.c_int, C.c_int, C.c_int, C.c_long, C.c_float, VP, VP]),
    "afd_argmax": (C.c_int, [VP, VP, C.c_int, C.c_int, C.c_long, C.c_int, VP, VP]),
    "afd_argmax_chunks": (C.c_int, [C.c_int]),
    "afd_tp_allgather_push": (C.c_int, [VP, VP]),
    "afd_tp_allgather_wait": (C.c_int, [VP, C.c_int, VP, C.c_ulonglong, VP, VP]),
    "afd_wait_flags_epoch": (C.c_int, [VP, C.c_int, VP, C.c_ulonglong, VP, VP]),
    "afd_sample": (C.c_int, [VP, C.c_long, C.c_int, C.c_int, C.c_int, VP, VP, VP, VP, VP, VP]),
    "afd_group_quant_fp8": (C.c_int, [VP, VP, VP, C.c_long, C.c_int, C.c_int, C.c_int, VP]),
    "afd_decode_attn_workspace_bytes": (C.c_long, [C.c_int] * 6),
    "afd_decode_attention": (C.c_int, [VP, VP, VP, VP, VP, VP, VP, C.c_int, C.c_int, C.c_int, C.c_int,
                                       C.c_int, C.c_int, C.c_int, C.c_long, C.c_int, C.c_float, VP, VP]),
    "afd_dispatch_push": (C.c_int, [C.POINTER(DispatchDesc), VP]),
    "afd_ag_route_dispatch": (C.c_int, [C.POINTER(RouteDispatchDesc), VP]),
    "afd_eg_group_gather": (C.c_int, [C.POINTER(GroupDesc), VP]),
    "afd_dispatch_direct": (C.c_int, [VP, VP, C.POINTER(DirectDesc), VP]),
    "afd_ag_route_direct": (C.c_int, [C.POINTER(RouteDirectDesc), VP]),
    "afd_eg_schedule": (C.c_int, [C.POINTER(ScheduleDesc), VP]),
    "afd_ag_combine": (C.c_int, [C.POINTER(CombineDesc), VP]),
    "afd_wait_flag": (C.c_int, [VP, C.c_uint, C.c_ulonglong, VP, VP]),
    "afd_set_flag": (C.c_int, [VP, C.c_uint, VP]),
    "afd_fabric_alloc": (C.c_int, [C.c_size_t, C.POINTER(VP), VP]),
    "afd_fabric_open": (C.c_int, [VP, C.POINTER(VP)]),
    "afd_fabric_close": (C.c_int, [VP]),
    "afd_fabric_free": (C.c_int, [VP]),
    "afd_device_alloc": (C.c_int, [C.c_size_t, C.POINTER(VP)]),
    "afd_can_access_peer": (C.c_int, [C.c_int, C.c_int, C.POINTER(C.c_int)]),
    "afd_memcpy_async": (C.c_int, [VP, VP, C.c_size_t, VP]),
    "afd_cuda_error_string": (C.c_char_p, [C.c_int]),
}


class KernelLibraryError(RuntimeError):
    pass


@lru_cache(maxsize=1)
def lib() -> C.CDLL:
    """Load the kernel library, building it first when the binary is absent."""
    import torch  # noqa: F401  (loads libcudart.so.12, which the kernel library links against)

    path = lib_path()
    if not path.exists():
        path = build_extension()
    handle = C.CDLL(str(path))
    for name, (res, args) in _SIGNATURES.items():
        fn = getattr(handle, name, None)
        if fn is None:
            continue  # optional symbols (later additions) are bound lazily
        fn.restype = res
        fn.argtypes = args
    return handle


# Kernel launches issued through this library since import (graph capture counts the
# launches recorded into the graph once; replays are accounted for by the caller).
LAUNCHES = {"count": 0}
_KERNELS_PER_CALL = {"eg_group_gather": 2, "argmax": 2, "gdn_decode": 2, "gdn_prefill": 3}


def check(code: int, what: str) -> None:
    if code == 0:
        LAUNCHES["count"] += _KERNELS_PER_CALL.get(what, 1)
        return
    if code > 0:
        msg = lib().afd_cuda_error_string(code).decode()
        raise KernelLibraryError(f"{what}: CUDA error {code}: {msg}")
    raise KernelLibraryError(f"{what}: invalid arguments (code {code})")


def ptr(t) -> int | None:
    """Device pointer of a tensor (None passes a null pointer)."""
    return None if t is None else t.data_ptr()


def cur_stream() -> int:
    import torch

    return torch.cuda.current_stream().cuda_stream
