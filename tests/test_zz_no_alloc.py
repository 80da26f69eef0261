"""The allocation-free decode-attention entry point, called through its exported C symbol.

Some users of the kernel library cannot allocate device memory when they call it (all HBM
already belongs to their KV pool, or their decode loop forbids cudaMalloc). For them the
library offers ``afd_decode_attention_noalloc``, which keeps the split-KV partial results in
an array inside the library image. This test checks that it returns what the regular entry
point (caller-provided workspace) returns, on calls in a row that differ in inputs, batch and
split count - the later calls reuse the array with the first call's leftovers in it - and that an oversized request
is refused with a clear error instead of being launched."""
import ctypes as C
import math

import pytest
import torch

from fastafd_b200 import ops
from fastafd_b200.ops._lib import lib

pytestmark = pytest.mark.gpu
DEV = "cuda"
VP = C.c_void_p


def _entry():
    fn = lib().afd_decode_attention_noalloc
    fn.restype = C.c_int
    fn.argtypes = [VP, VP, VP, VP, VP, VP, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                   C.c_long, C.c_int, C.c_float, VP, VP]
    return fn


def _case(seed, B, Hq, Hkv, D, page, lens):
    g = torch.Generator().manual_seed(seed)
    max_pages = (max(lens) + page - 1) // page + 1
    n_pages = B * max_pages + 2
    pt = torch.randperm(n_pages, generator=g)[:B * max_pages].view(B, max_pages).to(torch.int32).to(DEV)
    kc = torch.randn(n_pages * page, Hkv, D, generator=g).to(torch.bfloat16).to(DEV)
    vc = torch.randn(n_pages * page, Hkv, D, generator=g).to(torch.bfloat16).to(DEV)
    q = torch.randn(B, Hq, D, generator=g).to(torch.bfloat16).to(DEV)
    return q, kc, vc, pt, torch.tensor(lens, dtype=torch.int32, device=DEV)


def test_noalloc_entry_matches_regular_entry_twice():
    fn = _entry()
    Hq, Hkv, D, page = 32, 4, 128, 16
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    # the calls differ in batch and in splits: the second and third find the first one's partial
    # results in the array, but their arrival counters at the same fixed place, left at zero
    for seed, lens, splits in ((0, [700, 33, 1500, 257], 3), (1, [64, 1200], 5), (2, [900, 5, 2000, 640, 31], 2)):
        q, kc, vc, pt, sl = _case(seed, len(lens), Hq, Hkv, D, page, lens)
        expect = ops.decode_attention(q, kc, vc, pt, sl, Hq, Hkv, D, 1, page, 1 / math.sqrt(D), splits=splits)
        out = torch.empty_like(q)
        stream = torch.cuda.current_stream().cuda_stream
        rc = fn(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), pt.data_ptr(), sl.data_ptr(), out.data_ptr(), len(lens),
                Hq, Hkv, D, 1, page, pt.shape[1], kc.shape[0], splits, 1 / math.sqrt(D), status.data_ptr(), stream)
        assert rc == 0, lib().afd_noalloc_strerror(rc)
        torch.cuda.synchronize()
        assert int(status) == 0
        torch.testing.assert_close(out.float(), expect.float(), atol=2e-2, rtol=2e-2)


def test_noalloc_entry_rejects_oversized_request():
    fn = _entry()
    need = lib().afd_decode_attention_noalloc_need
    need.restype = C.c_long
    need.argtypes = [C.c_int] * 6
    assert need(4096, 64, 4, 1, 128, 32) > 8 * 1024 * 1024
    rc = fn(None, None, None, None, None, None, 4096, 64, 4, 128, 1, 16, 8, 128, 32, 0.1, None, None)
    assert rc == -20
    msg = lib().afd_noalloc_strerror
    msg.restype = C.c_char_p
    assert b"scratch" in msg(rc)
