"""The allocation-free decode entry point, called through the C ABI.

lssab8_decode_noalloc serves hosts that cannot give the library a workspace (an engine that
plans all device memory up front and passes each attention call only its inputs and outputs, or
a plugin host that owns every allocation).  It uses the library's fixed device scratch buffer
instead.  This test checks, on two calls in a row, that it returns exactly what lssab8_decode
returns with a caller workspace (bit-identical: the contract has no tolerance), and that a
problem too large for the buffer is refused with LSSAB8_ESCRATCH.  The file name makes pytest
collect it last; it also passes alone in a fresh process.
"""
import ctypes

import numpy as np
import pytest
import torch

from lockstep_b200 import _lib
from lockstep_b200 import decode as D

pytestmark = pytest.mark.gpu

ESCRATCH = 6
SCRATCH_BYTES = 48 << 20


def _args(q, kv, out):
    s = torch.cuda.current_stream().cuda_stream
    return (q.data_ptr(), 2, _lib.i64x(q.stride()), q.shape[0], q.shape[1], kv.KVH, kv.dh, kv.seq_lens.data_ptr(),
            kv.block_table.data_ptr(), kv.block_table.shape[1], kv.num_pages, kv.k8p.data_ptr(), kv.v8p.data_ptr(),
            kv.ek.data_ptr(), kv.ev.data_ptr(), kv.ev0.data_ptr(), kv.max_blocks, 4, int(kv.sink), out.data_ptr(), 2,
            _lib.i64x(out.stride())), s


def test_noalloc_decode_matches_workspace_decode_twice():
    L = _lib.load()
    torch.manual_seed(0)
    B, H, KVH, Lmax, dh = 4, 32, 8, 3000, 128
    k = torch.randn(B, KVH, Lmax, dh, device="cuda").to(torch.bfloat16)
    v = torch.randn(B, KVH, Lmax, dh, device="cuda").to(torch.bfloat16)
    lens = torch.tensor([3000, 1, 129, 2048], dtype=torch.int32, device="cuda")
    bt, npages = D.identity_pages(B, Lmax, k.device)
    for sink in (False, True):
        kv = D.build_paged_kv(k, v, lens, bt, npages, sink=sink)
        assert L.lssab8_decode_workspace_size(B, H, KVH, dh, kv.max_blocks) <= SCRATCH_BYTES
        for call in range(2):
            q = torch.randn(B, H, dh, device="cuda").to(torch.bfloat16)
            ref = torch.empty(B, H, dh, dtype=torch.bfloat16, device="cuda")
            got = torch.full((B, H, dh), float("nan"), dtype=torch.bfloat16, device="cuda")
            nbytes = L.lssab8_decode_workspace_size(B, H, KVH, dh, kv.max_blocks)
            ws = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
            a, s = _args(q, kv, ref)
            _lib.check(L.lssab8_decode(*a, ws.data_ptr(), ws.numel(), s), "lssab8_decode")
            a, s = _args(q, kv, got)
            _lib.check(L.lssab8_decode_noalloc(*a, s), "lssab8_decode_noalloc")
            torch.cuda.synchronize()
            assert _lib.device_errors() == 0
            assert torch.equal(got.view(torch.int16), ref.view(torch.int16)), (sink, call)


def test_noalloc_refuses_problems_larger_than_its_buffer():
    L = _lib.load()
    B, H, KVH, dh, max_blocks = 64, 64, 8, 128, 1024          # needs ~1 GiB of partials
    assert L.lssab8_decode_workspace_size(B, H, KVH, dh, max_blocks) > SCRATCH_BYTES
    z = torch.zeros(16, dtype=torch.int32, device="cuda")
    p = z.data_ptr()
    rc = L.lssab8_decode_noalloc(p, 2, _lib.i64x([H * dh, dh, 1]), B, H, KVH, dh, p, p, 8 * max_blocks, 1, p, p, p, p,
                                 p, max_blocks, 4, 0, p, 2, _lib.i64x([H * dh, dh, 1]), None)
    assert rc == ESCRATCH
    assert "scratch" in _lib.strerror(rc)
