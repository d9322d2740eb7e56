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


@pytest.mark.parametrize("dh", [64, 128])
def test_noalloc_decode_matches_workspace_decode_twice(dh):
    """dh 128 runs the tensor-core streaming kernel and its refold kernel, dh 64 the dp4a kernel
    with the last-split ticket merge; both take their partials from the shared buffer."""
    L = _lib.load()
    torch.manual_seed(dh)
    B, H, KVH, Lmax = 4, 32, 8, 3000
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


def _refused(B, H, KVH, dh, max_blocks):
    """True when the call is refused for its size.  Every buffer is real and sized for the shape,
    and every sequence is empty, so even a call that were accepted would read nothing it does not
    own (no key page is touched for an empty sequence, and no output row is written)."""
    L = _lib.load()
    q = torch.zeros((B, H, dh), dtype=torch.bfloat16, device="cuda")
    lens = torch.zeros(B, dtype=torch.int32, device="cuda")
    bt = torch.zeros((B, 8 * max_blocks), dtype=torch.int32, device="cuda")
    k8p = torch.zeros((1, KVH, 16, dh), dtype=torch.int8, device="cuda")
    v8p = torch.zeros((1, KVH, dh, 16), dtype=torch.int8, device="cuda")
    e = torch.zeros((B, KVH, max_blocks), dtype=torch.int32, device="cuda")
    e0 = torch.zeros((B, KVH), dtype=torch.int32, device="cuda")
    out = torch.zeros((B, H, dh), dtype=torch.bfloat16, device="cuda")
    rc = L.lssab8_decode_noalloc(q.data_ptr(), 2, _lib.i64x(q.stride()), B, H, KVH, dh, lens.data_ptr(), bt.data_ptr(),
                                 8 * max_blocks, 1, k8p.data_ptr(), v8p.data_ptr(), e.data_ptr(), e.data_ptr(),
                                 e0.data_ptr(), max_blocks, 4, 0, out.data_ptr(), 2, _lib.i64x(out.stride()), None)
    torch.cuda.synchronize()
    return rc == ESCRATCH


def test_noalloc_scratch_limit_is_exact():
    """The refusal rule is workspace_size - 256 > LSSAB8_NOALLOC_SCRATCH_BYTES (the 256 bytes are
    alignment slack the aligned buffer does not need).  max_blocks sizes the partials, whatever
    the sequences' lengths, so the largest accepted max_blocks is run on a short real lattice
    padded out to it (and must equal lssab8_decode), and the next one must be refused."""
    L = _lib.load()
    B, H, KVH, dh, Lmax = 16, 32, 8, 128, 300
    need = lambda mb: L.lssab8_decode_workspace_size(B, H, KVH, dh, mb) - 256
    mb = 1
    while need(mb + 1) <= SCRATCH_BYTES:
        mb += 1
    assert need(mb) <= SCRATCH_BYTES < need(mb + 1)
    assert _refused(B, H, KVH, dh, mb + 1)

    torch.manual_seed(5)
    k = torch.randn(B, KVH, Lmax, dh, device="cuda").to(torch.bfloat16)
    v = torch.randn(B, KVH, Lmax, dh, device="cuda").to(torch.bfloat16)
    lens = torch.randint(1, Lmax + 1, (B,), dtype=torch.int32, device="cuda")
    bt, npages = D.identity_pages(B, Lmax, k.device)
    kv = D.build_paged_kv(k, v, lens, bt, npages, sink=True)
    pad = lambda x, n: torch.cat([x, x.new_zeros(x.shape[:-1] + (n - x.shape[-1],))], dim=-1).contiguous()
    kv = D.PagedKV(k8p=kv.k8p, v8p=kv.v8p, ek=pad(kv.ek, mb), ev=pad(kv.ev, mb), ev0=kv.ev0,
                   block_table=pad(kv.block_table, 8 * mb), seq_lens=lens, max_blocks=mb, num_pages=npages, sink=True)
    q = torch.randn(B, H, dh, device="cuda").to(torch.bfloat16)
    ref = D.decode(q, kv)
    got = torch.full((B, H, dh), float("nan"), dtype=torch.bfloat16, device="cuda")
    a, st = _args(q, kv, got)
    _lib.check(L.lssab8_decode_noalloc(*a, st), "lssab8_decode_noalloc at the size limit")
    torch.cuda.synchronize()
    assert _lib.device_errors() == 0
    assert torch.equal(got.view(torch.int16), ref.view(torch.int16))


def test_noalloc_refuses_problems_larger_than_its_buffer():
    L = _lib.load()
    B, H, KVH, dh, max_blocks = 64, 64, 8, 128, 1024          # needs ~1 GiB of partials
    assert L.lssab8_decode_workspace_size(B, H, KVH, dh, max_blocks) > SCRATCH_BYTES
    assert _refused(B, H, KVH, dh, max_blocks)
    assert "scratch" in _lib.strerror(ESCRATCH)
