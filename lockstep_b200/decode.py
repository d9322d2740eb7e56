"""LSSA-B8 / B9.1 split-KV decode over a paged int8 KV lattice (host layer over the C ABI).

Contract v2: a generated row uses LSSA-B8 too, so the decode output for a sequence of L keys is
bit-identical to row L-1 of the prefill over the same keys (reference/lssab8_selftest.py:320-336).
The decode kernel reads the int8 lattice once (the HBM-bound part) and merges its split-KV
block partials in the contract's ascending order (reference/lssab8_golden.py:350-394).

Lattice layout (16-key pages; KB = 128 keys = 8 pages per contract block):
    k8p [num_pages, KVH, 16, dh]   int8 key rows
    v8p [num_pages, KVH, dh, 16]   int8 values, transposed within the page
    ek, ev [B, KVH, max_blocks]    int32 per logical 128-key block; ev0 [B, KVH] (sink)
    block_table [B, max_pages]     int32 physical page of each logical page (-1 = none)
"""
from dataclasses import dataclass

import torch

from . import _lib
from . import attention as _A

PAGE = 16
KB = 128


@dataclass
class PagedKV:
    k8p: torch.Tensor
    v8p: torch.Tensor
    ek: torch.Tensor
    ev: torch.Tensor
    ev0: torch.Tensor
    block_table: torch.Tensor
    seq_lens: torch.Tensor
    max_blocks: int
    num_pages: int
    sink: bool

    @property
    def KVH(self):
        return self.k8p.shape[1]

    @property
    def dh(self):
        return self.k8p.shape[3]

    def nbytes_lattice(self, lengths):
        """Algorithmic bytes of one decode step's lattice read: int8 K and V of every present key."""
        return int(sum(int(L) for L in lengths)) * self.KVH * self.dh * 2


def alloc_paged(B, KVH, dh, max_len, num_pages, device, sink=False):
    max_blocks = (max_len + KB - 1) // KB
    return dict(
        k8p=torch.zeros((num_pages, KVH, PAGE, dh), dtype=torch.int8, device=device),
        v8p=torch.zeros((num_pages, KVH, dh, PAGE), dtype=torch.int8, device=device),
        ek=torch.zeros((B, KVH, max_blocks), dtype=torch.int32, device=device),
        ev=torch.zeros((B, KVH, max_blocks), dtype=torch.int32, device=device),
        ev0=torch.zeros((B, KVH), dtype=torch.int32, device=device),
        max_blocks=max_blocks,
    )


def build_paged_kv(keys, values, seq_lens, block_table, num_pages, sink=False, cu_seqlens=None, check=True,
                   out=None):
    """Quantise K/V into a paged lattice.

    keys/values: dense [B, KVH, L, dh] (then cu_seqlens is None and seq_lens[b] <= L), or flat
    [N, KVH, dh] with cu_seqlens [B+1] (int64, host or device) giving each sequence's first token.
    seq_lens [B] int32, block_table [B, max_pages] int32 (CUDA tensors).  out: an existing
    PagedKV of the same B, KVH, dh, num_pages and sink with room for the longest sequence, whose
    buffers are rewritten in place (its pages outside the sequences keep their contents) instead of
    allocating a new lattice; it is returned with the new seq_lens and block_table."""
    dev = _A._require_cuda(keys, values, seq_lens, block_table)
    if keys.dtype != values.dtype or keys.shape != values.shape:
        raise ValueError("keys and values must share shape and dtype")
    B = seq_lens.numel()
    if cu_seqlens is None:
        if keys.dim() != 4 or keys.shape[0] != B:
            raise ValueError("dense keys must be [B, KVH, L, dh]")
        _, KVH, Lmax, dh = keys.shape
        s = keys.stride()
        seq_off = torch.arange(B, dtype=torch.int64) * s[0]
        st, sg, sc = s[2], s[1], s[3]
    else:
        if keys.dim() != 3:
            raise ValueError("flat keys must be [N, KVH, dh]")
        _, KVH, dh = keys.shape
        s = keys.stride()
        cu = torch.as_tensor(cu_seqlens, dtype=torch.int64).cpu()
        seq_off = cu[:B] * s[0]
        st, sg, sc = s[0], s[1], s[2]
        Lmax = int((cu[1:B + 1] - cu[:B]).max())
    if values.stride() != keys.stride():
        raise ValueError("keys and values must share strides")
    max_pages = block_table.shape[1]
    Lcap = max(int(Lmax), 1)
    if out is None:
        a = alloc_paged(B, KVH, dh, Lcap, num_pages, dev, sink)
    else:
        if (out.ek.shape[0] != B or out.KVH != KVH or out.dh != dh or out.num_pages != num_pages or
                out.sink != bool(sink) or out.max_blocks * KB < Lcap):
            raise ValueError("out: a lattice of another shape")
        a = dict(k8p=out.k8p, v8p=out.v8p, ek=out.ek, ev=out.ev, ev0=out.ev0, max_blocks=out.max_blocks)
    seq_off = seq_off.to(dev)
    with torch.cuda.device(dev):
        _lib.check(_lib.load().lssab8_decode_prep_kv(
            keys.data_ptr(), values.data_ptr(), _A.dtype_code(keys.dtype), B, KVH, dh, seq_lens.data_ptr(),
            seq_off.data_ptr(), st, sg, sc, block_table.data_ptr(), max_pages, a["max_blocks"], num_pages,
            int(bool(sink)), a["k8p"].data_ptr(), a["v8p"].data_ptr(), a["ek"].data_ptr(), a["ev"].data_ptr(),
            a["ev0"].data_ptr(), _A._stream_handle(dev)), "lssab8_decode_prep_kv")
    if check:
        _A.check_device_errors(dev)
    return PagedKV(k8p=a["k8p"], v8p=a["v8p"], ek=a["ek"], ev=a["ev"], ev0=a["ev0"], block_table=block_table,
                   seq_lens=seq_lens, max_blocks=a["max_blocks"], num_pages=num_pages, sink=bool(sink))


def empty_paged_kv(B, KVH, dh, max_len, block_table, num_pages, sink=False):
    """An empty lattice (every sequence of length 0) with room for max_len tokens per sequence,
    to be filled by append_kv.  block_table [B, max_pages] int32 (CUDA)."""
    dev = block_table.device
    a = alloc_paged(B, KVH, dh, max_len, num_pages, dev, sink)
    return PagedKV(k8p=a["k8p"], v8p=a["v8p"], ek=a["ek"], ev=a["ev"], ev0=a["ev0"], block_table=block_table,
                   seq_lens=torch.zeros(B, dtype=torch.int32, device=dev), max_blocks=a["max_blocks"],
                   num_pages=num_pages, sink=bool(sink))


def append_kv(kv, keys, values, new_lens, src_block_table=None, check=True):
    """Append-only lattice update (lssab8_kv_append): the sequences grew from kv.seq_lens to
    new_lens [B] int32 tokens.  keys / values hold every token so far, either dense
    [B, KVH, Lcap, dh] or, with src_block_table [B, max_pages], paged [num_pages, 16, KVH, dh]
    (the engine's float cache).  Blocks complete before the append are not rewritten; the open
    block and the new ones are quantised over their present rows, so the lattice equals a fresh
    build_paged_kv over new_lens bit for bit.  Updates kv.seq_lens in place and returns kv."""
    dev = _A._require_cuda(keys, values, new_lens, kv.k8p)
    if keys.dtype != values.dtype or keys.shape != values.shape or keys.stride() != values.stride():
        raise ValueError("keys and values must share shape, strides and dtype")
    B = kv.seq_lens.numel()
    new_lens = new_lens.to(device=dev, dtype=torch.int32).contiguous()
    if src_block_table is None:
        if keys.dim() != 4 or keys.shape[0] != B:
            raise ValueError("dense keys must be [B, KVH, Lcap, dh]")
        s = keys.stride()
        seq_off = (torch.arange(B, dtype=torch.int64) * s[0]).to(dev)
        st, sg, sc, ps, sbt = s[2], s[1], s[3], 0, None
    else:
        if keys.dim() != 4 or keys.shape[1] != PAGE:
            raise ValueError("paged keys must be [num_pages, 16, KVH, dh]")
        if keys.shape[0] < kv.num_pages:
            raise ValueError("the paged float cache must hold the lattice's num_pages pages (its page ids are "
                             "checked against num_pages)")
        s = keys.stride()
        seq_off, st, sg, sc, ps, sbt = None, s[1], s[2], s[3], s[0], src_block_table
    if sc != 1:
        raise ValueError("the channel dimension must be contiguous")
    start = kv.seq_lens.clone()
    with torch.cuda.device(dev):
        _lib.check(_lib.load().lssab8_kv_append(
            keys.data_ptr(), values.data_ptr(), _A.dtype_code(keys.dtype), B, kv.KVH, kv.dh, new_lens.data_ptr(),
            start.data_ptr(), None if seq_off is None else seq_off.data_ptr(), st, sg,
            None if sbt is None else sbt.data_ptr(), ps, kv.block_table.data_ptr(), kv.block_table.shape[1],
            kv.max_blocks, kv.num_pages, int(kv.sink), kv.k8p.data_ptr(), kv.v8p.data_ptr(), kv.ek.data_ptr(),
            kv.ev.data_ptr(), kv.ev0.data_ptr(), _A._stream_handle(dev)), "lssab8_kv_append")
    kv.seq_lens.copy_(new_lens)
    if check:
        _A.check_device_errors(dev)
    return kv


def identity_pages(B, L, device):
    """Block table of a contiguous cache: sequence b owns pages [b*P, (b+1)*P), P = ceil(L/16)."""
    P = (L + PAGE - 1) // PAGE
    bt = torch.arange(B * P, dtype=torch.int32, device=device).view(B, P)
    return bt, B * P


def contiguous_kv(keys, values, sink=False, check=True, out=None):
    """Lattice of a dense cache keys/values [B, KVH, L, dh] (every sequence of length L); out: a
    lattice from an earlier call of the same shape, rewritten in place."""
    B, KVH, L, dh = keys.shape
    if out is not None:
        bt, npages, seq_lens = out.block_table, out.num_pages, out.seq_lens
    else:
        bt, npages = identity_pages(B, L, keys.device)
        seq_lens = torch.full((B,), L, dtype=torch.int32, device=keys.device)
    return build_paged_kv(keys, values, seq_lens, bt, npages, sink=sink, check=check, out=out)


def decode(q, kv, split_blocks=4, out=None, out_dtype=None, check=True):
    """One decode step: q [B, H, dh] -> out [B, H, dh] (default q.dtype).

    split_blocks = 128-key blocks per split (config 3: 64 blocks in 16 splits -> 4)."""
    dev = _A._require_cuda(q, kv.k8p)
    B, H, dh = q.shape
    if dh != kv.dh or kv.seq_lens.numel() != B:
        raise ValueError("query does not match the lattice")
    if out is None:
        out = torch.empty((B, H, dh), dtype=out_dtype or q.dtype, device=dev)
    L = _lib.load()
    nbytes = L.lssab8_decode_workspace_size(B, H, kv.KVH, dh, kv.max_blocks)
    if nbytes == 0:
        raise ValueError("unsupported decode shape")
    ws = _A.workspace(dev, nbytes)
    with torch.cuda.device(dev):
        _lib.check(L.lssab8_decode(
            q.data_ptr(), _A.dtype_code(q.dtype), _lib.i64x(q.stride()), B, H, kv.KVH, dh, kv.seq_lens.data_ptr(),
            kv.block_table.data_ptr(), kv.block_table.shape[1], kv.num_pages, kv.k8p.data_ptr(), kv.v8p.data_ptr(),
            kv.ek.data_ptr(), kv.ev.data_ptr(), kv.ev0.data_ptr(), kv.max_blocks, int(split_blocks), int(kv.sink),
            out.data_ptr(), _A.dtype_code(out.dtype), _lib.i64x(out.stride()), ws.data_ptr(), ws.numel(),
            _A._stream_handle(dev)), "lssab8_decode")
    if check:
        _A.check_device_errors(dev)
    return out
