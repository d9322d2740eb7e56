"""The serving-engine seam: one attention call per layer and engine step, over a paged float KV
cache, with prompt rows and generated rows routed by the scheduler's flag.

The reference's engine is a vLLM plugin that registers a custom attention backend
(paper/main.tex:846-860): the scheduler's is_prefilling flag -- never the number of query rows --
decides whether a sequence's rows in a step are prompt rows (docs/SPEC.md:88-93), prompt chunks
start on 128-token boundaries (a scheduler hook; the 128-aligned chunk invariance,
reference/lssab8_selftest.py:292-317, makes each chunk's rows equal the whole prefill's), and
generated rows are LSSA-B8 rows too (contract v2).  This module is that backend's forward pass on
this library, in the engine's own terms:

  * the engine keeps its float K/V cache in 16-token pages, [num_pages, 16, KVH, dh], addressed
    by its block table [nseq, max_pages] and written at slot_mapping (page * 16 + row);
  * LatticeLayer keeps the int8 lattice that shadows that cache for one layer: pages with the same
    ids as the engine's (so the engine's block table addresses both), and per-sequence block
    exponents in slots keyed by the sequence's first page, the identity a sequence keeps across
    steps (as the reference's row verifier keys it, tools/verify_rows.py:63-104);
  * Lssab8Attention.forward(layer, query, key, value, k_cache, v_cache, meta) stores the step's new
    keys and values in the float cache, appends them to the lattice (lssab8_kv_append: only the
    open block and new blocks are quantised), then runs each prompt chunk through the block-aligned
    chunked prefill and every generated row through one split-KV decode call.

lockstep_b200.vllm_backend wraps this forward pass as a vLLM attention backend: its metadata
builder supplies query_start_loc, seq_lens, block_table, slot_mapping and the scheduler's prefill
flags; the 128-aligned chunk boundaries are the scheduler's to keep.
"""
from dataclasses import dataclass

import torch

from . import attention as A
from . import decode as D

PAGE = 16
KB = 128


@dataclass
class StepMeta:
    """One engine step: nseq sequences, ntok new tokens in sequence order.

    query_start_loc [nseq + 1] (host ints): sequence i's new tokens are rows [qsl[i], qsl[i+1]);
    seq_lens [nseq] (host ints): each sequence's length after this step; block_table
    [nseq, max_pages] int32 (CUDA): the pages of each sequence; slot_mapping [ntok] int64 (CUDA):
    page * 16 + row of each new token; is_prefill [nseq] (host bools): the scheduler's flag."""
    query_start_loc: list
    seq_lens: list
    block_table: torch.Tensor
    slot_mapping: torch.Tensor
    is_prefill: list


class LatticeLayer:
    """The int8 lattice of one layer: pages shared with the engine's float cache page ids, block
    exponents per sequence slot (keyed by the sequence's first page)."""

    def __init__(self, num_pages, KVH, dh, max_len, max_seqs, sink, device):
        self.KVH, self.dh, self.sink = KVH, dh, bool(sink)
        self.max_blocks = (max_len + KB - 1) // KB
        self.max_pages = self.max_blocks * 8
        self.num_pages = num_pages
        self.k8p = torch.zeros((num_pages, KVH, PAGE, dh), dtype=torch.int8, device=device)
        self.v8p = torch.zeros((num_pages, KVH, dh, PAGE), dtype=torch.int8, device=device)
        self.ek = torch.zeros((max_seqs, KVH, self.max_blocks), dtype=torch.int32, device=device)
        self.ev = torch.zeros_like(self.ek)
        self.ev0 = torch.zeros((max_seqs, KVH), dtype=torch.int32, device=device)
        self.lens = [0] * max_seqs
        self.slot_of = {}                                 # first page -> slot
        self.last_use = [0] * max_seqs                    # step of the slot's last use
        self.step = 0

    def slots(self, first_pages, lens_before):
        """Slots of the step's sequences.  A sequence seen for the first time (its length before
        the step is 0) takes a free slot, or the least recently used one of a sequence not in this
        step (an engine that never calls release() reuses its finished sequences' slots this way).
        A sequence that continues (length before > 0) must still hold its slot: if it was taken,
        its block exponents are gone and the step is refused."""
        self.step += 1
        out = []
        for fp, l0 in zip(first_pages, lens_before):
            s = self.slot_of.get(fp)
            if s is None:
                if l0 != 0:
                    raise RuntimeError("the sequence with first page %d continues at length %d, but its lattice "
                                       "slot was reused (more live sequences than slots)" % (fp, l0))
                s = self._take_slot()
                self.slot_of[fp] = s
            if l0 == 0:
                self.lens[s] = 0                          # a new sequence (possibly on a reused first page)
            self.last_use[s] = self.step
            out.append(s)
        return out

    def _take_slot(self):
        used = set(self.slot_of.values())
        for i in range(len(self.lens)):
            if i not in used:
                return i
        idle = [i for i in range(len(self.lens)) if self.last_use[i] < self.step]
        if not idle:
            raise RuntimeError("more sequences in one step than lattice slots")
        victim = min(idle, key=lambda i: self.last_use[i])
        for fp, s in list(self.slot_of.items()):
            if s == victim:
                del self.slot_of[fp]
        return victim

    def release(self, first_page):
        """Forget a finished sequence (the engine frees its pages)."""
        s = self.slot_of.pop(first_page, None)
        if s is not None:
            self.lens[s] = 0


class Lssab8Attention:
    """LSSA-B8 (sink=False) / B9.1 sink_alone (sink=True) attention for a paged serving engine."""

    def __init__(self, num_heads, num_kv_heads, head_size, num_pages, max_len, max_seqs, num_layers=1, sink=False,
                 device=None):
        if num_heads % num_kv_heads:
            raise ValueError("query heads must be a multiple of kv heads")
        self.H, self.KVH, self.dh = num_heads, num_kv_heads, head_size
        self.sink = bool(sink)
        dev = torch.device("cuda", torch.cuda.current_device()) if device is None else device
        self.layers = [LatticeLayer(num_pages, num_kv_heads, head_size, max_len, max_seqs, sink, dev)
                       for _ in range(num_layers)]

    def forward(self, layer, query, key, value, k_cache, v_cache, meta, out=None):
        """query [ntok, H, dh], key / value [ntok, KVH, dh] (this step's new tokens), k_cache /
        v_cache [num_pages, 16, KVH, dh] (the engine's float cache; rows and channels contiguous,
        any page stride) -> out [ntok, H, dh] in
        query.dtype.  Prompt chunks must start on a multiple of 128 tokens."""
        st = self.layers[layer]
        dev = query.device
        nseq = len(meta.seq_lens)
        qsl = [int(x) for x in meta.query_start_loc]
        lens = [int(x) for x in meta.seq_lens]
        qlen = [qsl[i + 1] - qsl[i] for i in range(nseq)]
        before = [lens[i] - qlen[i] for i in range(nseq)]
        if out is None:
            out = torch.empty_like(query)
        # 1. the step's keys and values into the engine's float cache (by page and row, so a cache
        #    whose pages are strided -- K and V interleaved per page -- is written in place)
        page, row = meta.slot_mapping // PAGE, meta.slot_mapping % PAGE
        k_cache[page, row] = key.to(k_cache.dtype)
        v_cache[page, row] = value.to(v_cache.dtype)
        # 2. the lattice: the open block and new blocks of every sequence, from the float cache
        bt = meta.block_table.to(device=dev, dtype=torch.int32)
        if bt.shape[1] < st.max_pages:
            bt = torch.cat([bt, bt.new_full((nseq, st.max_pages - bt.shape[1]), -1)], 1)
        bt = bt[:, :st.max_pages].contiguous()
        first = [int(x) for x in bt[:, 0].tolist()]
        slots = st.slots(first, before)
        sidx = torch.tensor(slots, dtype=torch.long, device=dev)
        kv = D.PagedKV(k8p=st.k8p, v8p=st.v8p, ek=st.ek[sidx].contiguous(), ev=st.ev[sidx].contiguous(),
                       ev0=st.ev0[sidx].contiguous(), block_table=bt,
                       seq_lens=torch.tensor(before, dtype=torch.int32, device=dev), max_blocks=st.max_blocks,
                       num_pages=st.num_pages, sink=self.sink)
        D.append_kv(kv, k_cache, v_cache, torch.tensor(lens, dtype=torch.int32, device=dev), src_block_table=bt)
        st.ek[sidx], st.ev[sidx], st.ev0[sidx] = kv.ek, kv.ev, kv.ev0
        for s, L in zip(slots, lens):
            st.lens[s] = L
        # 3. prompt rows: block-aligned chunks of the causal prefill
        for i in range(nseq):
            if not meta.is_prefill[i] or qlen[i] == 0:
                continue
            T0, T = before[i], lens[i]
            if T0 % KB:
                raise ValueError("prompt chunk of sequence %d starts at %d, not a multiple of %d (the scheduler's "
                                 "chunk alignment)" % (i, T0, KB))
            out[qsl[i]:qsl[i + 1]] = self._prompt_rows(query[qsl[i]:qsl[i + 1]], k_cache, v_cache, bt[i], T0, T)
        # 4. generated rows: one split-KV decode over the lattice for every one-row sequence
        gen = [i for i in range(nseq) if not meta.is_prefill[i] and qlen[i] > 0]
        if any(qlen[i] != 1 for i in gen):
            raise NotImplementedError("generated steps of more than one row (speculative tokens) are not routed")
        if gen:
            gi = torch.tensor(gen, dtype=torch.long, device=dev)
            rows = torch.tensor([qsl[i] for i in gen], dtype=torch.long, device=dev)
            dkv = D.PagedKV(k8p=st.k8p, v8p=st.v8p, ek=kv.ek[gi].contiguous(), ev=kv.ev[gi].contiguous(),
                            ev0=kv.ev0[gi].contiguous(), block_table=bt[gi].contiguous(),
                            seq_lens=torch.tensor([lens[i] for i in gen], dtype=torch.int32, device=dev),
                            max_blocks=st.max_blocks, num_pages=st.num_pages, sink=self.sink)
            out[rows] = D.decode(query[rows].contiguous(), dkv, out_dtype=query.dtype)
        return out

    def _prompt_rows(self, q, k_cache, v_cache, bt_row, T0, T):
        """Rows [T0, T) of one sequence's causal prefill: the chunk's queries against the lattice of
        keys [0, T), gathered from the paged float cache."""
        npg = (T + PAGE - 1) // PAGE
        pages = bt_row[:npg].long()
        kk = k_cache[pages].reshape(npg * PAGE, self.KVH, self.dh)[:T].transpose(0, 1)[None]
        vv = v_cache[pages].reshape(npg * PAGE, self.KVH, self.dh)[:T].transpose(0, 1)[None]
        q8, eq = A.quant_rows(q.transpose(0, 1)[None])
        k8, ek, _ = A.quant_blocks(kk, 0)
        v8, ev, ev0 = A.quant_blocks(vv, 2 if self.sink else 0)
        o = A.prefill_chunk_lattice(q8, eq, k8, ek, v8, ev, ev0 if self.sink else None, T0, T, out_dtype=q.dtype)
        return o[0]
