"""The append-only paged lattice (lssab8_kv_append) on the GPU.

A lattice is built the way an engine builds it: the prompt appended in one call, then one token
per decode step (and a few multi-token appends crossing block boundaries).  After every append
the lattice must equal a fresh lssab8_decode_prep_kv over the same tokens -- values, exponents and
the sink exponent, bit for bit -- and decode on it must equal the oracle's row.  Blocks complete
before an append are never rewritten (a planted sentinel in a complete block's exponent survives).
The float cache is dense, and paged with the lattice's own block table."""
import numpy as np
import pytest
import torch

import oracle as O
from lockstep_b200 import decode as D
from lockstep_b200 import workloads as W

pytestmark = pytest.mark.gpu


def _same(a, b):
    for name in ("k8p", "v8p", "ek", "ev"):
        assert torch.equal(getattr(a, name), getattr(b, name)), name
    if a.sink:
        assert torch.equal(a.ev0, b.ev0)


def _fresh(keys, values, lens, bt, npages, sink):
    return D.build_paged_kv(keys, values, lens, bt, npages, sink=sink)


@pytest.mark.parametrize("sink", [False, True])
@pytest.mark.parametrize("dh", [128, 64])
def test_prompt_then_token_appends_equal_fresh_lattice(sink, dh):
    B, H, KVH, Lcap = 3, 8, 2, 700
    rng = np.random.default_rng(dh + sink)
    k = W.bf16_round(rng.standard_normal((B, KVH, Lcap, dh)).astype(np.float32))
    v = W.bf16_round(rng.standard_normal((B, KVH, Lcap, dh)).astype(np.float32))
    q = W.bf16_round(rng.standard_normal((B, H, dh)).astype(np.float32))
    kd = torch.from_numpy(k).to(torch.bfloat16).cuda()
    vd = torch.from_numpy(v).to(torch.bfloat16).cuda()
    qd = torch.from_numpy(q).to(torch.bfloat16).cuda()
    bt, npages = W.page_table(np.full(B, Lcap), 16, seed=3)
    bt = torch.tensor(bt).cuda()
    kv = D.empty_paged_kv(B, KVH, dh, Lcap, bt, npages, sink=sink)
    lens = np.array([126, 1, 300])                              # the prompts
    steps = [1] * 5 + [128, 1, 130, 2]                          # decode tokens, then chunks across blocks
    for i, n in enumerate([0] + steps):
        lens = lens + n if i else lens
        lt = torch.tensor(lens, dtype=torch.int32).cuda()
        D.append_kv(kv, kd, vd, lt)
        fresh = _fresh(kd, vd, lt, bt, npages, sink)
        _same(kv, fresh)
        got = D.decode(qd, kv, split_blocks=2)
        for b in range(B):
            L = int(lens[b])
            ref = O.f32_to_bf16_bits(O.decode_rows(q[b], k[b, :, :L], v[b, :, :L], sink=sink))
            assert np.array_equal(got[b].cpu().view(torch.int16).numpy().view(np.uint16), ref), (i, b)


def test_complete_blocks_are_not_rewritten_and_paged_source():
    B, KVH, dh, Lcap = 2, 2, 128, 600
    g = torch.Generator(device="cuda").manual_seed(1)
    kd = torch.randn(B, KVH, Lcap, dh, device="cuda", generator=g).to(torch.bfloat16)
    vd = torch.randn(B, KVH, Lcap, dh, device="cuda", generator=g).to(torch.bfloat16)
    bt, npages = W.page_table(np.full(B, Lcap), 16, seed=4)
    bt = torch.tensor(bt).cuda()
    kv = D.empty_paged_kv(B, KVH, dh, Lcap, bt, npages)
    D.append_kv(kv, kd, vd, torch.tensor([300, 257], dtype=torch.int32).cuda())
    kv.ek[:, :, 0] = 99                                          # a sentinel in complete block 0
    D.append_kv(kv, kd, vd, torch.tensor([301, 258], dtype=torch.int32).cuda())
    assert (kv.ek[:, :, 0] == 99).all()                          # untouched: block 0 was complete
    # the same tokens from a paged float cache [pages, 16, KVH, dh] laid out by the same table
    kc = torch.zeros((npages, 16, KVH, dh), dtype=torch.bfloat16, device="cuda")
    vc = torch.zeros_like(kc)
    for b in range(B):
        for p in range(Lcap // 16 + 1):
            if p < bt.shape[1] and int(bt[b, p]) >= 0 and p * 16 < Lcap:
                n = min(16, Lcap - p * 16)
                kc[int(bt[b, p]), :n] = kd[b, :, p * 16:p * 16 + n].transpose(0, 1)
                vc[int(bt[b, p]), :n] = vd[b, :, p * 16:p * 16 + n].transpose(0, 1)
    kv2 = D.empty_paged_kv(B, KVH, dh, Lcap, bt, npages)
    lt = torch.tensor([301, 258], dtype=torch.int32).cuda()
    D.append_kv(kv2, kc, vc, lt, src_block_table=bt)
    _same(kv2, _fresh(kd, vd, lt, bt, npages, False))
