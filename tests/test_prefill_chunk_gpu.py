"""Block-aligned chunked prefill on an append-only lattice, bit for bit against the whole prefill
and against the pinned CPU oracle.

The reference's 128-aligned chunk invariance (reference/lssab8_selftest.py:292-317): the
quantisation of a prefix is the prefix of the quantisation, and every row of the prefix has a
bit-identical output.  So a chunk of query rows [T0, T1) computed against the lattice of keys
[0, T1) must equal rows [T0, T1) of the prefill of the whole sequence.  Each chunk here quantises
only its own query rows and the key prefix it needs, as an engine appending to a paged cache would.
"""
import numpy as np
import pytest
import torch

import oracle as O
from lockstep_b200 import attention as A
from lockstep_b200 import workloads as W

pytestmark = pytest.mark.gpu


def _bits(t):
    return t.float().cpu().numpy().view(np.uint32)


def _full_and_chunks(B, H, KVH, T, dh, cuts, sink, seed, oracle=False):
    q, k, v = W.prefill_inputs(B, H, KVH, T, dh, outliers=0.01, seed=seed)
    if oracle:                                  # the chunks against the oracle, not only each other
        ref = np.stack([O.attention(q[b], k[b], v[b], sink=sink).transpose(1, 0, 2) for b in range(B)])
    to = lambda x: torch.from_numpy(np.ascontiguousarray(x)).to(torch.bfloat16).cuda()
    qd, kd, vd = to(q), to(k), to(v)
    mode = 2 if sink else 0
    q8, eq = A.quant_rows(qd)
    k8, ek, _ = A.quant_blocks(kd, 0)
    v8, ev, ev0 = A.quant_blocks(vd, mode)
    full = A.prefill_lattice(q8, eq, k8, ek, v8, ev, ev0 if sink else None, T, out_dtype=torch.float32)
    bounds = list(cuts) + [T]
    for T0, T1 in zip(bounds[:-1], bounds[1:]):
        q8c, eqc = A.quant_rows(qd[:, :, T0:T1])
        k8p, ekp, _ = A.quant_blocks(kd[:, :, :T1], 0)
        v8p, evp, ev0p = A.quant_blocks(vd[:, :, :T1], mode)
        nfull = T1 // 128                                      # blocks the prefix completes
        assert torch.equal(k8p[:, :, :nfull * 128], k8[:, :, :nfull * 128])     # append-only lattice
        assert torch.equal(ekp[:, :, :nfull], ek[:, :, :nfull])
        assert torch.equal(evp[:, :, :nfull], ev[:, :, :nfull])
        out = A.prefill_chunk_lattice(q8c, eqc, k8p, ekp, v8p, evp, ev0p if sink else None, T0, T1,
                                      out_dtype=torch.float32)
        assert out.shape == (B, T1 - T0, H, dh)
        assert np.array_equal(_bits(out), _bits(full[:, T0:T1])), (T0, T1)
        if oracle:
            assert np.array_equal(_bits(out), np.ascontiguousarray(ref[:, T0:T1]).view(np.uint32)), (T0, T1)
    A.check_device_errors(torch.device("cuda:0"))


@pytest.mark.parametrize("sink", [False, True])
@pytest.mark.parametrize("dh", [128, 64])
def test_chunks_equal_whole_prefill(dh, sink):
    _full_and_chunks(2, 4, 2, 640, dh, (0, 128, 384, 512), sink, seed=3, oracle=(dh == 64))


def _s8_fixture():
    """The reference's own S8 inputs (reference/lssab8_selftest.py:292-317): 2 query heads and one
    kv head, dh 128, T 640, float32 draws of RandomState(11)."""
    T = 640
    g = np.random.RandomState(11)
    q = g.standard_normal((2, T, 128)).astype(np.float32)
    k = g.standard_normal((1, T, 128)).astype(np.float32)
    v = g.standard_normal((1, T, 128)).astype(np.float32)
    return q, k, v


@pytest.mark.parametrize("sink", [False, True])
def test_s8_fixture_chunks_equal_oracle(sink):
    """Each aligned chunk [T0, T1) of the S8 fixture, run on the lattice of [0, T1) from float32
    inputs with float32 outputs, equals rows [T0, T1) of the oracle's whole prefill, and the
    chunk at each S8 cut (128, 256, 384, 512) equals the prefill of that prefix (the selftest's
    statement)."""
    q, k, v = _s8_fixture()
    T = q.shape[1]
    ref = O.attention(q, k, v, sink=sink).transpose(1, 0, 2)            # [T, H, dh]
    qd, kd, vd = (torch.from_numpy(x).cuda()[None] for x in (q, k, v))
    mode = 2 if sink else 0
    for T0, T1 in ((0, 128), (128, 256), (256, 384), (384, 512), (512, 640), (0, 640), (256, 640)):
        q8c, eqc = A.quant_rows(qd[:, :, T0:T1])
        k8, ek, _ = A.quant_blocks(kd[:, :, :T1], 0)
        v8, ev, ev0 = A.quant_blocks(vd[:, :, :T1], mode)
        out = A.prefill_chunk_lattice(q8c, eqc, k8, ek, v8, ev, ev0 if sink else None, T0, T1,
                                      out_dtype=torch.float32)
        assert np.array_equal(_bits(out[0]), np.ascontiguousarray(ref[T0:T1]).view(np.uint32)), (T0, T1)
    for cut in (128, 256, 384, 512):
        part = O.attention(q[:, :cut], k[:, :cut], v[:, :cut], sink=sink).transpose(1, 0, 2)
        assert np.array_equal(part.view(np.uint32), np.ascontiguousarray(ref[:cut]).view(np.uint32)), cut
    A.check_device_errors(torch.device("cuda:0"))


@pytest.mark.parametrize("sink", [False, True])
def test_ragged_last_chunk(sink):
    # the last chunk ends inside a block: its trailing block is quantised over the present rows,
    # exactly as the whole prefill of that length does
    _full_and_chunks(1, 8, 2, 1000, 128, (0, 256, 768), sink, seed=4, oracle=True)


def test_chunk_rows_spanning_several_fold_segments():
    # T > 4096: rows of the last chunk fold more than 32 key blocks (segment -> row fold)
    _full_and_chunks(1, 2, 1, 4480, 128, (0, 4096), False, seed=5)


def test_unaligned_chunk_start_is_rejected():
    x8 = torch.zeros((1, 1, 256, 128), dtype=torch.int8, device="cuda")
    e = torch.zeros((1, 1, 2), dtype=torch.int32, device="cuda")
    with pytest.raises(ValueError):
        A.prefill_chunk_lattice(x8, e, x8, e, x8, e, None, 100, 300)
