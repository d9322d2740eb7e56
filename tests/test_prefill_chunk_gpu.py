"""Block-aligned chunked prefill on an append-only lattice, bit for bit against the whole prefill.

The reference's 128-aligned chunk invariance (reference/lssab8_selftest.py:292-317): the
quantisation of a prefix is the prefix of the quantisation, and every row of the prefix has a
bit-identical output.  So a chunk of query rows [T0, T1) computed against the lattice of keys
[0, T1) must equal rows [T0, T1) of the prefill of the whole sequence.  Each chunk here quantises
only its own query rows and the key prefix it needs, as an engine appending to a paged cache would.
"""
import numpy as np
import pytest
import torch

from lockstep_b200 import attention as A
from lockstep_b200 import workloads as W

pytestmark = pytest.mark.gpu


def _bits(t):
    return t.float().cpu().numpy().view(np.uint32)


def _full_and_chunks(B, H, KVH, T, dh, cuts, sink, seed):
    q, k, v = W.prefill_inputs(B, H, KVH, T, dh, outliers=0.01, seed=seed)
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
    A.check_device_errors(torch.device("cuda:0"))


@pytest.mark.parametrize("sink", [False, True])
@pytest.mark.parametrize("dh", [128, 64])
def test_chunks_equal_whole_prefill(dh, sink):
    _full_and_chunks(2, 4, 2, 640, dh, (0, 128, 384, 512), sink, seed=3)


@pytest.mark.parametrize("sink", [False, True])
def test_ragged_last_chunk(sink):
    # the last chunk ends inside a block: its trailing block is quantised over the present rows,
    # exactly as the whole prefill of that length does
    _full_and_chunks(1, 8, 2, 1000, 128, (0, 256, 768), sink, seed=4)


def test_chunk_rows_spanning_several_fold_segments():
    # T > 4096: rows of the last chunk fold more than 32 key blocks (segment -> row fold)
    _full_and_chunks(1, 2, 1, 4480, 128, (0, 4096), False, seed=5)


def test_unaligned_chunk_start_is_rejected():
    x8 = torch.zeros((1, 1, 256, 128), dtype=torch.int8, device="cuda")
    e = torch.zeros((1, 1, 2), dtype=torch.int32, device="cuda")
    with pytest.raises(ValueError):
        A.prefill_chunk_lattice(x8, e, x8, e, x8, e, None, 100, 300)
