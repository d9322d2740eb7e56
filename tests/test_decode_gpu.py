"""GPU parity of the split-KV decode against the reference's recorded decode rows and the
pinned oracle (bit-exact), including paged/ragged caches, the sink, and split invariance."""
import numpy as np
import pytest
import torch

import golden_data as GD
import oracle as O
from lockstep_b200 import attention as A
from lockstep_b200 import decode as D
from lockstep_b200 import workloads as W

pytestmark = pytest.mark.gpu


def _cuda(x, dtype=torch.bfloat16):
    return torch.from_numpy(np.ascontiguousarray(x)).to(dtype).cuda()


@pytest.mark.parametrize("sink", [False, True])
def test_cfg3_equals_reference_golden(sink):
    c = W.CONFIGS[3]
    q, k, v = W.decode_inputs(c["B"], c["H"], c["KVH"], c["L"], c["dh"], seed=0)
    kv = D.contiguous_kv(_cuda(k), _cuda(v), sink=sink)
    out = D.decode(_cuda(q), kv, split_blocks=c["L"] // 128 // c["nsplit"])
    bits = GD.bf16_bits_of_torch(out)
    g = GD.golden()["cfg3"]
    n = g["seqs"]                                    # sequences the reference itself evaluated
    assert GD.sha(bits[:n]) == (g["b9_sink"] if sink else g["b8"])
    for b in range(n, c["B"]):                       # the rest against the pinned oracle
        ref = O.f32_to_bf16_bits(O.decode_rows(q[b], k[b], v[b], sink=sink))
        assert np.array_equal(bits[b], ref), b


@pytest.mark.parametrize("L", [1, 2, 100, 128, 129, 1000, 4096, 4097, 9000])
@pytest.mark.parametrize("sink", [False, True])
@pytest.mark.parametrize("dh", [128, 64])
def test_decode_equals_prefill_last_row_and_oracle(L, sink, dh):
    """dh 128 runs the tensor-core streaming kernel and the refold kernel; dh 64 the dp4a kernel
    whose last split of each (sequence, kv head) refolds the block partials."""
    rng = np.random.default_rng(L + 17 * sink + dh)
    H, KVH = 8, 2
    q = W.bf16_round(rng.standard_normal((1, H, L, dh)).astype(np.float32))
    k = W.bf16_round(rng.standard_normal((1, KVH, L, dh)).astype(np.float32))
    v = W.bf16_round(rng.standard_normal((1, KVH, L, dh)).astype(np.float32))
    kv = D.contiguous_kv(_cuda(k), _cuda(v), sink=sink)
    dec = D.decode(_cuda(q[:, :, L - 1]), kv, split_blocks=3)
    ref = O.f32_to_bf16_bits(O.decode_rows(q[0, :, L - 1], k[0], v[0], sink=sink))
    assert np.array_equal(GD.bf16_bits_of_torch(dec[0]), ref)
    if L <= 4097:
        pre = A.prefill(_cuda(q), _cuda(k), _cuda(v), sink=sink)
        assert np.array_equal(GD.bf16_bits_of_torch(pre[0, L - 1]), ref)


@pytest.mark.parametrize("dh", [128, 64])
def test_split_invariance(dh):
    rng = np.random.default_rng(3)
    B, H, KVH, L = 3, 16, 4, 5000
    q = rng.standard_normal((B, H, dh)).astype(np.float32)
    k = rng.standard_normal((B, KVH, L, dh)).astype(np.float32)
    v = rng.standard_normal((B, KVH, L, dh)).astype(np.float32)
    kv = D.contiguous_kv(_cuda(k), _cuda(v), sink=True)
    outs = [GD.bf16_bits_of_torch(D.decode(_cuda(q), kv, split_blocks=s)) for s in (1, 2, 4, 7, 40)]
    for o in outs[1:]:
        assert np.array_equal(o, outs[0])


@pytest.mark.parametrize("dh", [128, 64])
def test_paged_ragged_sink_against_oracle(dh):
    B, H, KVH = 6, 32, 4
    lens = np.array([1, 17, 128, 1500, 4097, 2222], np.int64)
    rng = np.random.default_rng(9)
    q = W.bf16_round(rng.standard_normal((B, H, dh)).astype(np.float32))
    ks = [W.bf16_round(rng.standard_normal((KVH, int(L), dh)).astype(np.float32)) for L in lens]
    vs = [W.bf16_round(rng.standard_normal((KVH, int(L), dh)).astype(np.float32)) for L in lens]
    cu = np.concatenate([[0], np.cumsum(lens)])
    flat_k = np.concatenate([x.transpose(1, 0, 2) for x in ks])      # [N, KVH, dh]
    flat_v = np.concatenate([x.transpose(1, 0, 2) for x in vs])
    bt, npages = W.page_table(lens, 16, seed=5)
    kv = D.build_paged_kv(_cuda(flat_k), _cuda(flat_v), torch.tensor(lens, dtype=torch.int32).cuda(),
                          torch.tensor(bt).cuda(), npages, sink=True, cu_seqlens=cu)
    out = D.decode(_cuda(q), kv, split_blocks=2)
    for b in range(B):
        ref = O.f32_to_bf16_bits(O.decode_rows(q[b], ks[b], vs[b], sink=True))
        assert np.array_equal(GD.bf16_bits_of_torch(out[b]), ref), b


def test_bad_page_raises_device_error():
    B, H, KVH, L, dh = 1, 4, 1, 300, 128
    k = torch.randn(B, KVH, L, dh, device="cuda", dtype=torch.bfloat16)
    kv = D.contiguous_kv(k, k)
    kv.block_table[0, 3] = 10 ** 6                                   # out of the pool
    with pytest.raises(RuntimeError, match="device error"):
        D.decode(torch.randn(B, H, dh, device="cuda", dtype=torch.bfloat16), kv)


def test_cfg5_picks_equal_reference_golden_and_oracle():
    c = W.CONFIGS[5]
    lens = W.ragged_lengths(c["B"], c["Lmin"], c["Lmax"], seed=0)
    q, ks, vs = W.ragged_inputs(c["B"], c["H"], c["KVH"], c["dh"], lens, seed=0)
    cu = np.concatenate([[0], np.cumsum(lens)])
    flat_k = torch.cat([_cuda(x).transpose(0, 1) for x in ks])
    flat_v = torch.cat([_cuda(x).transpose(0, 1) for x in vs])
    bt, npages = W.page_table(lens, c["page"], seed=0)
    kv = D.build_paged_kv(flat_k, flat_v, torch.tensor(lens, dtype=torch.int32).cuda(), torch.tensor(bt).cuda(),
                          npages, sink=True, cu_seqlens=cu)
    out = D.decode(_cuda(q), kv, split_blocks=8)
    g = GD.golden()["cfg5"]
    assert g["lengths_sum"] == int(lens.sum())
    for pk in g["picks"]:
        assert GD.sha(GD.bf16_bits_of_torch(out[pk["b"]])) == pk["bf16"], pk["b"]
    for b in range(0, c["B"], 9):                                      # oracle on a spread of lengths
        ref = O.f32_to_bf16_bits(O.decode_rows(q[b], ks[b], vs[b], sink=True))
        assert np.array_equal(GD.bf16_bits_of_torch(out[b]), ref), b
