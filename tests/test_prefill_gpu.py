"""GPU parity of the tcgen05 prefill against the reference's recorded outputs and the pinned
oracle: every comparison is bit-exact (integer/byte work and a fixed sequence of RN binary32
operations; there is no floating-point tolerance in this contract)."""
import numpy as np
import pytest
import torch

import fixtures as FX
import golden_data as GD
import oracle as O
from lockstep_b200 import attention as A
from lockstep_b200 import lssab8_torch as L8
from lockstep_b200 import lssab9_torch as L9
from lockstep_b200 import workloads as W

pytestmark = pytest.mark.gpu


class _Mod:
    layer_idx = 0


def _cuda(x, dtype):
    return torch.from_numpy(np.ascontiguousarray(x)).to(dtype).cuda()


def drop_in(q, k, v, sink=False, dtype=torch.float32):
    """Reference-shaped call: q [H,T,dh] numpy -> out [H,T,dh] numpy (in dtype)."""
    fn = L9.make_lssab9_long_attn(sink_alone=True) if sink else L8.make_lssab8_long_attn()
    o, none = fn(_Mod(), _cuda(q[None], dtype), _cuda(k[None], dtype), _cuda(v[None], dtype), None)
    assert none is None and o.dtype == dtype and o.is_contiguous()
    return o[0].transpose(0, 1).float().cpu().numpy()


def test_cfg1_equals_reference_torch_output():
    c = W.CONFIGS[1]
    q, k, v = W.prefill_inputs(c["B"], c["H"], c["KVH"], c["T"], c["dh"], seed=0)
    for sink, name in ((False, "cfg1_out_b8.npy"), (True, "cfg1_out_b9sink.npy")):
        fn = L9.make_lssab9_long_attn(sink_alone=True) if sink else L8.make_lssab8_long_attn()
        o, _ = fn(_Mod(), _cuda(q, torch.bfloat16), _cuda(k, torch.bfloat16), _cuda(v, torch.bfloat16), None)
        ref = np.load(GD.GOLDEN_DIR + "/" + name)
        assert np.array_equal(GD.bf16_bits_of_torch(o[0]), ref), name


CASES = FX.all_cases() + FX.sink300_cases()


@pytest.mark.parametrize("case", CASES, ids=[c["tag"] for c in CASES])
def test_selftest_fixtures_equal_reference_golden(case):
    rec = GD.case_by_tag()[case["tag"]]
    q, k, v = case["q"], case["k"], case["v"]
    if "b8" in rec:
        assert GD.sha(GD.f32bits(drop_in(q, k, v))) == rec["b8"]
    if rec["b9_sink"].startswith("assert"):
        with pytest.raises(AssertionError):
            drop_in(q, k, v, sink=True)
    else:
        assert GD.sha(GD.f32bits(drop_in(q, k, v, sink=True))) == rec["b9_sink"]


def test_cfg2_equals_reference_torch_output():
    c = W.CONFIGS[2]
    q, k, v = W.prefill_inputs(c["B"], c["H"], c["KVH"], c["T"], c["dh"], outliers=c["outliers"], seed=0)
    out = A.prefill(_cuda(q, torch.bfloat16), _cuda(k, torch.bfloat16), _cuda(v, torch.bfloat16))
    g = GD.golden()["cfg2"]
    for b in range(c["B"]):
        assert GD.sha(GD.bf16_bits_of_torch(out[b])) == g["b8_per_batch"][b], "batch %d" % b


@pytest.mark.parametrize("T", [1, 2, 127, 128, 129, 255, 257, 1000, 4096, 4097, 8200])
@pytest.mark.parametrize("dh", [64, 128])
def test_edge_lengths_against_oracle(T, dh):
    rng = np.random.default_rng(T * 7 + dh)
    H, KVH = 4, 2
    q = rng.standard_normal((H, T, dh)).astype(np.float32)
    k = rng.standard_normal((KVH, T, dh)).astype(np.float32)
    v = rng.standard_normal((KVH, T, dh)).astype(np.float32)
    rows = None if T <= 1100 else sorted(set(x for x in [0, 1, 127, 128, 4095, 4096, T - 2, T - 1] + list(range(0, T, 331))
                                             if x < T))
    for sink in (False, True):
        got = drop_in(q, k, v, sink=sink)
        ref = O.attention(q, k, v, sink=sink, rows=rows)
        if rows is None:
            assert np.array_equal(GD.f32bits(got), GD.f32bits(ref)), (T, dh, sink)
        else:
            assert np.array_equal(GD.f32bits(got[:, rows]), GD.f32bits(ref[:, rows])), (T, dh, sink)


@pytest.mark.parametrize("H,KVH", [(1, 1), (8, 1), (6, 3), (32, 8)])
def test_gqa_groups_bf16(H, KVH):
    rng = np.random.default_rng(H * 100 + KVH)
    T, dh = 384, 128
    q = W.bf16_round(rng.standard_normal((H, T, dh)).astype(np.float32))
    k = W.bf16_round(rng.standard_normal((KVH, T, dh)).astype(np.float32))
    v = W.bf16_round(rng.standard_normal((KVH, T, dh)).astype(np.float32))
    fn = L8.make_lssab8_long_attn()
    o, _ = fn(_Mod(), _cuda(q[None], torch.bfloat16), _cuda(k[None], torch.bfloat16), _cuda(v[None], torch.bfloat16), None)
    ref = O.f32_to_bf16_bits(O.attention(q, k, v).transpose(1, 0, 2))
    assert np.array_equal(GD.bf16_bits_of_torch(o[0]), ref)


def test_prep_arrays_bit_exact():
    rng = np.random.default_rng(5)
    T, dh = 300, 128
    q = rng.standard_normal((1, 3, T, dh)).astype(np.float32) * 5
    k = rng.standard_normal((1, 2, T, dh)).astype(np.float32)
    v = rng.standard_normal((1, 2, T, dh)).astype(np.float32)
    v[:, :, 0] *= 300.0
    q8, eq = A.quant_rows(_cuda(q, torch.float32))
    oq8, oeq = O.quant_rows(q[0])
    assert np.array_equal(q8[0, :, :T].cpu().numpy(), oq8) and np.array_equal(eq[0, :, :T].cpu().numpy(), oeq)
    assert not q8[0, :, T:].any()
    for mode in (0, 1, 2):
        x8, e, e0 = A.quant_blocks(_cuda(v, torch.float32), mode=mode)
        ox8, oe, oe0, _ = O.quant_blocks(v[0], mode)
        assert np.array_equal(x8[0, :, :T].cpu().numpy(), ox8)
        assert np.array_equal(e[0].cpu().numpy(), oe)
        if mode == 2:
            assert np.array_equal(e0[0].cpu().numpy(), oe0)


def test_lean_single_token_vector_through_the_lattice_entry():
    dev = torch.device("cuda")
    q8 = torch.zeros((1, 1, 128, 128), dtype=torch.int8, device=dev); q8[0, 0, 0, 0] = 1
    k8 = torch.zeros_like(q8); k8[0, 0, 0, 0] = 1
    v8 = torch.zeros_like(q8); v8[0, 0, 0, 0] = 2
    z = torch.zeros((1, 1, 128), dtype=torch.int32, device=dev)
    e = torch.zeros((1, 1, 1), dtype=torch.int32, device=dev)
    out = A.prefill_lattice(q8, z, k8, e, v8, e, None, T=1, out_dtype=torch.bfloat16)
    assert GD.bf16_bits_of_torch(out[0, 0, 0]).tolist() == GD.golden()["lean_single_token"]


def test_strided_and_fp16_inputs():
    rng = np.random.default_rng(11)
    H, KVH, T, dh = 4, 2, 200, 64
    q = rng.standard_normal((T, H, dh)).astype(np.float32)       # [T, H, dh] layout, viewed as [H, T, dh]
    k = rng.standard_normal((T, KVH, dh)).astype(np.float32)
    v = rng.standard_normal((T, KVH, dh)).astype(np.float32)
    qt = _cuda(q, torch.float16).transpose(0, 1)[None]
    kt = _cuda(k, torch.float16).transpose(0, 1)[None]
    vt = _cuda(v, torch.float16).transpose(0, 1)[None]
    assert not qt.is_contiguous()
    o, _ = L8.make_lssab8_long_attn()(_Mod(), qt, kt, vt, None)
    qf = q.astype(np.float16).astype(np.float32).transpose(1, 0, 2)
    kf = k.astype(np.float16).astype(np.float32).transpose(1, 0, 2)
    vf = v.astype(np.float16).astype(np.float32).transpose(1, 0, 2)
    ref = O.attention(qf, kf, vf).transpose(1, 0, 2).astype(np.float16)
    assert np.array_equal(o[0].cpu().numpy().view(np.uint16), ref.view(np.uint16))


def test_cfg4_sampled_rows_equal_reference_golden():
    c = W.CONFIGS[4]
    q, k, v = W.prefill_inputs(c["B"], c["H"], c["KVH"], c["T"], c["dh"], seed=0)
    g = GD.golden()["cfg4"]
    out = A.prefill(_cuda(q, torch.bfloat16), _cuda(k, torch.bfloat16), _cuda(v, torch.bfloat16))
    for s in g["samples"]:
        got = GD.bf16_bits_of_torch(out[s["b"], s["row"], s["h"]])
        assert got.tolist() == s["bf16"], s
