"""The CPU oracle pinned to the reference's own outputs (tests/golden/, made by running the
reference).  CPU only: these tests are what makes the oracle a trustworthy checker for the GPU
parity tests."""
import numpy as np
import pytest

import fixtures as FX
import golden_data as GD
import oracle as O
from lockstep_b200 import workloads as W


def test_t2_table_digest_and_anchors():
    g = GD.golden()["t2"]
    t = O.t2_table()
    assert O.table_digest(t) == g["digest"] == O.T2_DIGEST
    assert [int(x) for x in t[:9 * 128]] == g["values"]
    assert int(t[0]) == 255 and int(t[128]) == 128 and int(t[1151]) == 1 and int(t[1152]) == 0
    assert not t[1152:].any()


def test_gbase_matches_reference():
    for dh, base in GD.golden()["gbase"].items():
        assert O.gbase(int(dh)) == base


def test_lean_single_token_vector():
    """formal/Lockstep/Attention/Concrete.lean:104-126: quantised single-token row -> 0x4000, zeros."""
    q8 = np.zeros((1, 1, 128), np.int8); q8[0, 0, 0] = 1
    k8 = np.zeros((1, 1, 128), np.int8); k8[0, 0, 0] = 1
    v8 = np.zeros((1, 1, 128), np.int8); v8[0, 0, 0] = 2
    z = np.zeros((1, 1), np.int32)
    out = O.core(dict(q8=q8, eq=z, k8=k8, ek=z, v8=v8, ev=z))
    bits = O.f32_to_bf16_bits(out[0, 0])
    assert [int(x) for x in bits] == GD.golden()["lean_single_token"]


CASES = FX.all_cases() + FX.sink300_cases()


@pytest.mark.parametrize("case", CASES, ids=[c["tag"] for c in CASES])
def test_oracle_equals_reference_golden(case):
    rec = GD.case_by_tag()[case["tag"]]
    assert GD.inputs_digest(case["q"], case["k"], case["v"]) == rec["inputs"]
    if "b8" in rec:
        assert GD.sha(GD.f32bits(O.attention(case["q"], case["k"], case["v"]))) == rec["b8"]
    if rec["b9_sink"].startswith("assert"):
        with pytest.raises(AssertionError):
            O.attention(case["q"], case["k"], case["v"], sink=True)
    else:
        assert GD.sha(GD.f32bits(O.attention(case["q"], case["k"], case["v"], sink=True))) == rec["b9_sink"]


def test_oracle_rescale_boundary():
    """reference/lssab8_selftest.py:141-152: the exponent-field rule flushes where a float
    multiply would round up to 2^-126, and a flush returns +0.0 even for negative inputs.
    Exercised through the fold: a row whose old segment is 127 doublings below the new max."""
    # two blocks, the second block's max 127 doublings above the first's (jump127 fixture)
    case = [c for c in FX.jump_cases() if c["tag"] == "jump127_T512"][0]
    out = O.attention(case["q"], case["k"], case["v"])
    assert np.isfinite(out).all()


def test_cfg1_oracle_equals_reference_torch_dropin():
    c = W.CONFIGS[1]
    q, k, v = W.prefill_inputs(c["B"], c["H"], c["KVH"], c["T"], c["dh"], seed=0)
    assert GD.inputs_digest(q, k, v) == GD.golden()["cfg1"]["inputs"]
    ref8 = np.load(GD.GOLDEN_DIR + "/cfg1_out_b8.npy")
    ref9 = np.load(GD.GOLDEN_DIR + "/cfg1_out_b9sink.npy")
    o8 = O.f32_to_bf16_bits(O.attention(q[0], k[0], v[0]).transpose(1, 0, 2))
    o9 = O.f32_to_bf16_bits(O.attention(q[0], k[0], v[0], sink=True).transpose(1, 0, 2))
    assert np.array_equal(o8, ref8)
    assert np.array_equal(o9, ref9)


def test_cfg2_oracle_equals_reference_torch_dropin():
    c = W.CONFIGS[2]
    q, k, v = W.prefill_inputs(c["B"], c["H"], c["KVH"], c["T"], c["dh"], outliers=c["outliers"], seed=0)
    g = GD.golden()["cfg2"]
    assert GD.inputs_digest(q, k, v) == g["inputs"]
    for b in range(c["B"]):
        o = O.f32_to_bf16_bits(O.attention(q[b], k[b], v[b]).transpose(1, 0, 2))
        assert GD.sha(o) == g["b8_per_batch"][b], "batch %d" % b


def test_cfg3_decode_oracle_equals_reference_golden():
    c = W.CONFIGS[3]
    q, k, v = W.decode_inputs(c["B"], c["H"], c["KVH"], c["L"], c["dh"], seed=0)
    g = GD.golden()["cfg3"]
    assert GD.inputs_digest(q, k, v) == g["inputs"]
    n = g["seqs"]                                    # sequences the reference itself evaluated
    r8 = np.stack([O.f32_to_bf16_bits(O.decode_rows(q[b], k[b], v[b])) for b in range(n)])
    r9 = np.stack([O.f32_to_bf16_bits(O.decode_rows(q[b], k[b], v[b], sink=True)) for b in range(n)])
    assert GD.sha(r8) == g["b8"]
    assert GD.sha(r9) == g["b9_sink"]


def test_decode_row_equals_prefill_last_row():
    """S9 (reference/lssab8_selftest.py:320-336) on the oracle, across a segment boundary."""
    for T in (1, 129, 4097):
        g = np.random.RandomState(T)
        q = g.standard_normal((2, T, 128)).astype(np.float32)
        k = g.standard_normal((1, T, 128)).astype(np.float32)
        v = g.standard_normal((1, T, 128)).astype(np.float32)
        full = O.attention(q, k, v, rows=[T - 1])[:, T - 1]
        row = O.decode_rows(q[:, T - 1], k, v)
        assert np.array_equal(GD.f32bits(full), GD.f32bits(row))


def _golden_mu():
    import json
    import os
    with open(os.path.join(GD.GOLDEN_DIR, "golden_mu.json")) as f:
        return json.load(f)


@pytest.mark.parametrize("case", FX.mu_cases(), ids=[c["tag"] for c in FX.mu_cases()])
def test_oracle_key_offset_equals_reference_golden(case):
    rec = _golden_mu()[case["tag"]]
    q, k, v, mu = case["q"], case["k"], case["v"], case["mu"]
    assert GD.sha(np.concatenate([q.ravel(), k.ravel(), v.ravel(), mu.ravel()])) == rec["inputs"]
    assert GD.sha(GD.f32bits(O.attention(q, k, v, mu=mu))) == rec["b8_mu"]
    assert GD.sha(GD.f32bits(O.attention(q, k, v, sink=True, mu=mu))) == rec["b9sink_mu"]
    assert GD.sha(GD.f32bits(O.attention(q, k, v))) == rec["b8_no_mu"]


@pytest.mark.parametrize("case", FX.keyshift_cases(), ids=[c["tag"] for c in FX.keyshift_cases()])
def test_oracle_value_keyshift_equals_reference_golden(case):
    import json
    import os
    with open(os.path.join(GD.GOLDEN_DIR, "golden_keyshift.json")) as f:
        rec = json.load(f)[case["tag"]]
    q, k, v, dmax = case["q"], case["k"], case["v"], case["dmax"]
    assert GD.sha(np.concatenate([q.ravel(), k.ravel(), v.ravel()])) == rec["inputs"]
    for sink, name in ((False, "nosink"), (True, "sink")):
        p = O.prep(q, k, v, sink=sink, v_keyshift=dmax)
        assert GD.sha(np.asarray(p["d8"], np.int8)) == rec["d8_" + name]
        assert int(p["d8"].max()) == rec["d8_max_" + name] > 0
        assert GD.sha(GD.f32bits(O.attention(q, k, v, sink=sink, v_keyshift=dmax))) == rec["out_" + name]


def test_oracle_aligned_chunk_invariance():
    """The property chunked prefill rests on (reference/lssab8_selftest.py:292-317): the prefill of a
    128-aligned prefix equals the prefix of the whole prefill bit for bit, while a non-aligned cut
    may differ (its last block is quantised over fewer rows)."""
    T = 640
    g = np.random.RandomState(11)
    q = g.standard_normal((2, T, 128)).astype(np.float32)
    k = g.standard_normal((1, T, 128)).astype(np.float32)
    v = g.standard_normal((1, T, 128)).astype(np.float32)
    full = O.attention(q, k, v)
    for cut in (128, 256, 384, 512):
        part = O.attention(q[:, :cut], k[:, :cut], v[:, :cut])
        assert np.array_equal(part.view(np.uint32), full[:, :cut].view(np.uint32)), cut
    k2, v2 = k.copy(), v.copy()
    k2[:, 505] *= np.float32(64.0)
    v2[:, 505] *= np.float32(64.0)
    full2 = O.attention(q, k2, v2)
    part2 = O.attention(q[:, :500], k2[:, :500], v2[:, :500])
    assert not np.array_equal(part2.view(np.uint32), full2[:, :500].view(np.uint32))


def test_oracle_masked_and_noncausal_equal_reference():
    """causal off, key_valid masks and the per-head query exponent, against the reference golden
    model's recorded outputs (tests/golden/make_golden_mask.py)."""
    import json
    import os
    gold = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "golden_mask.json")))
    for c in FX.mask_cases():
        rec = gold[c["tag"]]
        parts = [c["q"].ravel(), c["k"].ravel(), c["v"].ravel()]
        if c["key_valid"] is not None:
            parts.append(np.asarray(c["key_valid"], np.float32))
        assert FX.digest(np.concatenate(parts)) == rec["inputs"], c["tag"]
        for sink, key in ((False, "b8"), (True, "b9sink")):
            o = O.attention(c["q"], c["k"], c["v"], sink=sink, causal=c["causal"], key_valid=c["key_valid"],
                            q_exp_mode=c["q_exp_mode"])
            assert FX.digest(o.view(np.uint32)) == rec[key], (c["tag"], key)
