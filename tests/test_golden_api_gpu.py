"""The golden-shaped entry points (lockstep_b200.golden: lssab8_attention, lssab9_attention) on the
GPU, bit for bit against the reference golden model's recorded outputs: the 52 selftest fixtures
(causal, sink off and on), and the general forms -- causal off, key_valid masks (random, a whole
block hidden, key 0 hidden, rows that see no key), the per-head query exponent, a non-causal row
folding more than one 32-block segment -- plus rows= / heads= restrictions and torch inputs."""
import json
import os

import numpy as np
import pytest
import torch

import fixtures as FX
import golden_data as GD
from lockstep_b200 import golden as G

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


def _bits(o):
    return np.ascontiguousarray(o, np.float32).view(np.uint32)


@pytest.mark.parametrize("case", FX.all_cases() + FX.sink300_cases(), ids=lambda c: c["tag"])
def test_selftest_fixtures_equal_reference(case):
    rec = {r["tag"]: r for r in GD.golden()["selftest_cases"]}[case["tag"]]
    q, k, v = case["q"], case["k"], case["v"]
    assert GD.inputs_digest(q, k, v) == rec["inputs"]
    if "b8" in rec:
        assert FX.digest(_bits(G.lssab8_attention(q, k, v))) == rec["b8"]
    if rec["b9_sink"].startswith("assert"):
        with pytest.raises(AssertionError):         # the reference's e_v assert, surfaced the same way
            G.lssab9_attention(q, k, v, sink_alone=True)
    else:
        assert FX.digest(_bits(G.lssab9_attention(q, k, v, sink_alone=True))) == rec["b9_sink"]


@pytest.mark.parametrize("case", [c["tag"] for c in FX.mask_cases()])
def test_general_forms_equal_reference(case):
    gold = json.load(open(os.path.join(HERE, "golden", "golden_mask.json")))[case]
    c = [x for x in FX.mask_cases() if x["tag"] == case][0]
    kw = dict(causal=c["causal"], key_valid=c["key_valid"], q_exp_mode=c["q_exp_mode"])
    assert FX.digest(_bits(G.lssab8_attention(c["q"], c["k"], c["v"], **kw))) == gold["b8"]
    assert FX.digest(_bits(G.lssab9_attention(c["q"], c["k"], c["v"], sink_alone=True, **kw))) == gold["b9sink"]
    if c["causal"] and c["key_valid"] is None:          # the torch drop-ins take the same forms
        from lockstep_b200 import lssab8_torch as L8
        from lockstep_b200 import lssab9_torch as L9
        args = [torch.from_numpy(x).cuda()[None] for x in (c["q"], c["k"], c["v"])]
        o8, _ = L8.make_lssab8_long_attn(qexp=c["q_exp_mode"])(None, *args, None)
        o9, _ = L9.make_lssab9_long_attn(qexp=c["q_exp_mode"], sink_alone=True)(None, *args, None)
        assert FX.digest(_bits(o8[0].transpose(0, 1).cpu().numpy())) == gold["b8"]
        assert FX.digest(_bits(o9[0].transpose(0, 1).cpu().numpy())) == gold["b9sink"]


def test_rows_heads_and_torch_inputs():
    c = FX.mask_cases()[1]
    full = G.lssab8_attention(c["q"], c["k"], c["v"], key_valid=c["key_valid"])
    part = G.lssab8_attention(c["q"], c["k"], c["v"], key_valid=c["key_valid"], rows=[0, 7, 259], heads=[1, 3])
    want = np.zeros_like(full)
    for h in (1, 3):
        for r in (0, 7, 259):
            want[h, r] = full[h, r]
    assert np.array_equal(_bits(part), _bits(want))
    t = G.lssab8_attention(*(torch.from_numpy(x).cuda() for x in (c["q"], c["k"], c["v"])), key_valid=c["key_valid"])
    assert isinstance(t, torch.Tensor) and np.array_equal(_bits(t.cpu().numpy()), _bits(full))
    with pytest.raises(NotImplementedError):
        G.lssab8_attention(c["q"], c["k"], c["v"], kb=64)


@pytest.mark.parametrize("case", FX.keyshift_cases(), ids=lambda c: c["tag"])
@pytest.mark.parametrize("sink", [False, True])
def test_value_keyshift_equals_reference(case, sink):
    """B9.3 v_keyshift (reference/lssab9_golden.py:37-70, 179-186) against the reference's recorded
    d8 shifts and outputs, through the golden entry point and through the torch drop-in."""
    from lockstep_b200 import attention as A
    from lockstep_b200 import lssab9_torch as L9
    rec = json.load(open(os.path.join(HERE, "golden", "golden_keyshift.json")))[case["tag"]]
    q, k, v, dmax = case["q"], case["k"], case["v"], case["dmax"]
    name = "sink" if sink else "nosink"
    _, _, _, d8 = A.quant_values_keyshift(torch.from_numpy(v).cuda()[None], dmax, sink)
    T = q.shape[1]
    assert GD.sha(d8[0, :, :T].cpu().numpy()) == rec["d8_" + name]
    out = G.lssab9_attention(q, k, v, sink_alone=sink, v_keyshift=dmax)
    assert FX.digest(_bits(out)) == rec["out_" + name]
    attn = L9.make_lssab9_long_attn(sink_alone=sink, v_keyshift=dmax)
    o, _ = attn(None, *(torch.from_numpy(x).cuda()[None] for x in (q, k, v)), None)
    assert np.array_equal(_bits(o[0].transpose(0, 1).cpu().numpy()), _bits(out))
