"""The row-replay verifier's host logic on the CPU, with the pinned oracle as the row computer:
accumulation of keys across steps, role from the engine's prefill flag, incomplete sequences,
records without a role, and detection of a single wrong output row."""
import torch

import verify_dump as VD
from lockstep_b200 import verify_rows as VR


def _mu():
    g = torch.Generator().manual_seed(3)
    return [torch.randn(VD.KVH, VD.DH, generator=g) * 2.0, torch.randn(VD.KVH, VD.DH, generator=g) * 2.0]


def test_replay_passes_on_oracle_outputs():
    mu = _mu()
    dump = VD.make(mu=mu)
    res = VR.replay(dump, compute=lambda q, k, v, layer: VD.oracle_rows(q, k, v, layer, mu))
    assert res["pass_"] and res["prompt_bad"] == 0
    for key, want in VD.EXPECT.items():
        assert res[key] == want, (key, res[key], want)


def test_replay_finds_one_wrong_row():
    mu = _mu()
    dump = VD.make(mu=mu)
    bad = dump[2]["out"].view(torch.int16).clone()
    bad[5, 1, 7] ^= 1                                       # one bit of one (token, head) row
    dump[2]["out"] = bad.view(torch.bfloat16)
    res = VR.replay(dump, compute=lambda q, k, v, layer: VD.oracle_rows(q, k, v, layer, mu))
    assert not res["pass_"] and res["prompt_bad"] == 1
    assert res["per_layer"]["0"]["prompt_bad"] == 1


def test_key_offset_matters():
    # outputs made with the offsets do not verify without them (the layer's mu is applied)
    mu = _mu()
    dump = VD.make(mu=mu)
    res = VR.replay(dump, compute=lambda q, k, v, layer: VD.oracle_rows(q, k, v, layer, None))
    assert not res["pass_"]


def test_max_steps_limits_checked_steps():
    dump = VD.make()
    res = VR.replay(dump, compute=lambda q, k, v, layer: VD.oracle_rows(q, k, v, layer), max_steps=1)
    assert res["prompt_steps"] == 2 and res["pass_"]
