"""The row-replay verifier's host logic on the CPU, with the pinned oracle as the row computer:
key streams across steps, role from the engine's prefill flag, generated rows under contract v2,
incomplete sequences, records without a role, the per-layer step budget, and detection of a
single wrong output row.  (tests/test_verify_rows_gpu.py runs the same dumps through the
kernels.)"""
import torch

import verify_dump as VD
from lockstep_b200 import verify_rows as VR


def _mu():
    g = torch.Generator().manual_seed(3)
    return [torch.randn(VD.KVH, VD.DH, generator=g) * 2.0, torch.randn(VD.KVH, VD.DH, generator=g) * 2.0]


def _oracle(mu):
    """rows [T - nq, T) of the oracle's causal attention for the step's queries q [nq, H, dh]."""
    def rows(q, k, v, layer):
        T, nq = k.shape[0], q.shape[0]
        full = torch.zeros((T,) + tuple(q.shape[1:]), dtype=q.dtype)
        full[T - nq:] = q
        return VD.oracle_rows(full, k, v, layer, mu)[T - nq:]
    return rows


def test_replay_passes_on_oracle_outputs():
    mu = _mu()
    dump = VD.make(mu=mu)
    res = VR.replay(dump, prompt_rows=_oracle(mu), generated_rows=_oracle(mu))
    assert res["pass_"] and res["prompt_bad"] == 0 and res["generated_bad"] == 0
    for key, want in VD.EXPECT.items():
        assert res[key] == want, (key, res[key], want)


def test_generated_rows_counted_only():
    mu = _mu()
    res = VR.replay(VD.make(mu=mu), prompt_rows=_oracle(mu), generated_rows=None, generated="count")
    assert res["pass_"] and not res["generated_checked"]
    assert res["generated_rows"] == VD.EXPECT["generated_rows"] and res["generated_bad"] == 0


def test_replay_finds_one_wrong_row():
    mu = _mu()
    dump = VD.make(mu=mu)
    bad = dump[2]["out"].view(torch.int16).clone()
    bad[5, 1, 7] ^= 1                                       # one bit of one (token, head) row
    dump[2]["out"] = bad.view(torch.bfloat16)
    res = VR.replay(dump, prompt_rows=_oracle(mu), generated_rows=_oracle(mu))
    assert not res["pass_"] and res["prompt_bad"] == 1
    assert res["per_layer"]["0"]["prompt_bad"] == 1


def test_replay_finds_one_wrong_generated_row():
    mu = _mu()
    dump = VD.make(mu=mu)
    bad = dump[1]["out"].view(torch.int16).clone()
    bad[1, 3, 0] ^= 0x40
    dump[1]["out"] = bad.view(torch.bfloat16)
    res = VR.replay(dump, prompt_rows=_oracle(mu), generated_rows=_oracle(mu))
    assert not res["pass_"] and res["generated_bad"] == 1 and res["prompt_bad"] == 0


def test_key_offset_matters():
    # outputs made with the offsets do not verify without them (the layer's mu is applied)
    mu = _mu()
    dump = VD.make(mu=mu)
    res = VR.replay(dump, prompt_rows=_oracle(None), generated_rows=_oracle(None))
    assert not res["pass_"]


def test_max_steps_counts_prompt_and_generated_steps():
    # the budget is per layer and in dump order; with 3 steps per layer the first three complete
    # sequence-steps of each layer are checked: two prompts, then one generated step
    dump = VD.make()
    rows = _oracle(None)
    res = VR.replay(dump, prompt_rows=rows, generated_rows=rows, max_steps=3)
    assert res["pass_"]
    assert res["prompt_steps"] == 2 * 2 and res["generated_steps"] == 2 * 1
    res = VR.replay(dump, prompt_rows=rows, generated_rows=rows, max_steps=1)
    assert res["prompt_steps"] == 2 and res["generated_steps"] == 0
