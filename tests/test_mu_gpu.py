"""The key offset mu through the drop-in modules, bit for bit against the reference's outputs.

The reference subtracts a per-layer offset mu[layer] [KVH, dh] from the keys in binary32 before
the key quantiser (reference/lssab8_torch.py:116-122, 143-144; reference/lssab_golden.py:221).
tests/golden/golden_mu.json holds the reference golden model's output digests for the
tests/fixtures.py:mu_cases() inputs (tests/golden/make_golden_mu.py).
"""
import json
import os

import numpy as np
import pytest
import torch

import fixtures as FX
import golden_data as GD
import oracle as O
from lockstep_b200 import attention as A
from lockstep_b200 import lssab8_torch as L8
from lockstep_b200 import lssab9_torch as L9

pytestmark = pytest.mark.gpu

CASES = FX.mu_cases()


class _Layer:
    def __init__(self, idx):
        self.layer_idx = idx


def _golden():
    with open(os.path.join(GD.GOLDEN_DIR, "golden_mu.json")) as f:
        return json.load(f)


def _run(fn, case, layer=1):
    c = lambda x: torch.from_numpy(np.ascontiguousarray(x))[None].cuda()
    o, none = fn(_Layer(layer), c(case["q"]), c(case["k"]), c(case["v"]), None)
    assert none is None
    return o[0].transpose(0, 1).float().cpu().numpy()


@pytest.mark.parametrize("case", CASES, ids=[c["tag"] for c in CASES])
def test_drop_in_with_key_offset_equals_reference(case):
    rec = _golden()[case["tag"]]
    # mu is indexed by the module's layer: layer 1 here, with a decoy at layer 0
    mu = [np.zeros_like(case["mu"]) + np.float32(3.0), case["mu"]]
    assert GD.sha(GD.f32bits(_run(L8.make_lssab8_long_attn(mu=mu), case))) == rec["b8_mu"]
    assert GD.sha(GD.f32bits(_run(L9.make_lssab9_long_attn(mu=mu, sink_alone=True), case))) == rec["b9sink_mu"]
    assert GD.sha(GD.f32bits(_run(L8.make_lssab8_long_attn(), case))) == rec["b8_no_mu"]


def test_batched_key_offset_equals_oracle():
    case = CASES[0]
    q, k, v, mu = case["q"], case["k"], case["v"], case["mu"]
    c = lambda x: torch.from_numpy(np.ascontiguousarray(x)).cuda()
    qb = torch.stack([c(q), c(q[:, ::-1])])                 # two sequences sharing the layer's mu
    kb = torch.stack([c(k), c(k[:, ::-1])])
    vb = torch.stack([c(v), c(v[:, ::-1])])
    out = A.prefill(qb, kb, vb, mu=c(mu), out_dtype=torch.float32)
    for b in range(2):
        want = O.attention(qb[b].cpu().numpy(), kb[b].cpu().numpy(), vb[b].cpu().numpy(), mu=mu)
        assert np.array_equal(out[b].transpose(0, 1).cpu().numpy().view(np.uint32), want.view(np.uint32))
