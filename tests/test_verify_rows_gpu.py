"""The row-replay verifier end to end on the GPU: the synthetic engine dump (outputs from the
pinned oracle) replayed through this library's kernels -- prompt rows as block-aligned prefill
chunks on the key lattice, generated rows through the split-KV decode (contract v2) -- with the
layer's key offsets, plus the negative cases: one flipped bit in a prompt row and in a generated
row, and outputs that were made with offsets replayed without them."""
import pytest
import torch

import verify_dump as VD
from lockstep_b200 import verify_rows as VR

pytestmark = pytest.mark.gpu


def _mu():
    g = torch.Generator().manual_seed(3)
    return [torch.randn(VD.KVH, VD.DH, generator=g) * 2.0, torch.randn(VD.KVH, VD.DH, generator=g) * 2.0]


def test_replay_on_kernels_passes():
    mu = _mu()
    res = VR.replay(VD.make(mu=mu), mu=mu)
    assert res["pass_"], res
    for key, want in VD.EXPECT.items():
        assert res[key] == want, (key, res[key], want)


def test_replay_on_kernels_finds_flipped_bits():
    mu = _mu()
    dump = VD.make(mu=mu)
    for rec, (t, h, c) in ((2, (5, 1, 7)), (1, (1, 3, 0))):
        bad = dump[rec]["out"].view(torch.int16).clone()
        bad[t, h, c] ^= 1
        dump[rec]["out"] = bad.view(torch.bfloat16)
    res = VR.replay(dump, mu=mu)
    assert not res["pass_"] and res["prompt_bad"] == 1 and res["generated_bad"] == 1


def test_replay_on_kernels_needs_the_offsets():
    res = VR.replay(VD.make(mu=_mu()), mu=None)
    assert not res["pass_"] and res["prompt_bad"] > 0


def test_cli_main(tmp_path):
    mu = _mu()
    dump = VD.make(mu=mu)
    torch.save(dump, tmp_path / "dump.pt")
    torch.save({"MU_MID": torch.stack(mu)}, tmp_path / "mu.pt")
    assert VR.main([str(tmp_path / "dump.pt"), str(tmp_path / "mu.pt"), str(tmp_path / "out.json")]) == 0
