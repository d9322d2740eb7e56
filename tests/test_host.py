"""Host-side behaviour of the drop-in modules that needs no GPU: the reference's asserts and
arm dispatch are mirrored, and nothing falls back to a CPU implementation."""
import pytest
import torch

from lockstep_b200 import lssab8_torch as L8
from lockstep_b200 import lssab9_torch as L9
from lockstep_b200 import workloads as W


class _Mod:
    layer_idx = 0


def test_build_arm8_unknown_name_returns_none():
    assert L8.build_arm8("E") is None
    assert L8.build_arm8("LB2") is None
    assert callable(L8.build_arm8("L8"))
    assert callable(L8.build_arm8("L8-RN-W9", long=False))


@pytest.mark.parametrize("arm", ["L8-RN-W8", "L8-TR", "L8-RN-n8", "L8-RN-KB64", "L16"])
def test_control_arms_have_no_kernel(arm):
    with pytest.raises(NotImplementedError):
        L8.build_arm8(arm)


def test_key_offset_selected_by_layer():
    assert callable(L8.make_lssab8_long_attn(mu=[torch.zeros(1, 128)]))

    class _M:
        layer_idx = 1
    mu = [torch.zeros(2, 64), torch.full((2, 64), 0.5)]
    got = L8._mu_for(mu, _M(), torch.device("cpu"))
    assert got.dtype == torch.float32 and got.shape == (2, 64) and float(got[0, 0]) == 0.5
    assert L8._mu_for(None, _M(), torch.device("cpu")) is None


def test_b9_options():
    assert L9.build_arm9("L9-v16") is None
    assert callable(L9.build_arm9("L9-sink"))
    with pytest.raises(NotImplementedError):
        L9.make_lssab9_long_attn(v_planes=2)


def test_batch_must_be_one_like_the_reference():
    attn = L8.make_lssab8_long_attn()
    q = torch.zeros(2, 4, 8, 64)
    k = torch.zeros(2, 4, 8, 64)
    with pytest.raises(AssertionError):
        attn(_Mod(), q, k, k, None)


def test_no_cpu_fallback():
    attn = L8.make_lssab8_long_attn()
    q = torch.zeros(1, 4, 8, 64, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        attn(_Mod(), q, q, q, None)


def test_workload_generators_are_seeded():
    q1, k1, v1 = W.prefill_inputs(1, 2, 1, 16, 64, seed=3)
    q2, k2, v2 = W.prefill_inputs(1, 2, 1, 16, 64, seed=3)
    assert (q1 == q2).all() and (k1 == k2).all() and (v1 == v2).all()
    assert (W.bf16_round(q1) == q1).all()
    lens = W.ragged_lengths(64, 1024, 32768, seed=0)
    assert int(lens.sum()) == 1101299           # the survey's seed-0 total
    bt, total = W.page_table(lens[:4], 16, seed=0)
    used = bt[bt >= 0]
    assert sorted(used.tolist()) == list(range(total))
