"""The reference switches to another contract version from the environment (LSSAB8_SEG,
LSSAB8_RESCALE, LSSAB_TABLE; reference/lssab8_golden.py:57-68, reference/lssab_golden.py:80).
The drop-ins implement the filed contract only: with a variant selected they refuse (no CUDA is
touched), and with the variables unset or at the filed values they build as usual."""
import numpy as np
import pytest

from lockstep_b200 import golden
from lockstep_b200 import lssab8_torch as L8
from lockstep_b200 import lssab9_torch as L9

VARIANTS = [("LSSAB8_SEG", "0"), ("LSSAB8_SEG", "16"), ("LSSAB8_RESCALE", "mul"), ("LSSAB_TABLE", "frac2")]


@pytest.mark.parametrize("var,val", VARIANTS)
def test_variant_environment_is_refused(monkeypatch, var, val):
    monkeypatch.setenv(var, val)
    with pytest.raises(NotImplementedError, match=var):
        L8.make_lssab8_long_attn()
    with pytest.raises(NotImplementedError, match=var):
        L9.make_lssab9_long_attn(sink_alone=True)
    x = np.zeros((1, 4, 8), np.float32)
    with pytest.raises(NotImplementedError, match=var):
        golden.lssab8_attention(x, x, x)


@pytest.mark.parametrize("var,val", [("LSSAB8_SEG", "32"), ("LSSAB8_RESCALE", "field"), ("LSSAB_TABLE", "frac")])
def test_filed_values_build(monkeypatch, var, val):
    monkeypatch.setenv(var, val)
    assert callable(L8.make_lssab8_long_attn())
    assert callable(L9.make_lssab9_long_attn(sink_alone=True))
