"""The vLLM attention backend (lockstep_b200.vllm_backend) inside a real vLLM engine: a tiny
random-weight Llama model (8/2 heads, dh 128, 2 layers) serves three prompts of ragged lengths
and decodes greedily in a child process (tests/vllm_run.py), which records every attention call
in the row-replay verifier's format.  The verifier then recomputes every recorded row of every
layer with the pinned CPU oracle -- prompt rows as causal prefill rows, generated rows as decode
rows -- and every one must match bit for bit (sink off and on)."""
import os
import subprocess
import sys

import numpy as np
import pytest
import torch

import oracle as O
from lockstep_b200 import verify_rows as VR

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


def _oracle_rows(sink):
    def rows(q, k, v, layer):
        T, nq = k.shape[0], q.shape[0]
        full = torch.zeros((T,) + tuple(q.shape[1:]), dtype=torch.float32)
        full[T - nq:] = q.float()
        o = O.attention(full.numpy().transpose(1, 0, 2), k.float().numpy().transpose(1, 0, 2),
                        v.float().numpy().transpose(1, 0, 2), sink=sink)
        bits = O.f32_to_bf16_bits(o).transpose(1, 0, 2)[T - nq:].copy()
        return torch.from_numpy(bits.view(np.int16)).view(torch.bfloat16)
    return rows


@pytest.mark.parametrize("sink", [False, True])
def test_vllm_engine_rows_equal_oracle(sink, tmp_path):
    pytest.importorskip("vllm")
    out = str(tmp_path / "dump.pt")
    cmd = [sys.executable, os.path.join(HERE, "vllm_run.py"), out] + (["--sink"] if sink else [])
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, (r.stdout[-3000:], r.stderr[-6000:])
    rec = torch.load(out, weights_only=False)
    assert all(len(t) == 6 for t in rec["tokens"])
    res = VR.replay(rec["dump"], prompt_rows=_oracle_rows(sink), generated_rows=_oracle_rows(sink))
    assert res["pass_"], res
    assert res["prompt_rows"] == 2 * 8 * (200 + 77 + 128)          # layers x heads x prompt tokens
    assert res["generated_rows"] == 2 * 8 * 3 * 5                   # the 6th token is sampled, never attended
