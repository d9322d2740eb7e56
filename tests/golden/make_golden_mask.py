#!/usr/bin/env python3
"""Record the reference's outputs for the golden entry points' general forms in
tests/golden/golden_mask.json: causal off, key_valid masks, the per-head query exponent.

Run where the reference project is importable (its ``reference/`` directory, given by the required
$LSSAB8_REFERENCE_DIR):

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden_mask.py

For every case of tests/fixtures.py:mask_cases() it stores sha256 of the inputs and of the float32
output bits of lssab8_golden.lssab8_attention(q, k, v, causal=..., key_valid=..., q_exp_mode=...)
(sink off) and lssab9_golden.lssab9_attention(..., sink_alone=True) (sink on).
"""
import hashlib
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(REPO, "tests"))
REF = os.environ.get("LSSAB8_REFERENCE_DIR")
if not REF:
    sys.exit("set LSSAB8_REFERENCE_DIR to the reference project's reference/ directory")
sys.path.insert(0, REF)
for var in ("LSSAB8_SEG", "LSSAB8_RESCALE", "LSSAB_TABLE"):
    assert not os.environ.get(var), "%s changes the reference function; unset it" % var

import lssab8_golden as G8  # noqa: E402
import lssab9_golden as G9  # noqa: E402

import fixtures as FX  # noqa: E402


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def f32bits(a):
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32)).view(np.uint32)


def main():
    out = {}
    for c in FX.mask_cases():
        q, k, v = c["q"], c["k"], c["v"]
        kw = dict(causal=c["causal"], key_valid=c["key_valid"], q_exp_mode=c["q_exp_mode"])
        parts = [q.ravel(), k.ravel(), v.ravel()]
        if c["key_valid"] is not None:
            parts.append(np.asarray(c["key_valid"], np.float32))
        rec = {"inputs": sha(np.concatenate(parts))}
        rec["b8"] = sha(f32bits(G8.lssab8_attention(q, k, v, **kw)))
        rec["b9sink"] = sha(f32bits(G9.lssab9_attention(q, k, v, sink_alone=True, **kw)))
        out[c["tag"]] = rec
        print(c["tag"], rec, flush=True)
    with open(os.path.join(HERE, "golden_mask.json"), "w") as f:
        json.dump(out, f, indent=1)


if __name__ == "__main__":
    main()
