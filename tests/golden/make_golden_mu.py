#!/usr/bin/env python3
"""Record the reference's outputs for the key-offset (mu) cases in tests/golden/golden_mu.json.

Run where the reference project is importable (its ``reference/`` directory, given by the required
$LSSAB8_REFERENCE_DIR):

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden_mu.py

For every case of tests/fixtures.py:mu_cases() it stores sha256 of the inputs and of the float32
output bits of lssab8_golden.lssab8_attention(q, k, v, mu=mu) (sink off) and
lssab9_golden.lssab9_attention(q, k, v, mu=mu, sink_alone=True) (sink on), and, as a control, of
lssab8_attention without mu.  Nothing in the test suite imports the reference: the GPU test reads
the JSON.
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
    for c in FX.mu_cases():
        q, k, v, mu = c["q"], c["k"], c["v"], c["mu"]
        rec = {"inputs": sha(np.concatenate([q.ravel(), k.ravel(), v.ravel(), mu.ravel()]))}
        rec["b8_mu"] = sha(f32bits(G8.lssab8_attention(q, k, v, mu=mu)))
        rec["b9sink_mu"] = sha(f32bits(G9.lssab9_attention(q, k, v, mu=mu, sink_alone=True)))
        rec["b8_no_mu"] = sha(f32bits(G8.lssab8_attention(q, k, v)))
        out[c["tag"]] = rec
        print(c["tag"], rec)
    with open(os.path.join(HERE, "golden_mu.json"), "w") as f:
        json.dump(out, f, indent=1)


if __name__ == "__main__":
    main()
