#!/usr/bin/env python3
"""Record the reference's outputs for the B9.3 v_keyshift cases in tests/golden/golden_keyshift.json.

Run where the reference project is importable (its ``reference/`` directory, given by the required
$LSSAB8_REFERENCE_DIR):

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden_keyshift.py

For every case of tests/fixtures.py:keyshift_cases() it stores sha256 of the inputs, of the
per-key shifts d8 and of the float32 output bits of
lssab9_golden.lssab9_attention(q, k, v, v_keyshift=dmax) with the sink off and on
(sink_alone=True).  Nothing in the test suite imports the reference.
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

import lssab9_golden as G9  # noqa: E402

import fixtures as FX  # noqa: E402


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def f32bits(a):
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32)).view(np.uint32)


def main():
    out = {}
    for c in FX.keyshift_cases():
        q, k, v, dmax = c["q"], c["k"], c["v"], c["dmax"]
        rec = {"inputs": sha(np.concatenate([q.ravel(), k.ravel(), v.ravel()])), "dmax": dmax}
        for sink in (False, True):
            p = G9.lssab9_quantize(q, k, v, sink_alone=sink, v_keyshift=dmax)
            name = "sink" if sink else "nosink"
            rec["d8_" + name] = sha(np.asarray(p["d8"], np.int8))
            rec["d8_max_" + name] = int(np.asarray(p["d8"]).max())
            rec["out_" + name] = sha(f32bits(G9.lssab9_attention(q, k, v, sink_alone=sink, v_keyshift=dmax)))
        out[c["tag"]] = rec
        print(c["tag"], rec)
    with open(os.path.join(HERE, "golden_keyshift.json"), "w") as f:
        json.dump(out, f, indent=1)


if __name__ == "__main__":
    main()
