"""Access to the committed golden fixtures (tests/golden/, written by make_golden.py from the
reference itself) plus small helpers shared by the CPU and GPU parity tests."""
import hashlib
import json
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN_DIR = os.path.join(HERE, "golden")
_G = None


def golden():
    global _G
    if _G is None:
        with open(os.path.join(GOLDEN_DIR, "golden.json")) as f:
            _G = json.load(f)
    return _G


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def f32bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def inputs_digest(q, k, v):
    return sha(np.concatenate([f32bits(q).ravel(), f32bits(k).ravel(), f32bits(v).ravel()]))


def case_by_tag():
    return {c["tag"]: c for c in golden()["selftest_cases"]}


def bf16_bits_of_torch(t):
    """uint16 numpy view of a bfloat16 torch tensor (on any device)."""
    import torch
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)
