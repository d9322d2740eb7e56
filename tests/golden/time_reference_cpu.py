"""Time the reference's own torch CPU path (make_lssab8_long_attn, its defaults) against the C
oracle port on the same inputs and the same host cores, and check their outputs are bit-equal.
It runs where the reference project is present (not on the GPU box); bench.py's reference arm
times the port, and this script gives the port-to-reference speed factor that arm stands for.

    LSSAB8_REFERENCE_DIR=<reference project>/reference python tests/golden/time_reference_cpu.py H KVH T [outliers]

Inputs: the seeded synthetic prefill inputs (lockstep_b200.workloads.prefill_inputs, seed 0;
`outliers` the fraction of K channels scaled x8, 0.01 for config 2), batch 1, dh 128, causal,
sink off.  Prints one dict: seconds and TOPS of each, the factor, and
whether the bf16 outputs are identical.
"""
import os
import sys
import time

os.environ["PYTHONDONTWRITEBYTECODE"] = "1"
sys.dont_write_bytecode = True
REF = os.environ.get("LSSAB8_REFERENCE_DIR")
if not REF:
    sys.exit("set LSSAB8_REFERENCE_DIR to the reference project's reference/ directory")
sys.path.insert(0, REF)
ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402
import torch  # noqa: E402

import oracle as O  # noqa: E402
from lockstep_b200 import workloads as W  # noqa: E402


class _Module:
    layer_idx = 0


def main():
    H, KVH, T = (int(x) for x in sys.argv[1:4])
    outliers = float(sys.argv[4]) if len(sys.argv) > 4 else 0.0
    dh = 128
    nt = os.cpu_count() or 1
    torch.set_num_threads(nt)
    import lssab8_torch as R
    q, k, v = W.prefill_inputs(1, H, KVH, T, dh, outliers=outliers, seed=0)
    ops = 4 * dh * H * T * (T + 1) // 2
    attn = R.make_lssab8_long_attn()
    qt, kt, vt = (torch.from_numpy(np.ascontiguousarray(x)).to(torch.bfloat16) for x in (q, k, v))
    t0 = time.time()
    out, _ = attn(_Module(), qt, kt, vt, None)
    tr = time.time() - t0
    O.build()
    t0 = time.time()
    o2 = O.attention(q[0], k[0], v[0], nthreads=nt)
    tp = time.time() - t0
    ref_bits = out[0].contiguous().view(torch.int16).numpy().view(np.uint16)
    port_bits = O.f32_to_bf16_bits(o2.transpose(1, 0, 2))
    print(dict(H=H, KVH=KVH, T=T, dh=dh, outliers=outliers, cores=nt, reference_s=round(tr, 3), port_s=round(tp, 3),
               reference_tops=round(ops / tr / 1e12, 5), port_tops=round(ops / tp / 1e12, 5),
               port_speedup=round(tr / tp, 2), bit_equal=bool(np.array_equal(ref_bits, port_bits))))


if __name__ == "__main__":
    main()
