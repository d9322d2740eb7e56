"""Run one LSSA-B8 case on cuda:0, for external profilers (Nsight Compute).

    python -m lockstep_b200.profile_case prefill --cfg 2 [--reps 3] [--batch B]
    python -m lockstep_b200.profile_case decode  --cfg 3 [--reps 3] [--sink]

Inputs are the seeded synthetic inputs of the named benchmark configuration; the lattice is
prepared once, then the hot kernel runs `reps` times (prefill: prefill_kernel on the prepared
lattice; decode: decode_kernel on the paged lattice).
"""
import argparse

import torch

from . import attention as A
from . import decode as D
from . import workloads as W


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("what", choices=["prefill", "decode"])
    ap.add_argument("--cfg", type=int, default=2)
    ap.add_argument("--reps", type=int, default=3)
    ap.add_argument("--batch", type=int, default=0, help="override the batch size")
    ap.add_argument("--sink", action="store_true")
    a = ap.parse_args()
    c = dict(W.CONFIGS[a.cfg])
    if a.batch:
        c["B"] = a.batch
    dev = torch.device("cuda:0")
    to = lambda x: torch.from_numpy(x).to(torch.bfloat16).to(dev)
    if a.what == "prefill":
        q, k, v = W.prefill_inputs(c["B"], c["H"], c["KVH"], c["T"], c["dh"], outliers=c.get("outliers", 0.0), seed=0)
        qd, kd, vd = to(q), to(k), to(v)
        q8, eq = A.quant_rows(qd)
        k8, ek, _ = A.quant_blocks(kd, 0)
        v8, ev, e0 = A.quant_blocks(vd, 2 if a.sink else 0)
        out = torch.empty((c["B"], c["T"], c["H"], c["dh"]), dtype=torch.bfloat16, device=dev)
        for _ in range(a.reps):
            A.prefill_lattice(q8, eq, k8, ek, v8, ev, e0 if a.sink else None, c["T"], out=out)
    else:
        q, k, v = W.decode_inputs(c["B"], c["H"], c["KVH"], c["L"], c["dh"], seed=0)
        kv = D.contiguous_kv(to(k), to(v), sink=a.sink)
        qd = to(q)
        for _ in range(a.reps):
            D.decode(qd, kv, split_blocks=c["L"] // 128 // c["nsplit"], check=False)
    torch.cuda.synchronize()
    A.check_device_errors(dev)
    print("ok")


if __name__ == "__main__":
    main()
