"""Run one LSSA-B8 case on cuda:0, for external profilers (Nsight Compute).

    python -m lockstep_b200.profile_case prefill --cfg 2 [--reps 3] [--batch B]
    python -m lockstep_b200.profile_case decode  --cfg 3 [--reps 3] [--sink]
    python -m lockstep_b200.profile_case decode  --cfg 5 [--reps 3]          (paged, ragged, sink on)
    python -m lockstep_b200.profile_case prep    --cfg 3 [--reps 3] [--sink]   (the paged lattice writer)

Inputs are the seeded synthetic inputs of the named benchmark configuration; the lattice is
prepared once, then the hot kernel runs `reps` times (prefill: prefill_kernel on the prepared
lattice; decode: the split-KV decode on the paged lattice; prep: the lattice writer from bf16).
"""
import argparse

import torch

from . import attention as A
from . import decode as D
from . import workloads as W


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("what", choices=["prefill", "decode", "prep"])
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
    elif c["kind"] == "paged_decode":
        import numpy as np
        lens = W.ragged_lengths(c["B"], c["Lmin"], c["Lmax"], seed=0)
        q, ks, vs = W.ragged_inputs(c["B"], c["H"], c["KVH"], c["dh"], lens, seed=0)
        fk = torch.cat([to(x).transpose(0, 1) for x in ks]).contiguous()
        fv = torch.cat([to(x).transpose(0, 1) for x in vs]).contiguous()
        del ks, vs
        bt, npages = W.page_table(lens, c["page"], seed=0)
        cu = np.concatenate([[0], np.cumsum(lens)])
        args = (fk, fv, torch.tensor(lens, dtype=torch.int32, device=dev), torch.tensor(bt, device=dev), npages)
        kv = D.build_paged_kv(*args, sink=True, cu_seqlens=cu)
        qd = to(q)
        for _ in range(a.reps):
            if a.what == "prep":
                D.build_paged_kv(*args, sink=True, cu_seqlens=cu, check=False)
            else:
                D.decode(qd, kv, split_blocks=8, check=False)
    else:
        q, k, v = W.decode_inputs(c["B"], c["H"], c["KVH"], c["L"], c["dh"], seed=0)
        kd, vd = to(k), to(v)
        kv = D.contiguous_kv(kd, vd, sink=a.sink)
        qd = to(q)
        for _ in range(a.reps):
            if a.what == "prep":
                D.contiguous_kv(kd, vd, sink=a.sink, check=False)
            else:
                D.decode(qd, kv, split_blocks=c["L"] // 128 // c["nsplit"], check=False)
    torch.cuda.synchronize()
    A.check_device_errors(dev)
    print("ok")


if __name__ == "__main__":
    main()
