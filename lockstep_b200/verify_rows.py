"""Row-replay verifier: recompute the prompt rows of an engine's attention dump with the B200 kernels
and check them bit for bit.

The dump is the one the reference's verifier reads (reference tools/verify_rows.py:1-18, 63-104):
a list of records, one per dumped (layer, engine step), each with

    layer    int                 the model layer
    nseq     int                 sequences in the step
    qsl      [nseq + 1] ints     query start offsets of each sequence's tokens in this step
    sl       [nseq] ints         each sequence's length after this step
    bt0      [nseq] ints         the sequence's first cache block (its identity across steps)
    pref     [nseq] bools        the engine's is_prefilling flag (absent: the record is skipped)
    q        [ntok, H, dh]       the step's query rows, k / v [ntok, KVH, dh] its new keys / values
    out      [ntok, H, dh]       the engine's attention output for those rows

Keys and values are accumulated per (layer, sequence) across the records; once a sequence's keys
are complete for a step (accumulated length == sl), its rows in that step are checked.  The role
comes from the engine's own prefill flag, never from the number of query rows.  Prompt rows are
LSSA-B8 rows: they are recomputed here (the query rows placed at the end of a zero query block --
rows are quantised independently, so the other rows do not matter) and compared as bit patterns,
with no tolerance.  Generated rows follow the reference's LSSA-B rule, a different contract with
no kernel in this library; they are counted, not checked.

usage: python -m lockstep_b200.verify_rows <dump.pt> <mu.pt | -> <out.json>
env:   MAX_STEPS (checked sequence-steps per layer, 0 = all), LOCKSTEP_LSSAB_MU_KIND (the key of
       the mu file holding the [layers, KVH, dh] offsets, default MU_MID)
"""
import json
import os
import sys
import time

import torch

from . import attention as A


def kernel_rows(q, k, v, layer, mu=None):
    """LSSA-B8 rows on the GPU: q [T, H, dh], k/v [T, KVH, dh] -> [T, H, dh] in q.dtype.
    mu: per-layer key offsets ([layers, KVH, dh] or a sequence of [KVH, dh]) or None."""
    dev = torch.device("cuda", torch.cuda.current_device())
    qq = q.to(dev).transpose(0, 1)[None]
    kk = k.to(dev).transpose(0, 1)[None]
    vv = v.to(dev).transpose(0, 1)[None]
    mu_l = None if mu is None else torch.as_tensor(mu[layer]).to(device=dev, dtype=torch.float32)
    return A.prefill(qq, kk, vv, mu=mu_l, out_dtype=q.dtype)[0]


def _bits(t):
    t = t.contiguous()
    return t.view(torch.int16) if t.element_size() == 2 else t.view(torch.int32)


def replay(dump, mu=None, compute=None, max_steps=0):
    """Check every complete prompt row of `dump`; returns the summary dict (pass_ is the verdict).

    compute(q [T, H, dh], k [T, KVH, dh], v [T, KVH, dh], layer) -> [T, H, dh] in the dump's
    output dtype; the default runs the B200 kernels (kernel_rows)."""
    if compute is None:
        compute = lambda q, k, v, layer: kernel_rows(q, k, v, layer, mu)  # noqa: E731
    t0 = time.time()
    acc, per_layer = {}, {}
    n = dict(prompt_rows=0, prompt_bad=0, prompt_steps=0, generated_rows=0, generated_steps=0,
             skipped_no_role=0)
    for d in dump:
        layer = int(d["layer"])
        pref = d.get("pref")
        if pref is None:
            n["skipped_no_role"] += 1
            continue
        qsl = [int(x) for x in d["qsl"]]
        sl = [int(x) for x in d["sl"]]
        pl = per_layer.setdefault(layer, dict(prompt_rows=0, prompt_bad=0, generated_rows=0, steps=0))
        for i in range(int(d["nseq"])):
            a0, a1 = qsl[i], qsl[i + 1]
            if a1 <= a0:
                continue
            key = (layer, int(d["bt0"][i]))
            kk, vv = acc.get(key, (None, None))
            k_i, v_i = d["k"][a0:a1].cpu(), d["v"][a0:a1].cpu()
            kk = k_i if kk is None else torch.cat([kk, k_i], 0)
            vv = v_i if vv is None else torch.cat([vv, v_i], 0)
            acc[key] = (kk, vv)
            T = kk.shape[0]
            if T != sl[i]:
                continue                                   # this step's keys are not all in the dump
            nq = a1 - a0
            rows = nq * int(d["q"].shape[1])
            if not bool(pref[i]):
                n["generated_rows"] += rows
                n["generated_steps"] += 1
                pl["generated_rows"] += rows
                continue
            if max_steps and pl["steps"] >= max_steps:
                continue
            pl["steps"] += 1
            q = torch.zeros((T,) + tuple(d["q"].shape[1:]), dtype=d["q"].dtype)
            q[T - nq:] = d["q"][a0:a1].cpu()
            ref = compute(q, kk, vv, layer)[T - nq:].cpu()
            got = d["out"][a0:a1].cpu()
            if got.dtype != ref.dtype:
                raise ValueError("the dump's outputs are %s, the recomputed rows %s" % (got.dtype, ref.dtype))
            bad = int((_bits(got) != _bits(ref)).any(-1).sum().item())
            n["prompt_rows"] += rows
            n["prompt_bad"] += bad
            n["prompt_steps"] += 1
            pl["prompt_rows"] += rows
            pl["prompt_bad"] += bad
    ok = n["prompt_bad"] == 0 and n["prompt_rows"] > 0
    res = dict(pass_=ok, secs=round(time.time() - t0, 1), max_steps=max_steps, **n,
               per_layer={str(k): v for k, v in sorted(per_layer.items())})
    return res


def main(argv=None):
    argv = sys.argv[1:] if argv is None else argv
    if len(argv) != 3:
        print(__doc__)
        return 2
    dump_path, mu_path, out_path = argv
    dump = torch.load(dump_path, map_location="cpu", weights_only=False)
    mu = None
    if mu_path != "-":
        blob = torch.load(mu_path, map_location="cpu", weights_only=False)
        mu = blob[os.environ.get("LOCKSTEP_LSSAB_MU_KIND", "MU_MID")].to(torch.float32)
    res = replay(dump, mu=mu, max_steps=int(os.environ.get("MAX_STEPS", "0")))
    res["dump"] = dump_path
    with open(out_path, "w") as f:
        json.dump(res, f, indent=1)
    print("[%s] prompt rows %d bad %d | generated rows %d (not checked: LSSA-B rule) | %d sequence-steps "
          "in %.1fs -> %s" % ("PASS" if res["pass_"] else "FAIL", res["prompt_rows"], res["prompt_bad"],
                              res["generated_rows"], res["prompt_steps"], res["secs"], out_path), flush=True)
    return 0 if res["pass_"] else 1


if __name__ == "__main__":
    sys.exit(main())
