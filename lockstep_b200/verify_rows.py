"""Row-replay verifier: recompute the rows of an engine's attention dump with the B200 kernels and
check them bit for bit.

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

The replay follows this library's own data flow.  Each (layer, sequence) owns a KeyStream that
appends the step's new keys and values; once a stream holds all sl keys of a step, the step's
rows are recomputed on the GPU and compared as bit patterns, with no tolerance:

  * prompt rows (the engine's prefill flag set) [T - nq, T) run as a block-aligned chunk of the
    causal prefill on the key lattice of [0, T) (lssab8_prefill_chunk_lattice): the chunk starts
    at the 128-row boundary at or below T - nq, and its rows before T - nq, absent from the dump,
    are zero queries (rows are quantised and folded independently, so they change no checked
    bit);
  * generated rows follow contract v2, under which a generated row is an LSSA-B8 row too
    (reference/lssab8_selftest.py:320-336): a one-row step runs the split-KV decode kernel on
    the paged lattice of its T keys, a longer one the prefill chunk.  The reference's verifier
    predates v2 and checks them under LSSA-B, which has no kernel here; generated="count" only
    counts them.

The role comes from the engine's flag, never from the number of query rows.  MAX_STEPS bounds
the checked (layer, sequence) steps per layer, prompt and generated alike, in dump order (the
reference's sampling rule, so both tools check the same steps).

usage: python -m lockstep_b200.verify_rows <dump.pt> <mu.pt | -> <out.json>
env:   MAX_STEPS (checked sequence-steps per layer, 0 = all), LOCKSTEP_LSSAB_MU_KIND (the key of
       the mu file holding the [layers, KVH, dh] offsets, default MU_MID), LOCKSTEP_GENERATED
       ("b8", the default: check generated rows under contract v2; "count": count them only)
"""
import json
import os
import sys
import time

import torch

from . import attention as A

KB = 128


class KeyStream:
    """The keys and values of one (layer, sequence) in arrival order ([n, KVH, dh] pieces)."""

    def __init__(self):
        self.k, self.v, self.n = [], [], 0

    def append(self, k, v):
        self.k.append(k)
        self.v.append(v)
        self.n += k.shape[0]

    def keys(self):
        if len(self.k) > 1:                        # coalesce, so later steps append to one piece
            self.k, self.v = [torch.cat(self.k)], [torch.cat(self.v)]
        return self.k[0], self.v[0]


def _mu_of(mu, layer, dev):
    return None if mu is None else torch.as_tensor(mu[layer]).to(device=dev, dtype=torch.float32)


def kernel_prompt_rows(q, k, v, layer, mu=None):
    """Rows [T - nq, T) of the LSSA-B8 causal prefill over keys [0, T), as a block-aligned chunk.

    q [nq, H, dh] (the rows' queries), k / v [T, KVH, dh] -> [nq, H, dh] in q.dtype."""
    dev = torch.device("cuda", torch.cuda.current_device())
    T, nq = k.shape[0], q.shape[0]
    T0 = (T - nq) // KB * KB
    qc = torch.zeros((1, q.shape[1], T - T0, q.shape[2]), dtype=q.dtype, device=dev)
    qc[0, :, T - nq - T0:] = q.to(dev).transpose(0, 1)
    kk = k.to(dev).transpose(0, 1)[None]
    vv = v.to(dev).transpose(0, 1)[None]
    q8, eq = A.quant_rows(qc)
    mu_l = _mu_of(mu, layer, dev)
    k8, ek = A.quant_keys_offset(kk, mu_l) if mu_l is not None else A.quant_blocks(kk, 0)[:2]
    v8, ev, _ = A.quant_blocks(vv, 0)
    out = A.prefill_chunk_lattice(q8, eq, k8, ek, v8, ev, None, T0, T, out_dtype=q.dtype)
    A.check_device_errors(dev)
    return out[0, T - nq - T0:]


def kernel_generated_rows(q, k, v, layer, mu=None):
    """Generated rows under contract v2: one row -> the split-KV decode over the paged lattice of
    the T keys (the offset keys k - mu in binary32 when the layer has an offset); more rows -> the
    prefill chunk."""
    if q.shape[0] != 1:
        return kernel_prompt_rows(q, k, v, layer, mu)
    from . import decode as D
    dev = torch.device("cuda", torch.cuda.current_device())
    kk = k.to(dev).transpose(0, 1)[None]
    mu_l = _mu_of(mu, layer, dev)
    if mu_l is not None:
        kk = kk.float() - mu_l[None, :, None, :]
        vv = v.to(dev).float().transpose(0, 1)[None]
    else:
        vv = v.to(dev).transpose(0, 1)[None]
    kv = D.contiguous_kv(kk.contiguous(), vv.contiguous(), sink=False)
    return D.decode(q.to(dev), kv, out_dtype=q.dtype)


def _bits(t):
    t = t.contiguous()
    return t.view(torch.int16) if t.element_size() == 2 else t.view(torch.int32)


def replay(dump, mu=None, prompt_rows=None, generated_rows=None, max_steps=0, generated="b8"):
    """Check the complete rows of `dump`; returns the summary dict (pass_ is the verdict).

    prompt_rows / generated_rows(q [nq, H, dh], k [T, KVH, dh], v [T, KVH, dh], layer) ->
    [nq, H, dh] in the dump's output dtype: the rows [T - nq, T) for the step's queries.  The
    defaults run the B200 kernels (kernel_prompt_rows, kernel_generated_rows with `mu`)."""
    if prompt_rows is None:
        prompt_rows = lambda q, k, v, layer: kernel_prompt_rows(q, k, v, layer, mu)  # noqa: E731
    if generated_rows is None:
        generated_rows = lambda q, k, v, layer: kernel_generated_rows(q, k, v, layer, mu)  # noqa: E731
    if generated not in ("b8", "count"):
        raise ValueError("generated must be 'b8' or 'count'")
    t0 = time.time()
    streams, per_layer = {}, {}
    n = dict(prompt_rows=0, prompt_bad=0, prompt_steps=0, generated_rows=0, generated_bad=0,
             generated_steps=0, generated_checked=generated == "b8", skipped_no_role=0)
    for d in dump:
        layer = int(d["layer"])
        pref = d.get("pref")
        if pref is None:
            n["skipped_no_role"] += 1
            continue
        qsl = [int(x) for x in d["qsl"]]
        sl = [int(x) for x in d["sl"]]
        pl = per_layer.setdefault(layer, dict(prompt_rows=0, prompt_bad=0, generated_rows=0, generated_bad=0,
                                              steps=0))
        for i in range(int(d["nseq"])):
            a0, a1 = qsl[i], qsl[i + 1]
            if a1 <= a0:
                continue
            ks = streams.setdefault((layer, int(d["bt0"][i])), KeyStream())
            ks.append(d["k"][a0:a1].cpu(), d["v"][a0:a1].cpu())
            if ks.n != sl[i]:
                continue                                   # this step's keys are not all in the dump
            if max_steps and pl["steps"] >= max_steps:
                continue
            pl["steps"] += 1
            prompt = bool(pref[i])
            rows = (a1 - a0) * int(d["q"].shape[1])
            kind = "prompt" if prompt else "generated"
            n[kind + "_rows"] += rows
            n[kind + "_steps"] += 1
            pl[kind + "_rows"] += rows
            if not prompt and generated == "count":
                continue
            k_all, v_all = ks.keys()
            fn = prompt_rows if prompt else generated_rows
            ref = fn(d["q"][a0:a1].cpu(), k_all, v_all, layer).cpu()
            got = d["out"][a0:a1].cpu()
            if got.dtype != ref.dtype:
                raise ValueError("the dump's outputs are %s, the recomputed rows %s" % (got.dtype, ref.dtype))
            bad = int((_bits(got) != _bits(ref)).any(-1).sum().item())
            n[kind + "_bad"] += bad
            pl[kind + "_bad"] += bad
    ok = n["prompt_bad"] == 0 and n["generated_bad"] == 0 and n["prompt_rows"] + n["generated_rows"] > 0
    return dict(pass_=ok, secs=round(time.time() - t0, 1), max_steps=max_steps, **n,
                per_layer={str(k): v for k, v in sorted(per_layer.items())})


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
    res = replay(dump, mu=mu, max_steps=int(os.environ.get("MAX_STEPS", "0")),
                 generated=os.environ.get("LOCKSTEP_GENERATED", "b8"))
    res["dump"] = dump_path
    with open(out_path, "w") as f:
        json.dump(res, f, indent=1)
    print("[%s] prompt rows %d bad %d | generated rows %d bad %d (%s) | %d + %d sequence-steps in %.1fs -> %s"
          % ("PASS" if res["pass_"] else "FAIL", res["prompt_rows"], res["prompt_bad"], res["generated_rows"],
             res["generated_bad"], "checked, contract v2" if res["generated_checked"] else "counted only",
             res["prompt_steps"], res["generated_steps"], res["secs"], out_path), flush=True)
    return 0 if res["pass_"] else 1


if __name__ == "__main__":
    sys.exit(main())
