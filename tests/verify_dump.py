"""A synthetic engine dump for the row-replay verifier, with outputs from the pinned oracle.

Two layers (their own key offsets), two sequences identified by their first cache block:
a prompt step, a generated step, a chunked prompt continuation, a record without the prefill
flag, and a sequence whose first step is missing from the dump (never complete, never checked).
"""
import numpy as np
import torch

import oracle as O

H, KVH, DH = 4, 2, 64


def oracle_rows(q, k, v, layer, mu=None):
    """[T, H, dh] bf16 rows of the oracle for q [T, H, dh], k/v [T, KVH, dh] (bf16 tensors)."""
    qn = q.float().numpy().transpose(1, 0, 2)
    kn = k.float().numpy().transpose(1, 0, 2)
    vn = v.float().numpy().transpose(1, 0, 2)
    o = O.attention(qn, kn, vn, mu=None if mu is None else np.asarray(mu[layer], np.float32))
    bits = O.f32_to_bf16_bits(o).transpose(1, 0, 2).copy()
    return torch.from_numpy(bits.view(np.int16)).view(torch.bfloat16)


def make(mu=None, seed=7):
    g = np.random.RandomState(seed)
    bf = lambda a: torch.from_numpy(a.astype(np.float32)).to(torch.bfloat16)   # noqa: E731
    seqs = {100: 0, 200: 0, 300: 0}            # tokens so far
    store = {}                                 # (layer, seq) -> (q, k, v) of all tokens so far

    def step(layer, plan, pref):
        """plan: [(seq, ntok)]; pref: per sequence prefill flag or None."""
        qs, ks, vs, outs, qsl, sl, bt0 = [], [], [], [], [0], [], []
        for s, nt in plan:
            q = bf(g.standard_normal((nt, H, DH)))
            k = bf(g.standard_normal((nt, KVH, DH)) + 2.0)
            v = bf(g.standard_normal((nt, KVH, DH)))
            pq, pk, pv = store.get((layer, s), (None, None, None))
            fq = q if pq is None else torch.cat([pq, q])
            fk = k if pk is None else torch.cat([pk, k])
            fv = v if pv is None else torch.cat([pv, v])
            store[(layer, s)] = (fq, fk, fv)
            out = oracle_rows(fq, fk, fv, layer, mu)[-nt:]
            qs.append(q); ks.append(k); vs.append(v); outs.append(out)
            qsl.append(qsl[-1] + nt); sl.append(fk.shape[0]); bt0.append(s)
        rec = dict(layer=layer, nseq=len(plan), qsl=torch.tensor(qsl), sl=torch.tensor(sl),
                   bt0=torch.tensor(bt0), q=torch.cat(qs), k=torch.cat(ks), v=torch.cat(vs), out=torch.cat(outs))
        if pref is not None:
            rec["pref"] = torch.tensor(pref)
        return rec

    dump = []
    for layer in (0, 1):
        dump.append(step(layer, [(100, 200), (200, 130)], [True, True]))      # prompts
        dump.append(step(layer, [(100, 1), (200, 1)], [False, False]))         # one generated token each
        dump.append(step(layer, [(100, 60)], [True]))                          # chunked prompt continuation
        dump.append(step(layer, [(200, 3)], None))                             # no role: skipped
    # sequence 300: its first step is not in the dump, so its keys are never complete
    first = step(0, [(300, 50)], [True])
    dump.append(step(0, [(300, 20)], [True]))
    del first
    return dump


EXPECT = dict(prompt_steps=2 * 3, generated_steps=2 * 2,
              prompt_rows=2 * (200 + 130 + 60) * H, generated_rows=2 * 2 * H, skipped_no_role=2)
