"""The serving-engine seam (lockstep_b200.engine) on the GPU: a scripted engine trace over a paged
float cache -- two layers, three sequences, prompts in 128-aligned chunks interleaved with decode
steps of the other sequences, a sequence that arrives later and one that finishes -- every output
row checked bit for bit against the pinned oracle (prompt rows: the causal prefill's rows;
generated rows: the decode row, equal to it under contract v2).  A prompt chunk off the 128-token
grid is refused."""
import numpy as np
import pytest
import torch

import oracle as O
from lockstep_b200 import engine as E
from lockstep_b200 import workloads as W

pytestmark = pytest.mark.gpu

H, KVH, DH, PAGES = 8, 2, 128, 200


class Seq:
    def __init__(self, seed, first_page, npages):
        self.rng = np.random.default_rng(seed)
        self.pages = list(range(first_page, first_page + npages))
        self.q, self.k, self.v = [], [], []

    def draw(self, n):
        f = lambda *s: W.bf16_round(self.rng.standard_normal(s).astype(np.float32))   # noqa: E731
        q, k, v = f(n, H, DH), f(n, KVH, DH), f(n, KVH, DH)
        self.q.append(q); self.k.append(k); self.v.append(v)
        return q, k, v

    @property
    def L(self):
        return sum(x.shape[0] for x in self.k)


def _oracle_rows(s, n, sink):
    q = np.concatenate(s.q)[-n:]
    k = np.concatenate(s.k).transpose(1, 0, 2)
    v = np.concatenate(s.v).transpose(1, 0, 2)
    L = k.shape[1]
    qf = np.zeros((L, H, DH), np.float32)
    qf[L - n:] = q
    o = O.attention(qf.transpose(1, 0, 2), k, v, sink=sink)          # [H, L, dh]
    return O.f32_to_bf16_bits(o.transpose(1, 0, 2)[L - n:])


@pytest.mark.parametrize("sink", [False, True])
def test_engine_trace_equals_oracle(sink):
    dev = torch.device("cuda")
    att = E.Lssab8Attention(H, KVH, DH, PAGES, max_len=1024, max_seqs=4, num_layers=2, sink=sink)
    caches = [(torch.zeros((PAGES, 16, KVH, DH), dtype=torch.bfloat16, device=dev),
               torch.zeros((PAGES, 16, KVH, DH), dtype=torch.bfloat16, device=dev)) for _ in range(2)]
    seqs = {"A": Seq(1, 0, 40), "B": Seq(2, 50, 40), "C": Seq(3, 100, 40)}
    # each step: [(sequence, new tokens, is_prefill)]
    steps = [[("A", 256, True), ("B", 100, True)],
             [("A", 44, True), ("B", 1, False)],
             [("A", 1, False), ("B", 1, False), ("C", 128, True)],
             [("C", 1, True), ("A", 1, False)],
             [("C", 1, False), ("B", 1, False), ("A", 1, False)]]
    for step in steps:
        # identical draws for both layers, as if the two layers saw the same activations
        draws = [(name, *seqs[name].draw(n), pf) for name, n, pf in step]
        qsl, lens, slots, bts = [0], [], [], []
        for name, q, k, v, pf in draws:
            s = seqs[name]
            L0 = s.L - q.shape[0]
            qsl.append(qsl[-1] + q.shape[0])
            lens.append(s.L)
            slots += [s.pages[t // 16] * 16 + t % 16 for t in range(L0, s.L)]
            bts.append(s.pages + [-1] * (64 - len(s.pages)))
        meta = E.StepMeta(query_start_loc=qsl, seq_lens=lens, block_table=torch.tensor(bts, dtype=torch.int32, device=dev),
                          slot_mapping=torch.tensor(slots, dtype=torch.long, device=dev),
                          is_prefill=[pf for *_, pf in draws])
        cat = lambda i: torch.from_numpy(np.concatenate([d[i] for d in draws])).to(torch.bfloat16).to(dev)  # noqa: E731
        q, k, v = cat(1), cat(2), cat(3)
        for layer in range(2):
            out = att.forward(layer, q, k, v, caches[layer][0], caches[layer][1], meta)
            bits = out.cpu().view(torch.int16).numpy().view(np.uint16)
            for i, (name, dq, *_rest) in enumerate(draws):
                ref = _oracle_rows(seqs[name], dq.shape[0], sink)
                assert np.array_equal(bits[qsl[i]:qsl[i + 1]], ref), (step, name, layer)


def test_unaligned_prompt_chunk_is_refused():
    dev = torch.device("cuda")
    att = E.Lssab8Attention(H, KVH, DH, PAGES, max_len=512, max_seqs=2)
    kc = torch.zeros((PAGES, 16, KVH, DH), dtype=torch.bfloat16, device=dev)
    vc = torch.zeros_like(kc)
    s = Seq(5, 0, 20)
    q, k, v = s.draw(100)
    bt = torch.tensor([s.pages + [-1] * 12], dtype=torch.int32, device=dev)
    meta = E.StepMeta([0, 100], [100], bt, torch.arange(100, dtype=torch.long, device=dev), [True])
    t = lambda x: torch.from_numpy(x).to(torch.bfloat16).to(dev)   # noqa: E731
    att.forward(0, t(q), t(k), t(v), kc, vc, meta)
    q2, k2, v2 = s.draw(20)
    meta2 = E.StepMeta([0, 20], [120], bt, torch.arange(100, 120, dtype=torch.long, device=dev), [True])
    with pytest.raises(ValueError, match="multiple of 128"):
        att.forward(0, t(q2), t(k2), t(v2), kc, vc, meta2)
