"""Seeded synthetic inputs with the shapes of the five LSSA-B8 benchmark configurations.

No public dataset is involved: every tensor is drawn from numpy's ``Generator(PCG64(seed))``
(stable across torch versions, unlike ``torch.randn``) as float32 ``standard_normal`` and
rounded to bfloat16 with round-to-nearest-even.  Draw order is fixed per config and
documented on each generator, so a digest of the inputs pins the workload.

  cfg 1  causal prefill   B=1  H=8  KVH=8 dh=64  T=128                       sink off
  cfg 2  causal prefill   B=4  H=32 KVH=8 dh=128 T=2048, 1% K channels x8    sink off
  cfg 3  split-KV decode  B=32 H=32 KVH=8 dh=128 L=8192, 16 splits            sink off / on
  cfg 4  causal prefill   B=8  H=64 KVH=8 dh=128 T=8192, sharded by kv group  sink off
  cfg 5  paged decode     B=64 H=32 KVH=4 dh=128 L~U[1024,32768], page 16     sink on
"""
import numpy as np

CONFIGS = {
    1: dict(kind="prefill", B=1, H=8, KVH=8, dh=64, T=128, outliers=0.0, sink=False),
    2: dict(kind="prefill", B=4, H=32, KVH=8, dh=128, T=2048, outliers=0.01, sink=False),
    3: dict(kind="decode", B=32, H=32, KVH=8, dh=128, L=8192, nsplit=16, sink=False),
    4: dict(kind="prefill", B=8, H=64, KVH=8, dh=128, T=8192, outliers=0.0, sink=False),
    5: dict(kind="paged_decode", B=64, H=32, KVH=4, dh=128, Lmin=1024, Lmax=32768, page=16,
            sink=True),
}


def bf16_round(x):
    """float32 -> float32 holding the nearest bfloat16 (ties to even)."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    return r.astype(np.uint32).view(np.float32)


def _normal_bf16(rng, shape):
    return bf16_round(rng.standard_normal(shape, dtype=np.float32))


def prefill_inputs(B, H, KVH, T, dh, outliers=0.0, seed=0):
    """q [B,H,T,dh], k/v [B,KVH,T,dh] float32 holding bf16 values.

    Draw order: q, k, v (each standard_normal float32 -> bf16), then for each kv head g the
    outlier channels ``rng.choice(dh, n, replace=False)`` with n = ceil(outliers*dh); those
    channels of k[:, g] are multiplied by 8 (exact in bf16)."""
    rng = np.random.Generator(np.random.PCG64(seed))
    q = _normal_bf16(rng, (B, H, T, dh))
    k = _normal_bf16(rng, (B, KVH, T, dh))
    v = _normal_bf16(rng, (B, KVH, T, dh))
    if outliers > 0:
        n = int(np.ceil(outliers * dh))
        for g in range(KVH):
            ch = rng.choice(dh, size=n, replace=False)
            k[:, g, :, ch] *= np.float32(8.0)
    return q, k, v


def decode_inputs(B, H, KVH, L, dh, seed=0):
    """q_new [B,H,dh], k/v [B,KVH,L,dh] float32 holding bf16 values; draw order q, k, v.
    The new token's own key/value is position L-1 of k/v."""
    rng = np.random.Generator(np.random.PCG64(seed))
    q = _normal_bf16(rng, (B, H, dh))
    k = _normal_bf16(rng, (B, KVH, L, dh))
    v = _normal_bf16(rng, (B, KVH, L, dh))
    return q, k, v


def ragged_lengths(B, Lmin, Lmax, seed=0):
    """Per-sequence KV lengths, uniform in [Lmin, Lmax] (first draw of a fresh PCG64(seed))."""
    rng = np.random.Generator(np.random.PCG64(seed))
    return rng.integers(Lmin, Lmax, size=B, endpoint=True).astype(np.int64)


def ragged_inputs(B, H, KVH, dh, lengths, seed=0):
    """Draws for the paged/ragged decode: q_new [B,H,dh] then, per sequence b in order,
    k_b [KVH,L_b,dh] and v_b [KVH,L_b,dh].  Uses a PCG64 stream independent of the length
    draw (seed + 1) so the lengths can be drawn alone."""
    rng = np.random.Generator(np.random.PCG64(seed + 1))
    q = _normal_bf16(rng, (B, H, dh))
    ks, vs = [], []
    for b in range(B):
        L = int(lengths[b])
        ks.append(_normal_bf16(rng, (KVH, L, dh)))
        vs.append(_normal_bf16(rng, (KVH, L, dh)))
    return q, ks, vs


def page_table(lengths, page, seed=0):
    """A random block table: the pages of all sequences, in sequence order, are a seeded
    permutation of the pool [0, total_pages).  Returns (block_table [B, max_pages] int32 with
    -1 padding, total_pages)."""
    npages = [(int(L) + page - 1) // page for L in lengths]
    total = int(sum(npages))
    rng = np.random.Generator(np.random.PCG64(seed + 2))
    perm = rng.permutation(total).astype(np.int32)
    bt = np.full((len(lengths), max(npages)), -1, np.int32)
    o = 0
    for b, n in enumerate(npages):
        bt[b, :n] = perm[o:o + n]
        o += n
    return bt, total


def prefill_inputs_shard(B, H, KVH, T, dh, heads, kv_heads, outliers=0.0, seed=0, pin=False):
    """The slice [:, h0:h1] of q and [:, g0:g1] of k and v from prefill_inputs, bit for bit, as
    bfloat16 torch tensors (heads = (h0, h1), kv_heads = (g0, g1)), without holding the whole
    arrays: the stream is drawn in the same order, one [T, dh] piece at a time (consecutive draws
    from one Generator continue one stream, so the pieces are the whole array's draws), and
    only this shard's pieces are kept.  pin: allocate the results in pinned host memory."""
    import torch
    h0, h1 = heads
    g0, g1 = kv_heads
    rng = np.random.Generator(np.random.PCG64(seed))

    def draw(nh, lo, hi):
        out = torch.empty((B, hi - lo, T, dh), dtype=torch.bfloat16, pin_memory=pin)
        for b in range(B):
            for x in range(nh):
                piece = rng.standard_normal((T, dh), dtype=np.float32)
                if lo <= x < hi:
                    out[b, x - lo] = torch.from_numpy(piece)     # float32 -> bfloat16 is RNE
        return out

    q = draw(H, h0, h1)
    k = draw(KVH, g0, g1)
    v = draw(KVH, g0, g1)
    if outliers > 0:
        n = int(np.ceil(outliers * dh))
        for g in range(KVH):
            ch = rng.choice(dh, size=n, replace=False)
            if g0 <= g < g1:
                k[:, g - g0, :, ch] *= 8.0                        # exact in bf16
    return q, k, v


def ragged_inputs_shard(B, H, KVH, dh, lengths, seqs, seed=0):
    """ragged_inputs restricted to the sequences `seqs`: returns (q [B, H, dh] float32 of every
    sequence, {b: (k_b, v_b)} float32 [KVH, L_b, dh] for b in seqs); the other sequences' draws
    are made and dropped, so the kept values equal ragged_inputs' bit for bit."""
    want = set(int(b) for b in seqs)
    rng = np.random.Generator(np.random.PCG64(seed + 1))
    q = _normal_bf16(rng, (B, H, dh))
    kv = {}
    for b in range(B):
        L = int(lengths[b])
        if b in want:
            kv[b] = (_normal_bf16(rng, (KVH, L, dh)), _normal_bf16(rng, (KVH, L, dh)))
        else:
            for _ in range(2 * KVH):
                rng.standard_normal((L, dh), dtype=np.float32)
    return q, kv
