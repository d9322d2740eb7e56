"""Test fixtures that restate the reference selftest's case generators.

Each generator draws exactly the arrays the reference selftest draws
(``reference/lssab8_selftest.py:157-241``, ``reference/lssab9_selftest.py:44-48``), so the
reference's own outputs on them -- recorded as digests in ``tests/golden/`` by
``tests/golden/make_golden.py`` -- pin the oracle and the CUDA path.  ``make_golden.py``
asserts that these constructors reproduce the reference's arrays bit for bit before it
records anything.
"""
import numpy as np

KB = 128
BHI = 26


def g_base(dh=128):
    import math
    return round((2.0 ** BHI) / (math.sqrt(dh) * math.log(2.0)))


def qk_from_scores(S, dh=128, pin_block=KB):
    """One query row and T keys whose quantisation is the identity (e_q = e_k = 0) and whose
    int8 scores equal S [1, T] exactly (construction of reference/lssab_selftest.py:25-41):
    q = [64, 1, ..., 1, 0]; key j = [a_j, r_j, 0, ..., 0] with S_j = 64 a_j + r_j; one key per
    block carries 127 in the channel q zeroes, pinning the block amax to 127."""
    Tq, Tk = S.shape
    assert Tq == 1
    q = np.zeros((1, 1, dh), np.float32)
    q[0, 0, 0] = 64.0
    q[0, 0, 1:dh - 1] = 1.0
    k = np.zeros((1, Tk, dh), np.float32)
    a = np.clip(np.round(S[0] / 64.0), -127, 127)
    r = S[0] - 64 * a
    assert np.abs(r).max() <= 127
    k[0, :, 0] = a
    k[0, :, 1] = r
    for b in range(0, Tk, pin_block):
        k[0, b, dh - 1] = 127.0
    return q, k


def random_cases():
    cs = []
    for T in (256, 320, 512, 1000, 1024, 2048):
        for (H, KVH) in ((1, 1), (4, 2), (7, 1)):
            g = np.random.RandomState(1000 + T + H)
            cs.append(dict(tag="rand_T%d_H%dx%d" % (T, H, KVH),
                           q=g.standard_normal((H, T, 128)).astype(np.float32),
                           k=g.standard_normal((KVH, T, 128)).astype(np.float32),
                           v=g.standard_normal((KVH, T, 128)).astype(np.float32)))
    return cs


def jump_cases():
    cs = []
    G = g_base(128)
    for jump in (50, 126, 127, 200, 400):
        dS = int(round(jump * (1 << BHI) / G))
        for T in (512, 1024):
            S = np.zeros((1, T), np.int64)
            for b in range(T // KB):
                S[0, b * KB:(b + 1) * KB] = (b % 2) * dS - np.arange(KB) % 37
            S = np.clip(S, -8255, 8255)
            q1, k1 = qk_from_scores(S)
            q = np.zeros((1, T, 128), np.float32)
            q[0] = q1[0, 0][None, :]
            g = np.random.RandomState(7 * T + jump)
            v = (g.standard_normal((1, T, 128)) * 8).astype(np.float32)
            cs.append(dict(tag="jump%d_T%d" % (jump, T), q=q, k=k1, v=v))
    return cs


def ftz_cases():
    cs = []
    for sp in (0, 8, 16, 24, 32, 40):
        T = 512
        g = np.random.RandomState(555 + sp)
        v = g.standard_normal((1, T, 128)).astype(np.float32)
        for b in range(0, T, KB):
            v[:, b:b + KB] *= np.float32(2.0 ** (-(b // KB) * sp))
        cs.append(dict(tag="ftz_evladder_%d" % sp,
                       q=g.standard_normal((2, T, 128)).astype(np.float32),
                       k=g.standard_normal((1, T, 128)).astype(np.float32), v=v))
    T = 384
    g = np.random.RandomState(99)
    v = g.standard_normal((1, T, 128)).astype(np.float32)
    v[:, :KB] *= np.float32(2.0 ** 30)
    v[:, KB:2 * KB] *= np.float32(2.0 ** -30)
    cs.append(dict(tag="ftz_extreme_v", q=g.standard_normal((2, T, 128)).astype(np.float32),
                   k=g.standard_normal((1, T, 128)).astype(np.float32), v=v))
    return cs


def degenerate_cases():
    cs = []
    for T in (1, 2, 128, 129, 130, 255, 257, 384):
        g = np.random.RandomState(31 * T)
        cs.append(dict(tag="deg_T%d" % T,
                       q=g.standard_normal((2, T, 128)).astype(np.float32),
                       k=g.standard_normal((1, T, 128)).astype(np.float32),
                       v=g.standard_normal((1, T, 128)).astype(np.float32)))
    for val in (0, 137, -55):
        T = 256
        S = np.full((1, T), val, np.int64)
        q1, k1 = qk_from_scores(S)
        q = np.zeros((1, T, 128), np.float32)
        q[0] = q1[0, 0][None, :]
        g = np.random.RandomState(abs(val) + 5)
        cs.append(dict(tag="ties_%d" % val, q=q, k=k1,
                       v=g.standard_normal((1, T, 128)).astype(np.float32)))
    T = 512
    S = np.random.RandomState(3).randint(-20, 20, size=(1, T)).astype(np.int64)
    S[0, KB:2 * KB] = -8000
    S[0, T - 1] = 300
    q1, k1 = qk_from_scores(S)
    q = np.zeros((1, T, 128), np.float32)
    q[0] = q1[0, 0][None, :]
    cs.append(dict(tag="dead_block", q=q, k=k1,
                   v=np.random.RandomState(4).standard_normal((1, T, 128)).astype(np.float32)))
    return cs


def sink300_cases():
    """reference/lssab9_selftest.py:44-48: key 0's value x300."""
    rng = np.random.default_rng(9)
    cs = []
    for T in (1, 2, 128, 129, 300):
        q = rng.standard_normal((4, T, 128)).astype(np.float32)
        k = rng.standard_normal((2, T, 128)).astype(np.float32)
        v = rng.standard_normal((2, T, 128)).astype(np.float32)
        v[:, 0] *= 300.0
        cs.append(dict(tag="sink300_T%d" % T, q=q, k=k, v=v))
    return cs


def all_cases():
    return random_cases() + jump_cases() + ftz_cases() + degenerate_cases()


def digest(a):
    import hashlib
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def mu_cases():
    """Inputs for the key-offset (mu) gate: keys carry a large per-channel offset, as real keys do,
    and mu [KVH, dh] removes most of it (float32; the offset stays inexact, so the binary32
    subtraction is exercised)."""
    out = []
    for tag, seed, H, KVH, T, dh in (("mu_h4kv2_t300_d64", 21, 4, 2, 300, 64),
                                     ("mu_h4kv1_t257_d128", 22, 4, 1, 257, 128)):
        g = np.random.RandomState(seed)
        off = (g.standard_normal((KVH, dh)) * 6.0).astype(np.float32)
        q = g.standard_normal((H, T, dh)).astype(np.float32)
        k = (g.standard_normal((KVH, T, dh)) + off[:, None, :]).astype(np.float32)
        v = g.standard_normal((KVH, T, dh)).astype(np.float32)
        mu = (off + g.standard_normal((KVH, dh)).astype(np.float32) * np.float32(0.1)).astype(np.float32)
        out.append(dict(tag=tag, q=q, k=k, v=v, mu=mu))
    return out


def keyshift_cases():
    """Inputs for B9.3 v_keyshift: value rows whose magnitudes differ by up to 2^6 inside a block,
    so the per-key shift d_j = clamp(e_j - e_v, 0, dmax) takes several values."""
    out = []
    for tag, seed, H, KVH, T, dh, dmax in (("ks_h4kv2_t300_d64_k3", 31, 4, 2, 300, 64, 3),
                                           ("ks_h2kv1_t200_d128_k6", 32, 2, 1, 200, 128, 6)):
        g = np.random.RandomState(seed)
        q = g.standard_normal((H, T, dh)).astype(np.float32)
        k = g.standard_normal((KVH, T, dh)).astype(np.float32)
        scale = np.exp2(-g.randint(0, 7, size=(KVH, T, 1))).astype(np.float32)
        v = (g.standard_normal((KVH, T, dh)).astype(np.float32) * scale).astype(np.float32)
        out.append(dict(tag=tag, q=q, k=k, v=v, dmax=dmax))
    return out


def mask_cases():
    """Inputs for the golden entry points' general forms: causal off, a key_valid mask (random;
    a whole block masked; key 0 masked; rows that see no key at all), the per-head query exponent
    (q_exp_mode "head"), and a non-causal row spanning more than one 32-block fold segment.
    Each case: tag, q/k/v float32, causal, key_valid ([T] bool or None), q_exp_mode."""
    out = []

    def draw(seed, H, KVH, T, dh):
        g = np.random.RandomState(seed)
        q = g.standard_normal((H, T, dh)).astype(np.float32)
        k = g.standard_normal((KVH, T, dh)).astype(np.float32)
        v = g.standard_normal((KVH, T, dh)).astype(np.float32)
        return g, q, k, v

    g, q, k, v = draw(41, 4, 2, 300, 64)
    out.append(dict(tag="noncausal_h4kv2_t300_d64", q=q, k=k, v=v, causal=False, key_valid=None, q_exp_mode="row"))
    g, q, k, v = draw(42, 4, 2, 260, 128)
    kv = g.rand(260) < 0.7
    out.append(dict(tag="kvrandom_h4kv2_t260_d128", q=q, k=k, v=v, causal=True, key_valid=kv, q_exp_mode="row"))
    g, q, k, v = draw(43, 2, 1, 400, 128)
    kv = np.ones(400, bool)
    kv[128:256] = False                      # block 1 fully masked
    kv[0] = False                            # key 0 masked (the sink's key)
    kv[300:310] = False
    out.append(dict(tag="kvblock_h2kv1_t400_d128", q=q, k=k, v=v, causal=True, key_valid=kv, q_exp_mode="row"))
    g, q, k, v = draw(44, 4, 1, 200, 64)
    kv = np.ones(200, bool)
    kv[:20] = False                          # rows 0..19 see no key (causal): output 0
    out.append(dict(tag="kvempty_h4kv1_t200_d64", q=q, k=k, v=v, causal=True, key_valid=kv, q_exp_mode="row"))
    g, q, k, v = draw(45, 4, 2, 333, 64)
    kv = g.rand(333) < 0.5
    out.append(dict(tag="noncausal_kv_h4kv2_t333_d64", q=q, k=k, v=v, causal=False, key_valid=kv, q_exp_mode="row"))
    g, q, k, v = draw(46, 4, 2, 200, 128)
    q[1] *= np.float32(9.0)                  # one head with a different scale
    out.append(dict(tag="qhead_h4kv2_t200_d128", q=q, k=k, v=v, causal=True, key_valid=None, q_exp_mode="head"))
    g, q, k, v = draw(47, 1, 1, 4200, 64)
    out.append(dict(tag="noncausal_h1kv1_t4200_d64", q=q, k=k, v=v, causal=False, key_valid=None, q_exp_mode="row"))
    return out
