"""CPU oracle for LSSA-B8 / B9.1 attention -- TEST INFRASTRUCTURE ONLY.

ctypes front end of ``liblssab8_oracle.so`` (``lssab8_oracle.c``), a plain-C restatement of
the reference's numpy golden.  Only ``tests/``, ``__graft_entry__.smoke()`` and
``bench.py``'s CPU-baseline leg may import this package, and only as the checker; the
product path (``lockstep_b200``) never touches it.

Parity: PINNED against digests and vectors produced by the reference itself
(``tests/golden/make_golden.py``); ``tests/test_oracle.py`` is the pin.

Array conventions follow the reference golden (``reference/lssab8_golden.py:341``):
``q [H, T, dh]``, ``k, v [KVH, T, dh]`` float32, output ``[H, T, dh]`` float32.  Exponent
arrays are kv-head major (``ek[KVH, nblk]``), the transpose of the golden's ``[nblk, KVH]``.
"""
import ctypes
import os
import subprocess

import numpy as np

KB = 128          # reference/lssab8_golden.py:55
SEG = 32          # reference/lssab8_golden.py:56
BHI = 26          # reference/lssab8_golden.py:54
T2_DIGEST = "7a42a785940f557d5d5a4188fa5683ea00cf8b29e8d5213c75c581a5a0d92fbb"

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIBPATH = os.path.join(_HERE, "liblssab8_oracle.so")
_lib = None


def build(force=False):
    """Compile the oracle library in place (gcc; see ``oracle/Makefile``)."""
    src = os.path.join(_HERE, "lssab8_oracle.c")
    if force or not os.path.exists(_LIBPATH) or os.path.getmtime(_LIBPATH) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIBPATH


def lib():
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(_LIBPATH)
        P = ctypes.c_void_p
        L.or_t2_table.argtypes = [P, ctypes.c_int]
        L.or_quant_rows.argtypes = [P, ctypes.c_int64, ctypes.c_int, P, P]
        L.or_quant_blocks.argtypes = [P, ctypes.c_int, ctypes.c_int, ctypes.c_int, P, P, P]
        L.or_quant_blocks.restype = ctypes.c_int
        L.or_gbase.argtypes = [ctypes.c_int]
        L.or_gbase.restype = ctypes.c_int64
        L.or_core.argtypes = [ctypes.c_int] * 4 + [P] * 8 + [ctypes.c_int] * 3 + [P, ctypes.c_int] + [P] * 4 + [ctypes.c_int] * 2 + [P]
        L.or_core.restype = ctypes.c_int
        _lib = L
    return _lib


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def nthreads_default():
    return os.cpu_count() or 1


def t2_table():
    """The 2,176-entry T2 table (reference/lssab8_golden.py:90-103)."""
    out = np.zeros(17 * 128, np.uint8)
    lib().or_t2_table(_p(out), out.size)
    return out


def table_digest(t):
    """sha256 of the ASCII csv of the table (reference/lssab8_golden.py:117-119)."""
    import hashlib
    return hashlib.sha256(",".join(str(int(x)) for x in np.asarray(t).ravel()).encode()).hexdigest()


def gbase(dh):
    return int(lib().or_gbase(int(dh)))


def quant_rows(x):
    """P1 (reference/t10_attn.py:40-48): x [..., dh] f32 -> (q8 int8 [..., dh], e int32 [...])."""
    x = np.ascontiguousarray(x, np.float32)
    dh = x.shape[-1]
    n = x.size // dh
    q8 = np.zeros(x.shape, np.int8)
    e = np.zeros(x.shape[:-1], np.int32)
    lib().or_quant_rows(_p(x), n, dh, _p(q8), _p(e))
    return q8, e


def quant_blocks(x, mode=0):
    """P2/P3 per kv head (reference/lssab_torch.py:62-85, reference/lssab9_torch.py:46-65,124-132).

    x [KVH, T, dh] f32; mode 0 = B8 grid, 1 = B9 value grid, 2 = B9.1 sink_alone value grid.
    Returns (x8 int8 [KVH, T, dh], e int32 [KVH, nblk], e0 int32 [KVH], err int)."""
    x = np.ascontiguousarray(x, np.float32)
    KVH, T, dh = x.shape
    nblk = (T + KB - 1) // KB
    x8 = np.zeros(x.shape, np.int8)
    e = np.zeros((KVH, nblk), np.int32)
    e0 = np.zeros(KVH, np.int32)
    err = 0
    for g in range(KVH):
        xg = np.ascontiguousarray(x[g])
        x8g = np.zeros((T, dh), np.int8)
        eg = np.zeros(nblk, np.int32)
        e0g = np.zeros(1, np.int32)
        err |= lib().or_quant_blocks(_p(xg), T, dh, mode, _p(x8g), _p(eg), _p(e0g))
        x8[g] = x8g
        e[g] = eg
        e0[g] = e0g[0]
    return x8, e, e0, err


def prep(q, k, v, sink=False, mu=None, v_keyshift=0, q_exp_mode="row"):
    """PREP of reference/lssab_golden.py:214-235 (+ B9 value grid when sink is on).  mu [KVH, dh]:
    the key offset, k' = fl32(k - mu) before the key quantiser (reference/lssab_golden.py:221).
    v_keyshift = dmax > 0: B9.3 (reference/lssab9_golden.py:37-70), key j of block b quantised on
    the grid e_v[b] + d_j, d_j = clamp(e_j - e_v[b], 0, dmax) with e_j the key's own exponent on
    the B9 value grid; returns d8 [KVH, T] for the PV weight shift.  q_exp_mode "head": one query
    exponent per head over all its rows and channels (reference/lssab_golden.py:230-232)."""
    if mu is not None:
        k = (np.asarray(k, np.float32) - np.asarray(mu, np.float32)[:, None, :]).astype(np.float32)
    T = q.shape[1]
    if q_exp_mode == "row":
        q8, eq = quant_rows(q)
    elif q_exp_mode == "head":
        qf = np.ascontiguousarray(q, np.float32)
        q8f, eh = quant_rows(qf.reshape(qf.shape[0], -1))     # the same rule over a whole head
        q8, eq = q8f.reshape(qf.shape), np.repeat(eh[:, None], T, axis=1).astype(np.int32)
    else:
        raise ValueError(q_exp_mode)
    k8, ek, _, _ = quant_blocks(k, 0)
    if sink:
        v8, ev, ev0, err = quant_blocks(v, 2 if T > 1 else 1)
        if err:
            raise AssertionError("e_v outside the contract clamp")
        ev0 = ev0 if T > 1 else None
    elif v_keyshift:
        v8, ev, _, err = quant_blocks(v, 1)             # the B9 value grid, sink off
        if err:
            raise AssertionError("e_v outside the contract clamp")
        ev0 = None
    else:
        v8, ev, _, _ = quant_blocks(v, 0)
        ev0 = None
    d8 = None
    if v_keyshift:
        v8, d8 = _keyshift(v, ev, ev0, int(v_keyshift))
    return dict(q8=q8, eq=eq, k8=k8, ek=ek, v8=v8, ev=ev, ev0=ev0, d8=d8)


def _keyshift(v, ev, ev0, dmax):
    """B9.3 values and shifts (reference/lssab9_golden.py:59-69): each key's own exponent is the B9
    value-grid exponent of that key alone (a one-key block); v8 = clamp(rint(v 2^(e_v + d)), +-127)."""
    v = np.ascontiguousarray(v, np.float32)
    KVH, T, dh = v.shape
    ekey = np.zeros((KVH, T), np.int64)
    for g in range(KVH):
        for j in range(T):
            _, e1, _, _ = quant_blocks(v[g:g + 1, j:j + 1], 1)
            ekey[g, j] = e1[0, 0]
    ev_tok = np.repeat(np.asarray(ev, np.int64), KB, axis=1)[:, :T]
    if ev0 is not None:
        ev_tok = ev_tok.copy()
        ev_tok[:, 0] = np.asarray(ev0, np.int64)
    d8 = np.clip(ekey - ev_tok, 0, dmax).astype(np.int64)
    sc = np.ldexp(np.float32(1.0), (ev_tok + d8).astype(np.int32)).astype(np.float32)
    v8 = np.clip(np.rint(v * sc[..., None]), -127.0, 127.0).astype(np.int8)
    return v8, d8.astype(np.int8)


def core(p, causal=True, rows=None, key_lo=0, key_hi=None, debug=False, nthreads=None, qrow=-1, key_valid=None):
    """The recurrence (reference/lssab8_golden.py:200-338, reference/lssab9_golden.py:189-224).

    qrow >= 0: p["q8"] is [H, 1, dh] (one query row per head standing at position qrow) and
    the result is [H, 1, dh].  key_valid: [T] bool mask of the keys every row may see
    (reference/lssab8_golden.py:245-246), or None."""
    q8 = np.ascontiguousarray(p["q8"], np.int8)
    k8 = np.ascontiguousarray(p["k8"], np.int8)
    KVH, T, dh = k8.shape
    H = q8.shape[0]
    eq = np.ascontiguousarray(p["eq"], np.int32)
    ek = np.ascontiguousarray(p["ek"], np.int32)
    v8 = np.ascontiguousarray(p["v8"], np.int8)
    ev = np.ascontiguousarray(p["ev"], np.int32)
    ev0 = p.get("ev0")
    ev0 = None if ev0 is None else np.ascontiguousarray(ev0, np.int32)
    d8 = p.get("d8")
    d8 = None if d8 is None else np.ascontiguousarray(d8, np.int8)
    nq = 1 if qrow >= 0 else T
    out = np.zeros((H, nq, dh), np.float32)
    dO = np.zeros((H, nq, dh), np.float32) if debug else None
    dl = np.zeros((H, nq), np.float32) if debug else None
    dnb = np.zeros((H, nq), np.int64) if debug else None
    r = None if rows is None else np.ascontiguousarray(rows, np.int32)
    kvm = None if key_valid is None else np.ascontiguousarray(np.asarray(key_valid, bool), np.uint8)
    if kvm is not None and kvm.shape != (T,):
        raise ValueError("key_valid must be [T]")
    nt = nthreads or nthreads_default()
    rc = lib().or_core(H, KVH, T, dh, _p(q8), _p(eq), _p(k8), _p(ek), _p(v8), _p(ev),
                       None if ev0 is None else _p(ev0), None if d8 is None else _p(d8), int(causal), int(key_lo),
                       int(T if key_hi is None else key_hi),
                       None if r is None else _p(r), 0 if r is None else len(r), _p(out),
                       None if dO is None else _p(dO), None if dl is None else _p(dl),
                       None if dnb is None else _p(dnb), nt, int(qrow), None if kvm is None else _p(kvm))
    if rc != 0:
        raise ValueError("oracle core rejected the shapes")
    if debug:
        return out, dict(O=dO, l=dl, nb=dnb)
    return out


def attention(q, k, v, sink=False, causal=True, rows=None, nthreads=None, mu=None, v_keyshift=0, key_valid=None,
              q_exp_mode="row"):
    """lssab8_attention / lssab9_attention(sink_alone) (reference/lssab8_golden.py:341,
    reference/lssab9_golden.py:254): q [H,T,dh], k/v [KVH,T,dh] -> f32 [H,T,dh]."""
    p = prep(np.asarray(q, np.float32), np.asarray(k, np.float32), np.asarray(v, np.float32), sink, mu=mu,
             v_keyshift=v_keyshift, q_exp_mode=q_exp_mode)
    return core(p, causal=causal, rows=rows, nthreads=nthreads, key_valid=key_valid)


def f32_to_bf16_bits(x):
    """RNE float32 -> bfloat16 bits (reference/lssab_golden.py:203-211)."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    r = u + 0x7FFF + ((u >> 16) & 1)
    out = ((r >> 16) & 0xFFFF).astype(np.uint16)
    nan = np.isnan(np.asarray(x, np.float32))
    return np.where(nan, np.uint16(0x7FC0), out)


def bf16_bits_to_f32(b):
    return (np.asarray(b, np.uint16).astype(np.uint32) << 16).view(np.float32)


def prefill_bsz(query, key, value, sink=False, nthreads=None):
    """Batched form of the torch drop-in (reference/lssab8_torch.py:134-271 per batch element):
    query [B,H,T,dh], key/value [B,KVH,T,dh] f32 (values of the caller's dtype) -> f32
    [B,T,H,dh] before the cast to the caller's dtype."""
    B = query.shape[0]
    outs = []
    for b in range(B):
        o = attention(query[b], key[b], value[b], sink=sink, nthreads=nthreads)
        outs.append(np.ascontiguousarray(o.transpose(1, 0, 2)))
    return np.stack(outs)


def decode_rows(q_new, key, value, sink=False, nthreads=None):
    """Decode oracle: one new query row per sequence attending to all L keys.

    q_new [H, dh] f32, key/value [KVH, L, dh] f32 -> f32 [H, dh].  This is row L-1 of the
    prefill (contract v2, decode row == prefill row, reference/lssab8_selftest.py:320-336)
    evaluated alone: rows=[L-1] (reference/lssab8_golden.py:207-209)."""
    H, dh = q_new.shape
    KVH, L, _ = key.shape
    q8r, eqr = quant_rows(q_new)
    k8, ek, _, _ = quant_blocks(key, 0)
    if sink:
        v8, ev, ev0, err = quant_blocks(value, 2 if L > 1 else 1)
        if err:
            raise AssertionError("e_v outside the contract clamp")
        ev0 = ev0 if L > 1 else None
    else:
        v8, ev, _, _ = quant_blocks(value, 0)
        ev0 = None
    p = dict(q8=q8r[:, None, :], eq=eqr[:, None], k8=k8, ek=ek, v8=v8, ev=ev, ev0=ev0)
    o = core(p, causal=True, qrow=L - 1, nthreads=nthreads)
    return o[:, 0]
