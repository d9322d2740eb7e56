"""Drop-in for reference/lssab8_torch.py: the LSSA-B8 eager-attention replacement on B200.

Same entry points, arguments, return value and asserts as the reference module
(reference/lssab8_torch.py:103-310); the arithmetic runs in liblssab8_b200.so (tcgen05 int8 MMA
prefill, sm_100a) and is bit-identical to the reference's.

  make_lssab8_long_attn(...) -> attn(module, query, key, value, attention_mask, ...) -> (out, None)
      query [1, H, T, dh], key/value [1, KVH, T, dh] CUDA tensors (float32/float16/bfloat16,
      contiguous or not); out [1, T, H, dh] in query.dtype, contiguous.  Batch must be 1
      (AssertionError, like the reference); lockstep_b200.attention.prefill is the batched form.
  make_lssab8_attn, ARM_SPECS, build_arm8: as in the reference.

Parameters the reference calls SCHEDULE (head_chunk, qblk, kblk; gate S10) and `skip` (exact,
gate S6) are accepted and do not change a bit.  Contract parameters must be the contract's
values (kb=128, bhi=26, n=7, w_loc=9, weight="rn", s_win=32, seg_keys=4096, clamp_sh=True;
qexp "row" or "head", the per-head query exponent): other arms of the reference (L8-RN-W8, L8-TR, L8-RN-n8, L8-RN-KB64, L16) are
research controls with no B200 kernel and raise NotImplementedError.  A key offset `mu` (a
sequence indexed by the module's layer_idx, each [KVH, dh]) is subtracted from the keys in binary32
before the key quantiser, as the reference does (reference/lssab8_torch.py:116-122, 143-144).
"""
from . import attention as _A

BHI = 26
KB = 128
SEG_KEYS = 32 * 128
S_WIN = 32
W_LOC = 9
NIDX = 7
NB_SENT = -(1 << 58)


# The reference selects a different contract version from the environment when it is imported
# (reference/lssab8_golden.py:57-68, reference/lssab_golden.py:80): LSSAB8_SEG (segment size; 0 =
# single-level fold), LSSAB8_RESCALE=mul (an RN-multiply rescale), LSSAB_TABLE=frac2 (another T2
# table).  The kernels implement the filed contract only, so a session that selects another
# version is refused rather than given the filed function under its name.
_ENV_CONTRACT = (("LSSAB8_SEG", ("", "32")), ("LSSAB8_RESCALE", ("", "field")), ("LSSAB_TABLE", ("", "frac")))


def env_contract_check():
    import os
    for var, ok in _ENV_CONTRACT:
        val = os.environ.get(var, "")
        if val not in ok:
            raise NotImplementedError("%s=%s selects a contract variant with no B200 kernel (only the filed "
                                      "contract: %s unset or %r)" % (var, val, var, ok[1]))


def _contract_check(kb, bhi, n, w_loc, weight, s_win, seg_keys, mu, qexp, clamp_sh):
    env_contract_check()
    assert n <= bhi and qexp in ("row", "head")
    assert seg_keys % kb == 0, "a segment must be a whole number of blocks"
    if (kb, bhi, n, w_loc, weight, s_win, seg_keys, bool(clamp_sh)) != (KB, BHI, NIDX, W_LOC, "rn", S_WIN,
                                                                        SEG_KEYS, True):
        raise NotImplementedError("only the LSSA-B8 contract arm (L8 = L8-RN-W9) has a B200 kernel")


def _mu_for(mu, module, device, cache=None):
    """The layer's key offset mu[layer_idx] [KVH, dh] as float32 on `device`, or None.  `cache`
    (one dict per attention closure, as in reference/lssab8_torch.py:116-122) keeps the copies."""
    if mu is None:
        return None
    import torch
    li = int(getattr(module, "layer_idx", -1))
    key = (li, str(device))
    if cache is not None and key in cache:
        return cache[key]
    t = torch.as_tensor(mu[li]).to(device=device, dtype=torch.float32).contiguous()
    if cache is not None:
        cache[key] = t
    return t


def _attn_closure(sink, mu=None, qexp="row"):
    mu_cache = {}

    def attn(module, query, key, value, attention_mask, *args, **kw):
        Bsz, H, T, dh = query.shape
        assert Bsz == 1, "B=1 windows only"
        out = _A.prefill(query, key, value, sink=sink, out_dtype=query.dtype,
                         mu=_mu_for(mu, module, query.device, mu_cache), qexp=qexp)
        return out, None
    return attn


def make_lssab8_long_attn(kb=KB, bhi=BHI, n=NIDX, w_loc=W_LOC, weight="rn", s_win=S_WIN,
                          seg_keys=SEG_KEYS, head_chunk=7, qblk=1024, kblk=8192, mu=None,
                          qexp="row", clamp_sh=True, stats=None, skip=True):
    """eager_attention_forward replacement implementing LSSA-B8 (reference/lssab8_torch.py:103-272).

    `stats` (the reference's debug counters) is not collected by the kernels and stays untouched."""
    _contract_check(kb, bhi, n, w_loc, weight, s_win, seg_keys, mu, qexp, clamp_sh)
    return _attn_closure(sink=False, mu=mu, qexp=qexp)


def make_lssab8_attn(kb=KB, bhi=BHI, n=NIDX, w_loc=W_LOC, weight="rn", head_chunk=16,
                     mu=None, qexp="row", stats=None, **kw):
    """Short-context entry point (reference/lssab8_torch.py:275-281): the same function."""
    return make_lssab8_long_attn(kb=kb, bhi=bhi, n=n, w_loc=w_loc, weight=weight,
                                 head_chunk=head_chunk, qblk=1 << 20, kblk=1 << 20,
                                 mu=mu, qexp=qexp, stats=stats, **kw)


ARM_SPECS = {
    "L8":          dict(kb=128, n=7, w_loc=9, weight="rn"),
    "L8-RN-W9":    dict(kb=128, n=7, w_loc=9, weight="rn"),
    "L8-RN-W8":    dict(kb=128, n=7, w_loc=8, weight="rn"),
    "L8-TR":       dict(kb=128, n=7, w_loc=9, weight="tr"),
    "L8-RN-n8":    dict(kb=128, n=8, w_loc=9, weight="rn"),
    "L8-RN-KB64":  dict(kb=64,  n=7, w_loc=9, weight="rn"),
    "L16":         dict(kb=128, n=13, w_loc=16, weight="l16"),
}


def build_arm8(name, bhi=BHI, head_chunk=7, mu=None, qblk=1024, kblk=8192, stats=None,
               long=True, qexp="row"):
    """Return an eager_attention_forward for an LSSA-B8 arm, or None if `name` is not one
    (reference/lssab8_torch.py:296-310).  Control arms raise NotImplementedError."""
    spec = ARM_SPECS.get(name)
    if spec is None:
        return None
    sk = dict(spec)
    if long:
        return make_lssab8_long_attn(head_chunk=head_chunk, qblk=qblk, kblk=kblk, mu=mu,
                                     bhi=bhi, stats=stats, qexp=qexp, **sk)
    return make_lssab8_attn(head_chunk=head_chunk, mu=mu, bhi=bhi, stats=stats, qexp=qexp, **sk)
