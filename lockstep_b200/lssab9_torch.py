"""Drop-in for reference/lssab9_torch.py with its B9.1 `sink_alone` and B9.3 `v_keyshift` options.

make_lssab9_long_attn(..., sink_alone=True) is LSSA-B8 with key 0 of the sequence quantised
alone on the value grid and folded as its own term first in block 0
(reference/lssab9_torch.py:68-327); v_keyshift = dmax (1 .. 16) puts key j of each block on the
finer value grid e_v + d_j, d_j = clamp(e_j - e_v, 0, dmax), and weighs its value by eh_j >> d_j
while l_b keeps eh_j (reference/lssab9_torch.py:145-153, 276-304).  With every option off it is
LSSA-B8 bit for bit, except that the B9 value quantiser clamps exponents to [-32, 48] and then
asserts [-32, 40] (reference/lssab9_torch.py:61,158) -- the same AssertionError is raised here.
The other B9 options (v_planes=2, v_sub, ks_round) have no B200 kernel and raise
NotImplementedError.
"""
from . import attention as _A
from . import lssab8_torch as B8

BHI, KB, SEG_KEYS, S_WIN, W_LOC, NIDX = B8.BHI, B8.KB, B8.SEG_KEYS, B8.S_WIN, B8.W_LOC, B8.NIDX
NB_SENT = B8.NB_SENT


def make_lssab9_long_attn(kb=KB, bhi=BHI, n=NIDX, w_loc=W_LOC, weight="rn", s_win=S_WIN,
                          seg_keys=SEG_KEYS, head_chunk=7, qblk=1024, kblk=8192, mu=None,
                          qexp="row", clamp_sh=True, stats=None, skip=True,
                          sink_alone=False, v_planes=1, v_keyshift=0, ks_round=False, v_sub=1):
    """eager_attention_forward replacement implementing LSSA-B9 (B9.1 sink_alone, B9.3 v_keyshift)."""
    B8._contract_check(kb, bhi, n, w_loc, weight, s_win, seg_keys, mu, qexp, clamp_sh)
    if v_planes != 1 or v_sub != 1 or ks_round:
        raise NotImplementedError("B9.2 / B9.4 value options and B9.3 rounding variants have no B200 kernel")
    if v_keyshift and not 1 <= int(v_keyshift) <= 16:
        raise NotImplementedError("v_keyshift above 16 has no B200 kernel")

    mu_cache = {}

    def attn(module, query, key, value, attention_mask, *args, **kw):
        Bsz, H, T, dh = query.shape
        assert Bsz == 1, "B=1 windows only"
        # B9's value grid is used even with the sink off (clamp 48, assert 40)
        mu_l = B8._mu_for(mu, module, query.device, mu_cache)
        out = _A.prefill(query, key, value, sink=bool(sink_alone), out_dtype=query.dtype, mu=mu_l, qexp=qexp,
                         v_keyshift=int(v_keyshift), b9grid=True)
        return out, None
    return attn


def make_lssab9_attn(head_chunk=16, **kw):
    return make_lssab9_long_attn(head_chunk=head_chunk, qblk=1 << 20, kblk=1 << 20, **kw)


ARM_SPECS = {
    "L9":      dict(sink_alone=False, v_planes=1),
    "L9-sink": dict(sink_alone=True, v_planes=1),
}


def build_arm9(name, bhi=BHI, head_chunk=7, mu=None, qblk=1024, kblk=8192, stats=None, long=True, qexp="row"):
    """reference/lssab9_torch.py:370-376 for the arms with a B200 kernel; None otherwise."""
    spec = ARM_SPECS.get(name)
    if spec is None:
        return None
    if long:
        return make_lssab9_long_attn(head_chunk=head_chunk, qblk=qblk, kblk=kblk, mu=mu, bhi=bhi, stats=stats,
                                     qexp=qexp, **spec)
    return make_lssab9_attn(head_chunk=head_chunk, mu=mu, bhi=bhi, stats=stats, qexp=qexp, **spec)
