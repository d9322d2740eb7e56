"""Golden-shaped entry points: the reference golden model's functions, on the B200 kernels.

    lssab8_attention(q, k, v, mu=None, kb=128, q_exp_mode="row", causal=True, key_valid=None, **kw)
        reference/lssab8_golden.py:341-346
    lssab9_attention(q, k, v, mu=None, kb=128, q_exp_mode="row", causal=True, key_valid=None,
                     sink_alone=False, v_planes=1, v_keyshift=0, ks_round=False, **kw)
        reference/lssab9_golden.py:254-259

q [H, T, dh], k / v [KVH, T, dh] (numpy float arrays, as the golden takes, or torch tensors) ->
float32 [H, T, dh] (numpy for numpy inputs, a CUDA tensor otherwise), bit-identical to the golden.
Keyword options of the golden core that are schedule or debug controls (skip, weight="rn",
rows, heads) are honoured: rows / heads restrict which entries are returned (the others are 0,
as the golden leaves them).  The research arms the golden also carries (weight "tr" / "l16",
kb != 128, B9.2 value planes, B9.3 rounding variants) have no kernel and raise
NotImplementedError.  Computation runs on the current CUDA device; there is no CPU path.
"""
import numpy as np
import torch

from . import lssab8_torch as _B8
from . import attention as A

KB = 128


def _to_dev(x):
    if isinstance(x, torch.Tensor):
        if x.device.type != "cuda":
            raise ValueError("LSSA-B8 on B200 needs CUDA tensors (no CPU fallback exists)")
        return x.float()
    return torch.from_numpy(np.ascontiguousarray(np.asarray(x, np.float32))).cuda()


def _core(q, k, v, mu, kb, q_exp_mode, causal, key_valid, sink, b9grid, v_keyshift, rows, heads, kw):
    _B8.env_contract_check()
    if kb != KB:
        raise NotImplementedError("only the contract's 128-key blocks have a kernel (kb=%r)" % kb)
    if kw.get("weight", "rn") != "rn":
        raise NotImplementedError("the control arms (weight=%r) have no kernel" % kw.get("weight"))
    for opt in ("table", "n", "w_loc", "bhi", "seg", "s_win"):
        if opt in kw:
            raise NotImplementedError("%s is fixed by the contract in these kernels" % opt)
    if kw.get("debug"):
        raise NotImplementedError("debug state is the CPU golden's; use the oracle")
    if q_exp_mode not in ("row", "head"):
        raise ValueError(q_exp_mode)
    numpy_in = not isinstance(q, torch.Tensor)
    qd, kd, vd = _to_dev(q)[None], _to_dev(k)[None], _to_dev(v)[None]
    _, H, T, dh = qd.shape
    KVH = kd.shape[1]
    if kd.shape != (1, KVH, T, dh) or vd.shape != kd.shape or H % KVH:
        raise ValueError("q [H, T, dh], k / v [KVH, T, dh] with KVH dividing H")
    dev = qd.device
    q8, eq = A.quant_rows(qd) if q_exp_mode == "row" else A.quant_heads(qd)
    if mu is not None:
        k8, ek = A.quant_keys_offset(kd, _to_dev(mu))
    else:
        k8, ek, _ = A.quant_blocks(kd, 0)
    vmode = (2 if T > 1 else 1) if sink else (1 if b9grid else 0)
    if v_keyshift:
        if not 1 <= int(v_keyshift) <= 16:
            raise NotImplementedError("v_keyshift above 16 has no kernel")
        if not causal or key_valid is not None:
            raise NotImplementedError("B9.3 runs on the causal form only")
        v8, ev, ev0, d8 = A.quant_values_keyshift(vd, int(v_keyshift), sink)
    else:
        v8, ev, ev0 = A.quant_blocks(vd, vmode)
    ev0 = ev0 if (sink and T > 1) else None
    if v_keyshift:
        out = A.prefill_lattice_keyshift(q8, eq, k8, ek, v8, ev, ev0, d8, T, out_dtype=torch.float32)
    elif causal and key_valid is None:
        out = A.prefill_lattice(q8, eq, k8, ek, v8, ev, ev0, T, out_dtype=torch.float32)
    else:
        km = A.key_mask_words(key_valid, 1, T, dev)
        out = A.prefill_lattice_general(q8, eq, k8, ek, v8, ev, ev0, T, causal, km)
    A.check_device_errors(dev)                  # e_v outside the clamp: AssertionError, as the golden
    res = out[0].transpose(0, 1).contiguous()     # [H, T, dh]
    if rows is not None or heads is not None:
        keep = torch.zeros((H, T), dtype=torch.bool, device=dev)
        hs = slice(None) if heads is None else torch.as_tensor(list(heads), device=dev)
        rs = slice(None) if rows is None else torch.as_tensor(list(rows), device=dev)
        if heads is None:
            keep[:, rs] = True
        elif rows is None:
            keep[hs, :] = True
        else:
            keep[hs[:, None], rs[None, :]] = True
        res = torch.where(keep[..., None], res, torch.zeros((), device=dev))
    return res.cpu().numpy() if numpy_in else res


def lssab8_attention(q, k, v, mu=None, kb=KB, q_exp_mode="row", causal=True, key_valid=None, rows=None,
                     heads=None, skip=True, **kw):
    """PREP + core of LSSA-B8 (reference/lssab8_golden.py:341-346)."""
    return _core(q, k, v, mu, kb, q_exp_mode, causal, key_valid, False, False, 0, rows, heads, kw)


def lssab9_attention(q, k, v, mu=None, kb=KB, q_exp_mode="row", causal=True, key_valid=None, sink_alone=False,
                     v_planes=1, v_keyshift=0, ks_round=False, rows=None, heads=None, skip=True, **kw):
    """LSSA-B9 (reference/lssab9_golden.py:254-259): the B9 value grid (exponents clamped to
    [-32, 48], then asserted inside [-32, 40]); sink_alone = B9.1, key 0 on its own grid."""
    if v_planes != 1:
        raise NotImplementedError("B9.2 value planes have no kernel")
    if ks_round:
        raise NotImplementedError("B9.3 rounding variants have no kernel")
    return _core(q, k, v, mu, kb, q_exp_mode, causal, key_valid, bool(sink_alone), True, v_keyshift, rows, heads, kw)
