"""Host layer over the C ABI: device buffers, streams and error checks for the prefill path.

PyTorch is used only for device memory and the current CUDA stream; every computation runs in
liblssab8_b200.so.  Tensors must be CUDA tensors of one floating dtype (float32 / float16 /
bfloat16); anything else raises -- there is no CPU path.
"""
import ctypes

import torch

from . import _lib

_DT = {torch.float32: _lib.DT_F32, torch.float16: _lib.DT_F16, torch.bfloat16: _lib.DT_BF16}
KB = 128


def dtype_code(dt):
    try:
        return _DT[dt]
    except KeyError:
        raise TypeError("LSSA-B8 kernels take float32, float16 or bfloat16 tensors, got %s" % dt) from None


def _stream_handle(device):
    return torch.cuda.current_stream(device).cuda_stream


def _require_cuda(*ts):
    for t in ts:
        if not isinstance(t, torch.Tensor) or t.device.type != "cuda":
            raise ValueError("LSSA-B8 on B200 needs CUDA tensors (no CPU fallback exists)")
    dev = ts[0].device
    if any(t.device != dev for t in ts):
        raise ValueError("all tensors must be on the same CUDA device")
    return dev


def tpad(T):
    return ((T + KB - 1) // KB) * KB


def check_device_errors(device=None):
    """Raise if a kernel on this device set the device error word (then clear it).

    e_v outside [-32, 40] raises AssertionError, mirroring the reference's assert
    (reference/lssab9_torch.py:158); other bits raise RuntimeError."""
    with torch.cuda.device(device):
        bits = _lib.device_errors(_stream_handle(device), clear=True)
    if bits & _lib.DEV_EV_RANGE:
        raise AssertionError("e_v outside the contract clamp")
    if bits:
        raise RuntimeError("LSSA-B8 device error bits 0x%x (timeout=2, bad page=4, misaligned row=8)" % bits)


_WS = {}


def workspace(device, nbytes):
    """A cached uint8 device buffer of at least nbytes (grown, never shrunk)."""
    key = (device.type, device.index)
    buf = _WS.get(key)
    if buf is None or buf.numel() < nbytes:
        buf = torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device=device)
        _WS[key] = buf
    return buf


def quant_rows(x, Tpad=None):
    """P1 on the device: x [B, H, T, dh] -> (q8 int8 [B, H, Tpad, dh], eq int32 [B, H, Tpad])."""
    dev = _require_cuda(x)
    B, H, T, dh = x.shape
    Tp = tpad(T) if Tpad is None else Tpad
    q8 = torch.empty((B, H, Tp, dh), dtype=torch.int8, device=dev)
    eq = torch.empty((B, H, Tp), dtype=torch.int32, device=dev)
    with torch.cuda.device(dev):
        _lib.check(_lib.load().lssab8_quant_rows(x.data_ptr(), dtype_code(x.dtype), B, H, T, dh, _lib.i64x(x.stride()),
                                                 Tp, q8.data_ptr(), eq.data_ptr(), _stream_handle(dev)),
                   "lssab8_quant_rows")
    return q8, eq


def quant_heads(x, Tpad=None):
    """P1 with one exponent per head (q_exp_mode "head"): x [B, H, T, dh] -> (q8 [B, H, Tpad, dh],
    eq [B, H, Tpad] holding the head's exponent on every row)."""
    dev = _require_cuda(x)
    B, H, T, dh = x.shape
    Tp = tpad(T) if Tpad is None else Tpad
    q8 = torch.empty((B, H, Tp, dh), dtype=torch.int8, device=dev)
    eq = torch.empty((B, H, Tp), dtype=torch.int32, device=dev)
    with torch.cuda.device(dev):
        _lib.check(_lib.load().lssab8_quant_heads(x.data_ptr(), dtype_code(x.dtype), B, H, T, dh, _lib.i64x(x.stride()),
                                                  Tp, q8.data_ptr(), eq.data_ptr(), _stream_handle(dev)),
                   "lssab8_quant_heads")
    return q8, eq


def key_mask_words(key_valid, B, T, device):
    """The general kernel's key mask: [B, Tpad / 32] int32 words, bit j % 32 of word j / 32 set when
    key j < T is visible.  key_valid: None (every key), [T] or [B, T] bool."""
    Tp = tpad(T)
    kv = torch.zeros((B, Tp), dtype=torch.bool, device=device)
    if key_valid is None:
        kv[:, :T] = True
    else:
        kv[:, :T] = torch.as_tensor(key_valid, dtype=torch.bool, device=device).reshape(-1, T).expand(B, T)
    w = torch.arange(32, device=device, dtype=torch.int64)
    words = (kv.view(B, Tp // 32, 32).to(torch.int64) << w).sum(-1)       # < 2^32
    return torch.where(words >= 2 ** 31, words - 2 ** 32, words).to(torch.int32).contiguous()   # same bits


def prefill_lattice_general(q8, eq, k8, ek, v8, ev, ev0, T, causal, kmask):
    """The general prefill on a prepared lattice (causal flag, key mask words from key_mask_words):
    returns float32 out [B, T, H, dh]."""
    dev = _require_cuda(q8, eq, k8, ek, v8, ev, kmask)
    B, H, Tp, dh = q8.shape
    KVH = k8.shape[1]
    out = torch.empty((B, T, H, dh), dtype=torch.float32, device=dev)
    with torch.cuda.device(dev):
        _lib.check(_lib.load().lssab8_prefill_lattice_general(
            q8.data_ptr(), eq.data_ptr(), k8.data_ptr(), ek.data_ptr(), v8.data_ptr(), ev.data_ptr(),
            None if ev0 is None else ev0.data_ptr(), B, H, KVH, T, dh, Tp, int(bool(causal)), kmask.data_ptr(),
            out.data_ptr(), _lib.i64x(out.stride()), _stream_handle(dev)), "lssab8_prefill_lattice_general")
    return out


def quant_blocks(x, mode=0):
    """P2/P3 on the device: x [B, KVH, T, dh] -> (x8 [B, KVH, Tpad, dh], e [B, KVH, nblk], e0 [B, KVH]).
    mode 0 = B8 grid, 1 = B9 value grid, 2 = B9.1 sink_alone value grid."""
    dev = _require_cuda(x)
    B, KVH, T, dh = x.shape
    Tp = tpad(T)
    x8 = torch.empty((B, KVH, Tp, dh), dtype=torch.int8, device=dev)
    e = torch.empty((B, KVH, Tp // KB), dtype=torch.int32, device=dev)
    e0 = torch.zeros((B, KVH), dtype=torch.int32, device=dev)
    with torch.cuda.device(dev):
        _lib.check(_lib.load().lssab8_quant_blocks(x.data_ptr(), dtype_code(x.dtype), B, KVH, T, dh,
                                                   _lib.i64x(x.stride()), Tp, int(mode), x8.data_ptr(), e.data_ptr(),
                                                   e0.data_ptr(), _stream_handle(dev)),
                   "lssab8_quant_blocks")
    return x8, e, e0


def quant_keys_offset(k, mu):
    """P2 with the key offset: k [B, KVH, T, dh], mu [KVH, dh] -> (k8 [B, KVH, Tpad, dh], ek [B, KVH, nblk])
    of k' = fl(f32(k) - mu[g, c]) (reference/lssab8_torch.py:143-144)."""
    dev = _require_cuda(k, mu)
    B, KVH, T, dh = k.shape
    mu = mu.to(device=dev, dtype=torch.float32).contiguous()
    if tuple(mu.shape) != (KVH, dh):
        raise ValueError("mu must be [KVH, dh] = [%d, %d], got %s" % (KVH, dh, tuple(mu.shape)))
    Tp = tpad(T)
    k8 = torch.empty((B, KVH, Tp, dh), dtype=torch.int8, device=dev)
    ek = torch.empty((B, KVH, Tp // KB), dtype=torch.int32, device=dev)
    with torch.cuda.device(dev):
        _lib.check(_lib.load().lssab8_quant_keys_offset(k.data_ptr(), dtype_code(k.dtype), B, KVH, T, dh,
                                                        _lib.i64x(k.stride()), Tp, mu.data_ptr(), k8.data_ptr(),
                                                        ek.data_ptr(), _stream_handle(dev)),
                   "lssab8_quant_keys_offset")
    return k8, ek


def prefill_lattice(q8, eq, k8, ek, v8, ev, ev0, T, out=None, out_dtype=torch.bfloat16):
    """Prefill on a prepared lattice; returns out [B, T, H, dh] (or writes `out`)."""
    dev = _require_cuda(q8, eq, k8, ek, v8, ev)
    B, H, Tp, dh = q8.shape
    KVH = k8.shape[1]
    if out is None:
        out = torch.empty((B, T, H, dh), dtype=out_dtype, device=dev)
    with torch.cuda.device(dev):
        _lib.check(_lib.load().lssab8_prefill_lattice(
            q8.data_ptr(), eq.data_ptr(), k8.data_ptr(), ek.data_ptr(), v8.data_ptr(), ev.data_ptr(),
            None if ev0 is None else ev0.data_ptr(), B, H, KVH, T, dh, Tp, None,
            out.data_ptr(), dtype_code(out.dtype), _lib.i64x(out.stride()), _stream_handle(dev)),
            "lssab8_prefill_lattice")
    return out


def prefill_chunk_lattice(q8, eq, k8, ek, v8, ev, ev0, T0, T, out=None, out_dtype=torch.bfloat16):
    """Block-aligned chunked prefill: query rows [T0, T) (T0 a multiple of 128) against keys [0, T).

    q8/eq: the chunk's rows from quant_rows (padded to a multiple of 128 rows); k8/ek/v8/ev/ev0:
    the key lattice of the whole prefix [0, T) from quant_blocks, whose complete blocks earlier
    chunks have already written.  Returns out [B, T - T0, H, dh] (or writes `out`), bit-identical
    to rows [T0, T) of the whole prefill of length T (the reference's 128-aligned chunk
    invariance, reference/lssab8_selftest.py:292-317).
    """
    dev = _require_cuda(q8, eq, k8, ek, v8, ev)
    B, H, Tq, dh = q8.shape
    KVH = k8.shape[1]
    if T0 % KB or not 0 <= T0 < T:
        raise ValueError("chunk start %d must be a multiple of %d below T = %d" % (T0, KB, T))
    if Tq != tpad(T - T0) or k8.shape[2] != tpad(T):
        raise ValueError("lattice shapes do not match the chunk [%d, %d)" % (T0, T))
    if out is None:
        out = torch.empty((B, T - T0, H, dh), dtype=out_dtype, device=dev)
    with torch.cuda.device(dev):
        _lib.check(_lib.load().lssab8_prefill_chunk_lattice(
            q8.data_ptr(), eq.data_ptr(), k8.data_ptr(), ek.data_ptr(), v8.data_ptr(), ev.data_ptr(),
            None if ev0 is None else ev0.data_ptr(), B, H, KVH, T0, T, dh,
            None, out.data_ptr(), dtype_code(out.dtype),
            _lib.i64x(out.stride()), _stream_handle(dev)),
            "lssab8_prefill_chunk_lattice")
    return out


def prefill_peers(query, key, value, out, peer_ptrs, sink=False, check=False):
    """The sharded prefill with the gather fused into the kernel (lssab8_prefill_peers): this
    rank's rows go into `out` (a view of this rank's output buffer, any strides) and, at the same
    element offsets, into every address of peer_ptrs (other ranks' buffers mapped into this
    process, already offset to the same place as `out`).  query [B, h, T, dh], key/value
    [B, kvh, T, dh]: this rank's heads.  The caller orders the ranks' barriers around it."""
    dev = _require_cuda(query, key, value, out)
    if not (query.dtype == key.dtype == value.dtype):
        raise TypeError("query, key and value must share one dtype")
    B, H, T, dh = query.shape
    KVH = key.shape[1]
    if tuple(out.shape) != (B, T, H, dh):
        raise ValueError("out must be [B, T, h, dh] for this rank's heads")
    if len(peer_ptrs) > 7:
        raise ValueError("at most 7 peers")
    L = _lib.load()
    nbytes = L.lssab8_prefill_workspace_size(B, H, KVH, T, dh)
    if nbytes == 0:
        raise ValueError("unsupported prefill shape")
    ws = workspace(dev, nbytes)
    arr = (ctypes.c_void_p * max(len(peer_ptrs), 1))(*[int(p) for p in peer_ptrs])
    with torch.cuda.device(dev):
        _lib.check(L.lssab8_prefill_peers(query.data_ptr(), key.data_ptr(), value.data_ptr(), dtype_code(query.dtype), B,
                                          H, KVH, T, dh, _lib.i64x(query.stride()), _lib.i64x(key.stride()),
                                          _lib.i64x(value.stride()), int(bool(sink)), out.data_ptr(),
                                          dtype_code(out.dtype), _lib.i64x(out.stride()), arr, len(peer_ptrs),
                                          ws.data_ptr(), ws.numel(), _stream_handle(dev)), "lssab8_prefill_peers")
    if check:
        check_device_errors(dev)
    return out


def quant_values_keyshift(x, dmax, sink=False):
    """B9.3 value PREP: x [B, KVH, T, dh] -> (v8 [B, KVH, Tpad, dh], ev [B, KVH, nblk], ev0 [B, KVH],
    d8 [B, KVH, Tpad] int8), v_keyshift = dmax (reference/lssab9_torch.py:145-153)."""
    dev = _require_cuda(x)
    B, KVH, T, dh = x.shape
    Tp = tpad(T)
    v8 = torch.empty((B, KVH, Tp, dh), dtype=torch.int8, device=dev)
    ev = torch.empty((B, KVH, Tp // KB), dtype=torch.int32, device=dev)
    ev0 = torch.zeros((B, KVH), dtype=torch.int32, device=dev)
    d8 = torch.empty((B, KVH, Tp), dtype=torch.int8, device=dev)
    with torch.cuda.device(dev):
        _lib.check(_lib.load().lssab8_quant_values_keyshift(
            x.data_ptr(), dtype_code(x.dtype), B, KVH, T, dh, _lib.i64x(x.stride()), Tp, int(bool(sink)), int(dmax),
            v8.data_ptr(), ev.data_ptr(), ev0.data_ptr(), d8.data_ptr(), _stream_handle(dev)),
            "lssab8_quant_values_keyshift")
    return v8, ev, ev0, d8


def prefill_lattice_keyshift(q8, eq, k8, ek, v8, ev, ev0, d8, T, out=None, out_dtype=torch.bfloat16):
    """B9.3 prefill on a prepared lattice (values and shifts from quant_values_keyshift)."""
    dev = _require_cuda(q8, eq, k8, ek, v8, ev, d8)
    B, H, Tp, dh = q8.shape
    KVH = k8.shape[1]
    if out is None:
        out = torch.empty((B, T, H, dh), dtype=out_dtype, device=dev)
    with torch.cuda.device(dev):
        _lib.check(_lib.load().lssab8_prefill_lattice_keyshift(
            q8.data_ptr(), eq.data_ptr(), k8.data_ptr(), ek.data_ptr(), v8.data_ptr(), ev.data_ptr(),
            None if ev0 is None else ev0.data_ptr(), d8.data_ptr(), B, H, KVH, T, dh, Tp, out.data_ptr(),
            dtype_code(out.dtype), _lib.i64x(out.stride()), _stream_handle(dev)), "lssab8_prefill_lattice_keyshift")
    return out


def prefill(query, key, value, sink=False, out=None, out_dtype=None, check=True, mu=None, qexp="row",
            v_keyshift=0, b9grid=False):
    """Batched LSSA-B8 (sink=False) / B9.1 sink_alone (sink=True) causal GQA prefill.

    query [B, H, T, dh], key/value [B, KVH, T, dh] (any strides, one dtype) -> out [B, T, H, dh]
    in out_dtype (default query.dtype).  Each batch element is the reference drop-in's function
    (reference/lssab8_torch.py:134-271, reference/lssab9_torch.py:109-326).  mu [KVH, dh]: the
    key offset subtracted before the key quantiser (reference/lssab8_torch.py:143-144).  qexp
    "head": one query exponent per head.  v_keyshift = dmax: B9.3 (the B9 value grid, key j on
    e_v + d_j, PV weight eh >> d_j).  b9grid: the B9 value grid (exponent clamp 48, assert 40) with
    the sink off."""
    dev = _require_cuda(query, key, value)
    if not (query.dtype == key.dtype == value.dtype):
        raise TypeError("query, key and value must share one dtype")
    B, H, T, dh = query.shape
    if key.dim() != 4 or key.shape[0] != B or key.shape[2] != T or key.shape[3] != dh or value.shape != key.shape:
        raise ValueError("key/value must be [B, KVH, T, dh] matching query [B, H, T, dh]")
    KVH = key.shape[1]
    if H % KVH:
        raise ValueError("query heads must be a multiple of kv heads")
    if out is None:
        out = torch.empty((B, T, H, dh), dtype=out_dtype or query.dtype, device=dev)
    if mu is not None or qexp != "row" or v_keyshift or b9grid:    # the lattice route
        if qexp not in ("row", "head"):
            raise ValueError(qexp)
        q8, eq = quant_rows(query) if qexp == "row" else quant_heads(query)
        k8, ek = quant_keys_offset(key, mu) if mu is not None else quant_blocks(key, 0)[:2]
        if v_keyshift:
            v8, ev, ev0, d8 = quant_values_keyshift(value, v_keyshift, sink)
            if out.dtype in (torch.float32, torch.bfloat16):
                prefill_lattice_keyshift(q8, eq, k8, ek, v8, ev, ev0 if (sink and T > 1) else None, d8, T, out=out)
            else:
                out.copy_(prefill_lattice_keyshift(q8, eq, k8, ek, v8, ev, ev0 if (sink and T > 1) else None, d8, T,
                                                   out_dtype=torch.float32))
        else:
            v8, ev, ev0 = quant_blocks(value, 2 if sink else (1 if b9grid else 0))
            prefill_lattice(q8, eq, k8, ek, v8, ev, ev0 if sink else None, T, out=out)
        if check:
            check_device_errors(dev)
        return out
    L = _lib.load()
    nbytes = L.lssab8_prefill_workspace_size(B, H, KVH, T, dh)
    if nbytes == 0:
        raise ValueError("unsupported prefill shape")
    ws = workspace(dev, nbytes)
    with torch.cuda.device(dev):
        _lib.check(L.lssab8_prefill(query.data_ptr(), key.data_ptr(), value.data_ptr(), dtype_code(query.dtype), B, H,
                                    KVH, T, dh, _lib.i64x(query.stride()), _lib.i64x(key.stride()),
                                    _lib.i64x(value.stride()), int(bool(sink)), out.data_ptr(), dtype_code(out.dtype),
                                    _lib.i64x(out.stride()), ws.data_ptr(), ws.numel(), _stream_handle(dev)),
                   "lssab8_prefill")
    if check:
        check_device_errors(dev)
    return out
