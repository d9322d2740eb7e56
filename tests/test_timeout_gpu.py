"""The bounded waits' failure path, on the GPU, with no fault.

lssab8_selftest_timeout runs the prefill kernel with one key block withheld by its TMA producer
(the pipeline barrier expects the bytes, nothing delivers them) and a wait limit of about a
millisecond.  Every role of every CTA must give up within the limit, record the timeout bit in
the device error word, free its tensor memory and exit; the host reads the status, and the next
ordinary call on the same context must run and be bit-exact.  The cycle runs twice, so a CTA
that kept its tensor memory would show up as the following launch never getting any.
"""
import time

import numpy as np
import pytest
import torch

import oracle as O
from lockstep_b200 import _lib
from lockstep_b200 import attention as A
from lockstep_b200 import workloads as W

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("withhold", [0, 2])
def test_withheld_block_times_out_and_context_survives(withhold):
    B, H, KVH, T, dh = 1, 4, 2, 512, 128
    q, k, v = W.prefill_inputs(B, H, KVH, T, dh, seed=21)
    to = lambda x: torch.from_numpy(np.ascontiguousarray(x)).to(torch.bfloat16).cuda()
    q8, eq = A.quant_rows(to(q))
    k8, ek, _ = A.quant_blocks(to(k), 0)
    v8, ev, _ = A.quant_blocks(to(v), 0)
    ref = O.attention(q[0], k[0], v[0]).transpose(1, 0, 2)
    L = _lib.load()
    assert _lib.device_errors() == 0
    for cycle in range(2):
        junk = torch.zeros((B, T, H, dh), dtype=torch.float32, device="cuda")
        t0 = time.time()
        _lib.check(L.lssab8_selftest_timeout(q8.data_ptr(), eq.data_ptr(), k8.data_ptr(), ek.data_ptr(),
                                             v8.data_ptr(), ev.data_ptr(), B, H, KVH, T, dh, withhold, 1000,
                                             junk.data_ptr(), _lib.i64x(junk.stride()),
                                             torch.cuda.current_stream().cuda_stream), "lssab8_selftest_timeout")
        bits = _lib.device_errors(clear=True)                 # synchronises the stream
        took = time.time() - t0
        assert bits & _lib.DEV_TIMEOUT, (cycle, bits)
        assert took < 1.0, took                               # gave up after ~1 ms, not the 2 s default
        out = A.prefill_lattice(q8, eq, k8, ek, v8, ev, None, T, out_dtype=torch.float32)
        torch.cuda.synchronize()
        assert _lib.device_errors() == 0
        assert np.array_equal(out[0].cpu().numpy().view(np.uint32), np.ascontiguousarray(ref).view(np.uint32)), cycle


def test_selftest_timeout_rejects_bad_arguments():
    """A negative block or a wait limit outside (0, 2 s] is refused before any launch.  The
    buffers are real and sized for the shape all the same, so nothing could read outside them."""
    B, H, KVH, T, dh = 1, 4, 2, 512, 128
    q8 = torch.zeros((B, H, T, dh), dtype=torch.int8, device="cuda")
    eq = torch.zeros((B, H, T), dtype=torch.int32, device="cuda")
    k8 = torch.zeros((B, KVH, T, dh), dtype=torch.int8, device="cuda")
    e = torch.zeros((B, KVH, T // 128), dtype=torch.int32, device="cuda")
    out = torch.zeros((B, T, H, dh), dtype=torch.float32, device="cuda")
    L = _lib.load()
    for withhold, wait_us in ((-1, 1000), (0, 0), (0, 2000001)):
        rc = L.lssab8_selftest_timeout(q8.data_ptr(), eq.data_ptr(), k8.data_ptr(), e.data_ptr(), k8.data_ptr(),
                                       e.data_ptr(), B, H, KVH, T, dh, withhold, wait_us, out.data_ptr(),
                                       _lib.i64x(out.stride()), None)
        assert rc == 1, (withhold, wait_us)
    torch.cuda.synchronize()
    assert _lib.device_errors() == 0
