"""The N > 1 path on CPU: world_size-2 gloo ranks run the sharding and the output gather with
the oracle standing in for the kernel (test infrastructure), and the gathered result must be
bit-identical to the single-process result -- the multi-GPU contract that results do not
depend on the GPU count."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from lockstep_b200 import sharding as SH


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _oracle_compute(q, k, v, sink):
    import oracle as O
    outs = []
    for b in range(q.shape[0]):
        o = O.attention(q[b].numpy(), k[b].numpy(), v[b].numpy(), sink=sink, nthreads=2)
        outs.append(torch.from_numpy(np.ascontiguousarray(o.transpose(1, 0, 2))))
    return torch.stack(outs)


def _worker(rank, world, port, q, k, v, lens, dq, dk, dv, ret):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        out = SH.prefill_sharded(q, k, v, sink=True, compute=_oracle_compute)
        import oracle as O

        def dec_local(idx):
            rows = [torch.from_numpy(O.decode_rows(dq[b].numpy(), dk[b][:, :int(lens[b])].numpy(),
                                                   dv[b][:, :int(lens[b])].numpy(), nthreads=2)) for b in idx]
            return torch.stack(rows)
        dec = SH.decode_sharded(dq, lens, dec_local)
        if rank == 0:
            ret["prefill"] = out.numpy().copy()
            ret["decode"] = dec.numpy().copy()
    finally:
        dist.destroy_process_group()


def test_partition_sequences_is_balanced_and_complete():
    lens = [28027, 21244, 17250, 9588, 10796, 2324, 5000, 30000]
    for world in (1, 2, 4, 8):
        parts = SH.partition_sequences(lens, world)
        assert sorted(sum(parts, [])) == list(range(len(lens)))
        loads = [sum(lens[b] for b in p) for p in parts]
        assert max(loads) - min(loads) <= max(lens)


def test_kv_group_range():
    assert SH.kv_group_range(8, 4, 3) == (6, 8)
    with pytest.raises(ValueError):
        SH.kv_group_range(8, 3, 0)


def test_two_gloo_ranks_equal_single_process():
    rng = np.random.default_rng(0)
    B, H, KVH, T, dh = 2, 4, 2, 200, 64
    q = torch.from_numpy(rng.standard_normal((B, H, T, dh)).astype(np.float32))
    k = torch.from_numpy(rng.standard_normal((B, KVH, T, dh)).astype(np.float32))
    v = torch.from_numpy(rng.standard_normal((B, KVH, T, dh)).astype(np.float32))
    lens = [300, 130, 260]
    dq = torch.from_numpy(rng.standard_normal((3, H, dh)).astype(np.float32))
    dk = torch.from_numpy(rng.standard_normal((3, KVH, 300, dh)).astype(np.float32))
    dv = torch.from_numpy(rng.standard_normal((3, KVH, 300, dh)).astype(np.float32))
    ret = mp.Manager().dict()
    mp.start_processes(_worker, args=(2, _free_port(), q, k, v, lens, dq, dk, dv, ret), nprocs=2,
                       join=True, start_method="spawn")
    single = _oracle_compute(q, k, v, True).numpy()
    assert np.array_equal(ret["prefill"].view(np.uint32), single.view(np.uint32))
    import oracle as O
    for b in range(3):
        ref = O.decode_rows(dq[b].numpy(), dk[b][:, :lens[b]].numpy(), dv[b][:, :lens[b]].numpy())
        assert np.array_equal(ret["decode"][b].view(np.uint32), ref.view(np.uint32))
