"""The sharded path on two GPUs, on the real kernels: kv-head-group prefill with the pipelined
NCCL output all-gather, with the gather fused into the kernel (epilogue P2P stores into the
other rank's buffer, CUDA IPC) and with it on the copy engines (a 2D copy of each chunk's head slab
into the other rank's buffer), each from device inputs and from pinned host inputs with this
rank's rows read back; and sequence-partitioned paged decode.  Every rank's gathered output must equal the
pinned oracle bit for bit, which is also the single-GPU result: no arithmetic crosses a rank.

Needs two GPUs in this process's view (skipped otherwise: NCCL does not run two ranks on one GPU).
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

B, H, KVH, T, DH = 3, 8, 4, 700, 128


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _inputs():
    from lockstep_b200 import workloads as W
    return W.prefill_inputs(B, H, KVH, T, DH, outliers=0.01, seed=8)


def _worker(rank, world, port, ret):
    import datetime
    import hashlib

    import torch.distributed as dist

    from lockstep_b200 import decode as D
    from lockstep_b200 import sharding as SH
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        q, k, v = _inputs()
        h, kvh = H // world, KVH // world
        sl = lambda x, n: torch.from_numpy(np.ascontiguousarray(x[:, rank * n:(rank + 1) * n])).to(torch.bfloat16)
        qd, kd, vd = sl(q, h).to(dev), sl(k, kvh).to(dev), sl(v, kvh).to(dev)
        out1 = SH.prefill_shard_gather(qd, kd, vd, H, chunk=1)
        qh, kh, vh = sl(q, h).pin_memory(), sl(k, kvh).pin_memory(), sl(v, kvh).pin_memory()
        rows = (rank * T // world, (rank + 1) * T // world)
        host = torch.empty((B, rows[1] - rows[0], H, DH), dtype=torch.bfloat16).pin_memory()
        out2 = SH.prefill_shard_gather(qh, kh, vh, H, chunk=2, host_out=host, host_rows=rows)
        torch.cuda.synchronize()
        # the gather fused into the kernel: P2P stores into the other rank's mapped buffer
        peers = SH.PeerOutputs((B, T, H, DH), torch.bfloat16, dev)
        peers.local.fill_(float("nan"))
        SH.prefill_shard_gather(qd, kd, vd, H, peers=peers, chunk=B)
        out3 = peers.local.clone()
        host3 = torch.empty_like(host).pin_memory()
        peers.local.fill_(float("nan"))
        SH.prefill_shard_gather(qh, kh, vh, H, peers=peers, chunk=1, host_out=host3, host_rows=rows)
        torch.cuda.synchronize()
        out4 = peers.local.clone()
        # the gather on the copy engines: each chunk's head slab copied into the other buffer
        peers.local.fill_(float("nan"))
        SH.prefill_shard_gather(qd, kd, vd, H, peers=peers, chunk=1, peer_copy=True)
        out5 = peers.local.clone()
        host5 = torch.empty_like(host).pin_memory()
        peers.local.fill_(float("nan"))
        SH.prefill_shard_gather(qh, kh, vh, H, peers=peers, chunk=2, host_out=host5, host_rows=rows, peer_copy=True)
        torch.cuda.synchronize()
        out6 = peers.local.clone()
        peers.close()
        # decode: sequences partitioned over the ranks, each rank quantises only its own
        lens = [700, 1, 130, 511, 256]
        rng = np.random.default_rng(4)
        dq = torch.from_numpy(rng.standard_normal((5, H, DH)).astype(np.float32)).to(torch.bfloat16).to(dev)
        dk = torch.from_numpy(rng.standard_normal((5, KVH, 700, DH)).astype(np.float32)).to(torch.bfloat16)
        dv = torch.from_numpy(rng.standard_normal((5, KVH, 700, DH)).astype(np.float32)).to(torch.bfloat16)

        def local(idx):
            L = max(lens[b] for b in idx)
            kk = dk[idx][:, :, :L].to(dev).contiguous()
            vv = dv[idx][:, :, :L].to(dev).contiguous()
            bt, npages = D.identity_pages(len(idx), L, dev)
            kv = D.build_paged_kv(kk, vv, torch.tensor([lens[b] for b in idx], dtype=torch.int32, device=dev), bt,
                                  npages, sink=True)
            return D.decode(dq[idx], kv)
        dec = SH.decode_sharded(dq, lens, local)
        torch.cuda.synchronize()
        dig = lambda t: hashlib.sha256(t.cpu().view(torch.int16).numpy().tobytes()).hexdigest()
        ret[rank] = dict(out1=dig(out1), out2=dig(out2), out3=dig(out3), out4=dig(out4), out5=dig(out5),
                         out6=dig(out6), host=host.view(torch.int16).numpy().copy(),
                         host3=host3.view(torch.int16).numpy().copy(), host5=host5.view(torch.int16).numpy().copy(),
                         rows=rows, dec=dec.cpu().view(torch.int16).numpy().copy())
        if rank == 0:
            ret["full"] = out1.cpu().view(torch.int16).numpy().copy()
            ret["dq"], ret["dk"], ret["dv"], ret["lens"] = (dq.float().cpu().numpy(), dk.float().numpy(),
                                                           dv.float().numpy(), lens)
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_nccl_ranks_equal_oracle():
    import oracle as O
    ret = mp.Manager().dict()
    mp.start_processes(_worker, args=(2, _free_port(), ret), nprocs=2, join=True, start_method="spawn")
    q, k, v = _inputs()
    ref = np.stack([O.f32_to_bf16_bits(O.attention(q[b], k[b], v[b]).transpose(1, 0, 2)) for b in range(B)])
    full = ret["full"].view(np.uint16)
    assert np.array_equal(full, ref)
    for r in range(2):
        for key in ("out1", "out2", "out3", "out4", "out5", "out6"):
            assert ret[r][key] == ret[0]["out1"], (r, key)
        t0, t1 = ret[r]["rows"]
        for key in ("host", "host3", "host5"):
            assert np.array_equal(ret[r][key].view(np.uint16), ref[:, t0:t1]), (r, key)
        assert np.array_equal(ret[r]["dec"], ret[0]["dec"]), r
    dq, dk, dv, lens = ret["dq"], ret["dk"], ret["dv"], ret["lens"]
    dec = ret[0]["dec"].view(np.uint16)
    for b, L in enumerate(lens):
        want = O.f32_to_bf16_bits(O.decode_rows(dq[b], dk[b][:, :L], dv[b][:, :L], sink=True))
        assert np.array_equal(dec[b], want), b
