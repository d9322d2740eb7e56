"""Failure detection of the multi-GPU host logic, on CPU ranks (gloo), with the failures made on
the host: a rank that leaves before a collective must end the other rank's next collective with an
error within the process group's timeout (never a hang), and a rank whose peer mapping fails (a
fake of lssab8_peer_import returning an error) must make every rank refuse the fused gather
together -- no rank may go on to use buffers another rank could not map."""
import contextlib
import ctypes
import datetime
import os
import socket
import time

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


def _dropout_worker(rank, world, port, ret):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=3))
    lens = torch.tensor([100, 300, 50, 700])
    if rank == 1:
        return                                        # leaves between steps: never joins the gather
    t0 = time.time()
    try:
        SH.decode_sharded(torch.zeros(4, 2, 8), lens, lambda idx: torch.zeros(len(idx), 2, 8))
        ret["outcome"] = "completed"
    except Exception as e:                              # noqa: BLE001 -- any error ends the wait
        ret["outcome"] = "error: %s" % type(e).__name__
    ret["secs"] = time.time() - t0


def test_rank_that_leaves_ends_the_other_ranks_collective_with_an_error():
    ret = mp.Manager().dict()
    mp.spawn(_dropout_worker, args=(2, _free_port(), ret), nprocs=2, join=True)
    assert ret["outcome"].startswith("error"), ret["outcome"]
    assert ret["secs"] < 60


class _FakeLib:
    """lssab8_peer_export / import / close on host memory; import fails on `fail_rank`."""

    def __init__(self, rank, fail_rank):
        self.rank, self.fail_rank, self.closed = rank, fail_rank, 0

    def lssab8_peer_export(self, ptr, handle, off):
        ctypes.memmove(handle, b"h" * 64, 64)
        off._obj.value = 0
        return 0

    def lssab8_peer_import(self, handle, off, device, ptr):
        if self.rank == self.fail_rank:
            return 3                                  # an error status of the C ABI
        ptr._obj.value = 4096
        return 0

    def lssab8_peer_close(self, ptr, off):
        self.closed += 1
        return 0

    def lssab8_strerror(self, code):
        return b"fake error"


def _peer_worker(rank, world, port, fail_rank, ret):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
    from lockstep_b200 import _lib
    fake = _FakeLib(rank, fail_rank)
    _lib.load = lambda: fake
    torch.cuda.device = lambda d: contextlib.nullcontext()
    try:
        SH.PeerOutputs((4, 8), torch.float32, torch.device("cpu"))
        ret[rank] = "mapped"
    except Exception as e:                              # noqa: BLE001
        ret[rank] = "refused: %s" % type(e).__name__
    ret["closed%d" % rank] = fake.closed
    dist.destroy_process_group()


def test_failed_peer_mapping_on_one_rank_makes_every_rank_refuse():
    ret = mp.Manager().dict()
    mp.spawn(_peer_worker, args=(2, _free_port(), 1, ret), nprocs=2, join=True)
    assert ret[0].startswith("refused") and ret[1].startswith("refused"), dict(ret)
    assert ret["closed0"] == 1                         # rank 0 unmapped the peer it had mapped
    ret = mp.Manager().dict()
    mp.spawn(_peer_worker, args=(2, _free_port(), -1, ret), nprocs=2, join=True)
    assert ret[0] == "mapped" and ret[1] == "mapped", dict(ret)
