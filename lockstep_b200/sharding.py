"""Multi-GPU partitioning of the LSSA-B8 path (one process per GPU, torch.distributed).

The path shards without any reduction: every output row is an independent recurrence.
  * prefill: rank r of n owns kv heads [r*KVH/n, (r+1)*KVH/n) and their query heads; it runs the
    prefill on its heads and the outputs are all-gathered (prefill_shard_gather);
  * decode: sequences are partitioned longest-first (greedy on KV length) so that ranks carry
    balanced KV bytes; each rank decodes its sequences and the rows are gathered.
The only collective is the output gather (NCCL over NVLink on GPUs; gloo works for CPU tests).
Results are bit-identical at every rank count because no arithmetic crosses a rank.

On GPUs the gather is fused into the prefill kernel: every rank's output buffer is mapped into
every other rank (PeerOutputs: CUDA IPC, P2P over NVLink), and the kernel's epilogue stores each
finished output tile into its own buffer and, at the same place, into every peer's, so the gather
overlaps the compute tile by tile and costs no SM time of its own.  Two barriers on the stream
(a one-element NCCL all-reduce) bracket the kernel: before it, so no rank writes into a buffer
its owner still reads; after it, so every rank's buffer is complete when the call returns.

Without peer buffers (CPU ranks, or GPUs that cannot reach each other), prefill_shard_gather
falls back to NCCL: the batch is cut into chunks, and while the kernel runs chunk c + 1 on the
caller's stream, a second stream all-gathers chunk c's head shards and scatters them into the
[B, T, H, dh] output.  Either way, inputs may sit in pinned host memory (copied chunk by chunk
on a third stream under the previous chunk's compute), and a pinned host tensor can receive
this rank's rows of every finished chunk on a fourth stream, so an end-to-end host -> device ->
host call overlaps them all.
"""
import ctypes

import torch
import torch.distributed as dist


def kv_group_range(KVH, world, rank):
    if KVH % world:
        raise ValueError("kv heads (%d) must divide evenly over %d ranks" % (KVH, world))
    n = KVH // world
    return rank * n, (rank + 1) * n


def partition_sequences(lengths, world):
    """Longest-first greedy: returns per-rank lists of sequence indices (each sorted), so that
    the per-rank sums of KV lengths are balanced.  Deterministic (ties by index)."""
    order = sorted(range(len(lengths)), key=lambda b: (-int(lengths[b]), b))
    load = [0] * world
    parts = [[] for _ in range(world)]
    for b in order:
        r = min(range(world), key=lambda x: (load[x], x))
        parts[r].append(b)
        load[r] += int(lengths[b])
    return [sorted(p) for p in parts]


def _world(group=None):
    if dist.is_available() and dist.is_initialized():
        return dist.get_world_size(group), dist.get_rank(group)
    return 1, 0


class PeerOutputs:
    """An output buffer on every rank of the group, mapped into every other rank (CUDA IPC).

    local: this rank's tensor (shape, dtype, on `device`); peers: {rank: (address, offset)} of the
    other ranks' buffers in this process.  Every process must see every GPU under the same
    ordinals (as torchrun leaves them).  close() (collective) unmaps them."""

    def __init__(self, shape, dtype, device, group=None):
        from . import _lib
        self.world, self.rank = _world(group)
        self.group = group
        self.local = torch.empty(shape, dtype=dtype, device=device)
        self.flag = torch.zeros(1, dtype=torch.float32, device=device)
        self.peers = {}
        L = _lib.load()
        h = ctypes.create_string_buffer(64)
        off = ctypes.c_uint64(0)
        _lib.check(L.lssab8_peer_export(self.local.data_ptr(), h, ctypes.byref(off)), "lssab8_peer_export")
        infos = [None] * self.world
        dist.all_gather_object(infos, (bytes(h.raw), int(off.value), self.local.get_device()), group=group)
        err = None
        with torch.cuda.device(self.local.device):
            for r, (hb, o, d) in enumerate(infos):
                if r == self.rank:
                    continue
                ptr = ctypes.c_void_p()
                rc = L.lssab8_peer_import(hb, o, d, ctypes.byref(ptr))
                if rc:
                    err = _lib.Lssab8Error(rc, "lssab8_peer_import of rank %d" % r)
                    break
                self.peers[r] = (int(ptr.value), int(o))
        # every rank takes the same branch: if any rank cannot map a peer, none uses the buffers
        ok = torch.tensor([0.0 if err else 1.0], device=self.local.device)
        dist.all_reduce(ok, op=dist.ReduceOp.MIN, group=group)
        if ok.item() < 1.0:
            for ptr, o in self.peers.values():
                L.lssab8_peer_close(ptr, o)
            self.peers = {}
            raise err or RuntimeError("another rank could not map its peer buffers")

    def barrier(self):
        """A barrier of the ranks ordered on the current stream (a one-element NCCL all-reduce)."""
        dist.all_reduce(self.flag, group=self.group)

    def addresses(self, view):
        """The peers' addresses of the element `view` starts at in the local buffer."""
        off = view.data_ptr() - self.local.data_ptr()
        return [self.peers[r][0] + off for r in sorted(self.peers)]

    def close(self):
        from . import _lib
        torch.cuda.synchronize(self.local.device)
        dist.barrier(group=self.group)                 # nobody writes into a buffer being unmapped
        L = _lib.load()
        for ptr, off in self.peers.values():
            _lib.check(L.lssab8_peer_close(ptr, off), "lssab8_peer_close")
        self.peers = {}
        dist.barrier(group=self.group)                 # every mapping is gone before owners free


def _kernel_compute(q, k, v, sink, out):
    from . import attention as A
    return A.prefill(q, k, v, sink=sink, out=out, check=False)


def prefill_shard_gather(q, k, v, H, sink=False, out=None, chunk=1, group=None, compute=None,
                         host_out=None, host_rows=None, peers=None, peer_copy=False):
    """Sharded causal GQA prefill, gathered: every rank returns the whole out [B, T, H, dh].

    q [B, h, T, dh], k / v [B, kvh, T, dh]: this rank's shard, query heads [r*h, (r+1)*h) and kv
    heads [r*kvh, (r+1)*kvh) of H = n*h and n*kvh (kv_group_range); on this rank's GPU, or in
    pinned host memory, in which case each chunk is copied in on its own stream.  chunk: batch
    elements per pipeline step.  compute(q, k, v, sink, out) -> out [b, T, h, dh] defaults to the
    B200 kernel (attention.prefill).  host_out [B, T1 - T0, H, dh] (pinned) receives rows
    host_rows = (T0, T1) of every gathered batch element.  The result's dtype is q's.
    peers: a PeerOutputs of shape [B, T, H, dh] (the result is peers.local; `out` must be None):
    every rank's rows reach every rank's buffer over NVLink, stored by the prefill kernel's epilogue
    (peer_copy=False; `compute` must be None), or copied by the copy engines after each chunk's
    compute (peer_copy=True: one 2D copy of the chunk's head slice per peer, no SM time, under the
    next chunk's compute)."""
    world, rank = _world(group)
    B, h, T, dh = q.shape
    if H != h * world:
        raise ValueError("H = %d query heads cannot be %d ranks x %d" % (H, world, h))
    if peers is not None:
        if out is not None or (compute is not None and not peer_copy):
            raise ValueError("with peers the result is peers.local and the kernel computes it")
        if tuple(peers.local.shape) != (B, T, H, dh) or peers.world != world:
            raise ValueError("the peer buffers do not match this call")
        out = peers.local
    compute = compute or _kernel_compute
    dev = torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() and (
        q.is_cuda or q.is_pinned()) else q.device
    on_gpu = dev.type == "cuda"
    if out is None:
        out = torch.empty((B, T, H, dh), dtype=q.dtype, device=dev)
    chunks = [(b0, min(b0 + chunk, B)) for b0 in range(0, B, chunk)]
    T0, T1 = host_rows if host_rows is not None else (0, T)

    if not on_gpu:                                   # CPU ranks (gloo): the same steps, in order
        for b0, b1 in chunks:
            loc = compute(q[b0:b1], k[b0:b1], v[b0:b1], sink, None).contiguous()
            _gather_into(out[b0:b1], loc, world, group)
            if host_out is not None:
                host_out[b0:b1].copy_(out[b0:b1, T0:T1])
        return out

    cur = torch.cuda.current_stream(dev)
    fused = peers is not None and world > 1 and not peer_copy
    copying = peers is not None and world > 1 and peer_copy
    s_in = torch.cuda.Stream(dev) if not q.is_cuda else None
    s_comm = torch.cuda.Stream(dev) if world > 1 and not fused else None
    # copy mode: one stream per peer, so the copies to different peers run on different copy engines
    s_peer = [torch.cuda.Stream(dev) for _ in range(world - 1)] if copying else []
    s_out = torch.cuda.Stream(dev) if host_out is not None else None
    start = torch.cuda.Event()
    start.record(cur)
    for s in [s_in, s_comm, s_out] + s_peer:
        if s is not None:
            s.wait_event(start)
    keep = []                                         # buffers used on the side streams
    loaded = None
    if s_in is not None:
        loaded = {}

        def load(c):
            b0, b1 = chunks[c]
            with torch.cuda.stream(s_in):
                t = tuple(x[b0:b1].to(dev, non_blocking=True) for x in (q, k, v))
                ev = torch.cuda.Event()
                ev.record(s_in)
            loaded[c] = (t, ev)
        load(0)
    if fused or copying:
        peers.barrier()                               # every owner is done reading its buffer
    for c, (b0, b1) in enumerate(chunks):
        if loaded is not None:
            if c + 1 < len(chunks):
                load(c + 1)                           # next chunk's copy under this chunk's compute
            (qc, kc, vc), ev = loaded.pop(c)
            cur.wait_event(ev)
            for t in (qc, kc, vc):                    # made on the copy stream, read on this one
                t.record_stream(cur)
        else:
            qc, kc, vc = q[b0:b1], k[b0:b1], v[b0:b1]
        if world == 1:
            compute(qc, kc, vc, sink, out[b0:b1])
            done = out[b0:b1]
        elif copying:
            from . import _lib
            mine = out[b0:b1, :, rank * h:(rank + 1) * h]
            compute(qc, kc, vc, sink, mine)
            ev = torch.cuda.Event()
            ev.record(cur)
            es = out.element_size()
            L = _lib.load()
            for sp, a in zip(s_peer, peers.addresses(mine)):   # the chunk's head slab: (b1 - b0) T rows of h dh
                sp.wait_event(ev)
                _lib.check(L.lssab8_peer_copy2d(a, H * dh * es, mine.data_ptr(), H * dh * es, h * dh * es,
                                                (b1 - b0) * T, sp.cuda_stream), "lssab8_peer_copy2d")
            if s_out is not None:
                for sp in s_peer:
                    s_comm.wait_stream(sp)
                with torch.cuda.stream(s_comm):
                    peers.barrier()                   # this chunk is complete on every rank
            done = out[b0:b1]
        elif fused:
            from . import attention as A
            mine = out[b0:b1, :, rank * h:(rank + 1) * h]
            A.prefill_peers(qc, kc, vc, mine, peers.addresses(mine), sink=sink)
            if s_out is not None or c + 1 == len(chunks):
                peers.barrier()                       # this chunk is complete on every rank
            done = out[b0:b1]
        else:
            loc = torch.empty((b1 - b0, T, h, dh), dtype=out.dtype, device=dev)
            compute(qc, kc, vc, sink, loc)
            ev = torch.cuda.Event()
            ev.record(cur)
            s_comm.wait_event(ev)
            with torch.cuda.stream(s_comm):
                _gather_into(out[b0:b1], loc, world, group)
            keep.append(loc)
            done = out[b0:b1]
        if s_out is not None:
            ev = torch.cuda.Event()
            ev.record(s_comm if s_comm is not None else cur)
            s_out.wait_event(ev)
            with torch.cuda.stream(s_out):
                host_out[b0:b1].copy_(done[:, T0:T1], non_blocking=True)
    for s in [s_comm, s_out] + s_peer:               # the caller's stream sees the whole result
        if s is not None:
            cur.wait_stream(s)
    if copying:
        peers.barrier()                               # every rank's copies into every buffer have landed
    del keep
    return out


def _gather_into(dst, loc, world, group):
    """All-gather the head shards loc [b, T, h, dh] of every rank into dst [b, T, world*h, dh]."""
    if world == 1:
        dst.copy_(loc)
        return
    b, T, h, dh = loc.shape
    g = torch.empty((world * b, T, h, dh), dtype=loc.dtype, device=loc.device)
    dist.all_gather_into_tensor(g, loc, group=group)
    dst.view(b, T, world, h, dh).copy_(g.view(world, b, T, h, dh).permute(1, 2, 0, 3, 4))


def prefill_sharded(query, key, value, sink=False, compute=None, group=None, chunk=1):
    """Prefill of query [B, H, T, dh], key/value [B, KVH, T, dh] held whole by every rank (or at
    least its heads), sharded by kv-head group; returns the full out [B, T, H, dh] on every rank.
    `compute(q, k, v, sink)` -> [B, T, h, dh] defaults to the B200 kernel."""
    world, rank = _world(group)
    B, H, T, dh = query.shape
    KVH = key.shape[1]
    grp = H // KVH
    g0, g1 = kv_group_range(KVH, world, rank)
    fn = None if compute is None else (lambda q, k, v, s, out: compute(q, k, v, s))
    return prefill_shard_gather(query[:, g0 * grp:g1 * grp], key[:, g0:g1], value[:, g0:g1], H, sink=sink,
                                group=group, compute=fn, chunk=chunk)


class DecodePartition:
    """The sequence partition of a decode batch over the ranks, with the index tensors its row
    gather needs (built once per batch layout, reused every step).

    parts[r]: the sequences rank r decodes (sorted); mine = parts[rank]; the gathered buffer holds
    nmax rows per rank, and row r * nmax + i of it is sequence parts[r][i]."""

    def __init__(self, lengths, world, rank, device=None):
        self.world, self.rank = world, rank
        self.parts = partition_sequences(lengths, world)
        self.mine = self.parts[rank]
        self.nmax = max(len(p) for p in self.parts)
        src = [r * self.nmax + i for r, p in enumerate(self.parts) for i in range(len(p))]
        dst = [b for p in self.parts for b in p]
        self.src = torch.tensor(src, dtype=torch.long, device=device)
        self.dst = torch.tensor(dst, dtype=torch.long, device=device)
        self.mine_idx = torch.tensor(self.mine, dtype=torch.long, device=device)


def decode_sharded(q, lengths, decode_local, group=None, plan=None):
    """Decode rows for all sequences, each rank computing its partition.

    q [B, H, dh]; lengths: host sequence of KV lengths; decode_local(indices) -> [len(indices),
    H, dh] computes the rows of those sequences on this rank.  plan: a DecodePartition of these
    lengths (made here when None).  Returns [B, H, dh] everywhere."""
    world, rank = _world(group)
    if plan is None:
        plan = DecodePartition(lengths, world, rank, q.device)
    out_local = decode_local(plan.mine) if plan.mine else q.new_empty((0,) + tuple(q.shape[1:]))
    if world == 1:
        return out_local
    # pad to the largest partition so the gather has equal sizes
    pad = q.new_zeros((plan.nmax,) + tuple(q.shape[1:]))
    pad[:len(plan.mine)] = out_local
    gathered = torch.empty((world * plan.nmax,) + tuple(pad.shape[1:]), dtype=pad.dtype, device=pad.device)
    dist.all_gather_into_tensor(gathered, pad, group=group)
    out = q.new_empty(q.shape)
    out[plan.dst] = gathered[plan.src]
    return out
