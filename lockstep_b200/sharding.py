"""Multi-GPU partitioning of the LSSA-B8 path (one process per GPU, torch.distributed).

The path shards without any reduction: every output row is an independent recurrence.
  * prefill: rank r of n owns kv heads [r*KVH/n, (r+1)*KVH/n) and their query heads; it runs
    the prefill on strided views of its heads (no copies) and the outputs are gathered;
  * decode: sequences are partitioned longest-first (greedy on KV length) so that ranks carry
    balanced KV bytes; each rank decodes its sequences and the rows are gathered.
The only collective is the output gather (NCCL over NVLink on GPUs; gloo works for CPU tests).
Results are bit-identical at every rank count because no arithmetic crosses a rank.
"""
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


def _world():
    if dist.is_available() and dist.is_initialized():
        return dist.get_world_size(), dist.get_rank()
    return 1, 0


def prefill_sharded(query, key, value, sink=False, compute=None, group=None):
    """Prefill of query [B, H, T, dh], key/value [B, KVH, T, dh] (every rank holds the full
    inputs or at least its heads) sharded by kv-head group; returns the full out [B, T, H, dh]
    on every rank.  `compute(q, k, v, sink)` -> [B, T, h, dh] defaults to the B200 kernel."""
    if compute is None:
        from . import attention as A
        compute = lambda q, k, v, s: A.prefill(q, k, v, sink=s)
    world, rank = _world()
    B, H, T, dh = query.shape
    KVH = key.shape[1]
    grp = H // KVH
    g0, g1 = kv_group_range(KVH, world, rank)
    local = compute(query[:, g0 * grp:g1 * grp], key[:, g0:g1], value[:, g0:g1], sink)   # [B, T, h, dh]
    if world == 1:
        return local
    parts = [torch.empty_like(local) for _ in range(world)]
    dist.all_gather(parts, local.contiguous(), group=group)
    return torch.cat(parts, dim=2)


def decode_sharded(q, lengths, decode_local, group=None):
    """Decode rows for all sequences, each rank computing its partition.

    q [B, H, dh]; lengths: host sequence of KV lengths; decode_local(indices) -> [len(indices),
    H, dh] computes the rows of those sequences on this rank.  Returns [B, H, dh] everywhere."""
    world, rank = _world()
    parts = partition_sequences(lengths, world)
    mine = parts[rank]
    out_local = decode_local(mine) if mine else q.new_empty((0,) + tuple(q.shape[1:]))
    if world == 1:
        return out_local
    # pad to the largest partition so the gather has equal sizes
    nmax = max(len(p) for p in parts)
    pad = q.new_zeros((nmax,) + tuple(q.shape[1:]))
    pad[:len(mine)] = out_local
    gathered = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(gathered, pad, group=group)
    out = q.new_empty(q.shape)
    for r, p in enumerate(parts):
        if p:
            out[torch.tensor(p, device=q.device)] = gathered[r][:len(p)]
    return out
