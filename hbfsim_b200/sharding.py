"""Channel sharding across ranks (one process per GPU).

Channels are address-interleaved and independent under the timing models,
so rank r of N owns the global channels g with g mod N == r (its local
channel c is global channel c*N + r) and times them with no data exchange.
The one coupling is thermal: once per epoch every rank needs the activity of
every die, gathered here with torch.distributed and put in global die order
g*D + d for hbfsim_advance_epoch_global_v1.
"""
from __future__ import annotations

import numpy as np


def remap_to_shard(address, rank: int, world: int, range_base: int, range_length: int,
                   channels: int, stripe: int):
    """Moves a trace laid out for `channels` channels onto the channels
    g mod world == rank of a geometry with channels*world channels, keeping
    each access's (local channel, die, plane, page) digits and its offset in
    the stripe.  Stripe units move independently, so an access that crosses
    a stripe boundary may land across a page boundary (then it is
    unsupported); traces of stripe-contained accesses (config 1's 1 KiB
    reads) keep every status.  Works on numpy arrays and torch tensors of
    int64/uint64."""
    if world == 1:
        return address
    inside = (address >= range_base) & (address < range_base + range_length)
    off = address - range_base
    u = off // stripe
    w = off % stripe
    g0 = u % channels
    rest = u // channels
    u2 = rest * (channels * world) + g0 * world + rank
    moved = range_base + u2 * stripe + w
    if isinstance(address, np.ndarray):
        return np.where(inside, moved, address)
    import torch
    return torch.where(inside, moved, address)


def global_die_order(per_rank, world: int, dies: int, channels_total: int):
    """[rank][c*D + d] activity -> global [g*D + d] (g = c*world + rank)."""
    per_rank = [np.asarray(a) for a in per_rank]
    out = np.zeros(channels_total * dies, per_rank[0].dtype)
    for r, a in enumerate(per_rank):
        local = a.reshape(-1, dies)
        for c in range(local.shape[0]):
            g = c * world + r
            if g < channels_total:
                out[g * dies:(g + 1) * dies] = local[c]
    return out


def global_die_index(world: int, local_channels: int, dies: int, channels_total: int):
    """Index map for the same reorder on the device: position in the
    rank-major gathered buffer of each global die (g*D + d order)."""
    idx = np.zeros(channels_total * dies, np.int64)
    for g in range(channels_total):
        r, c = g % world, g // world
        for d in range(dies):
            idx[g * dies + d] = (r * local_channels + c) * dies + d
    return idx


_INDEX_CACHE: dict = {}


def _device_index(world: int, local_channels: int, dies: int, channels_total: int, device):
    """global_die_index as a device tensor, built once per shape."""
    import torch
    key = (world, local_channels, dies, channels_total, str(device))
    idx = _INDEX_CACHE.get(key)
    if idx is None:
        idx = torch.from_numpy(global_die_index(world, local_channels, dies,
                                                channels_total)).to(device)
        _INDEX_CACHE[key] = idx
    return idx


def gather_die_activity(ctx, local_channels: int, dies: int, channels_total: int,
                        group=None):
    """Device tensors (read bytes, writes) of every global die, from each
    rank's activity since the last epoch: one all-gather (NCCL on GPU ranks)
    of the rank's [read bytes | writes] packed in one buffer, then one
    gather into global die order with an index kept on the device.
    Everything runs on torch's current stream, after the batches submitted
    on it."""
    import torch
    import torch.distributed as dist
    world = dist.get_world_size(group)
    n = local_channels * dies
    packed = torch.empty(2 * n, dtype=torch.int64, device="cuda")
    ctx.copy_die_activity(packed[:n], packed[n:], torch.cuda.current_stream())
    flat = torch.empty(world * 2 * n, dtype=torch.int64, device="cuda")
    dist.all_gather_into_tensor(flat, packed, group=group)
    idx = _device_index(world, local_channels, dies, channels_total, flat.device)
    by_rank = flat.view(world, 2, n)
    rb = by_rank[:, 0, :].reshape(-1).index_select(0, idx)
    wr = by_rank[:, 1, :].reshape(-1).index_select(0, idx)
    return rb, wr


def advance_epoch_sharded(ctx, epoch_s: float, local_channels: int, dies: int,
                          channels_total: int, group=None):
    """One thermal epoch of a sharded context: gather every die's activity
    and run the replicated grid step; each rank derives its own factors."""
    import torch
    rb, wr = gather_die_activity(ctx, local_channels, dies, channels_total, group)
    ctx.advance_epoch_global(epoch_s, rb, wr, torch.cuda.current_stream())
