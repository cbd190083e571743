"""Ensemble-member sharding across the GPUs of one node (one process per GPU).

Mosaic forecasts an ensemble by batching members along the attention batch
dimension (`batch = b * members`, mosaic.py:301,308); members never interact
inside the network. So the members are partitioned across ranks, every rank runs
the block-sparse attention (and the rest of the step) for its own members only,
and the single collective is an all-gather of the per-member output fields
(NCCL over NVLink on GPUs, gloo on CPU ranks in the tests).

Parity detail (NoiseGenerator, primitives.py:287-302): the reference draws
randn(batch, noise_dim) for ALL members from one generator seeded 42; a rank must
draw that full-batch tensor and keep its rows (`shard_rows`), otherwise member i
would see different noise than in a one-GPU run.
"""
import torch
import torch.distributed as dist

__all__ = ["member_range", "shard_rows", "gather_members", "full_batch_noise", "run_sharded"]


def member_range(num_members, rank, world):
    """[start, stop) of the members owned by `rank`: contiguous, sizes differ by at most 1."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} / world {world}")
    base, rem = divmod(num_members, world)
    start = rank * base + min(rank, rem)
    return start, start + base + (1 if rank < rem else 0)


def shard_rows(full, rank, world, dim=0):
    """The rows of a full-ensemble tensor that belong to `rank` (along `dim`)."""
    start, stop = member_range(full.shape[dim], rank, world)
    return full.narrow(dim, start, stop - start)


def full_batch_noise(num_members, noise_dim, device, seed=42):
    """randn(num_members, noise_dim) from a generator seeded like NoiseGenerator
    (primitives.py:294-302); every rank draws all rows, then shards."""
    g = torch.Generator(device=device).manual_seed(seed)
    return torch.randn(num_members, noise_dim, generator=g, device=device)


def gather_members(local, num_members, group=None, dim=0):
    """All-gather the per-rank member shards (along `dim`) into the full ensemble on
    every rank. Shards may differ by one member; they are padded to the largest
    shard for the collective and trimmed afterwards."""
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    if world == 1:
        return local
    sizes = [member_range(num_members, r, world) for r in range(world)]
    longest = max(b - a for a, b in sizes)
    mine = sizes[rank][1] - sizes[rank][0]
    if local.shape[dim] != mine:
        raise ValueError(f"rank {rank} holds {local.shape[dim]} members, expected {mine}")
    x = local.movedim(dim, 0).contiguous()
    if mine < longest:
        pad = torch.zeros((longest - mine, *x.shape[1:]), dtype=x.dtype, device=x.device)
        x = torch.cat([x, pad], dim=0)
    out = torch.empty((world * longest, *x.shape[1:]), dtype=x.dtype, device=x.device)
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(out, x, group=group)
    else:
        dist.all_gather(list(out.chunk(world)), x, group=group)
    parts = [out[r * longest: r * longest + (b - a)] for r, (a, b) in enumerate(sizes)]
    return torch.cat(parts, dim=0).movedim(0, dim)


def run_sharded(fn, full_inputs, num_members, group=None, batch_dims=None):
    """Run `fn(*member_shards)` on this rank's members and all-gather its output.

    `full_inputs` are full-ensemble tensors (member axis given by `batch_dims`,
    default 0 for each); `fn` must return one tensor whose dim 0 is the member axis.
    """
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    rank = dist.get_rank(group) if dist.is_initialized() else 0
    dims = batch_dims or [0] * len(full_inputs)
    shards = [shard_rows(t, rank, world, d) for t, d in zip(full_inputs, dims)]
    out = fn(*shards)
    return gather_members(out, num_members, group) if world > 1 else out
