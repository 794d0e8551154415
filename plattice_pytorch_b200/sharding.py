"""Image-level data parallelism: one process per GPU, each filtering its own
contiguous share of a batch of independent images (one lattice per image, no
exchange between images, so no collective on the data path).  The only
collectives are the barrier and the max over ranks of the measured times."""
import torch

__all__ = ["shard_range", "max_over_ranks", "barrier"]


def shard_range(n_items, world, rank):
    """Contiguous share [start, stop) of n_items for `rank` of `world`; the
    first n_items % world ranks get one item more."""
    if world < 1 or not 0 <= rank < world or n_items < 0:
        raise ValueError(f"bad shard request n_items={n_items} world={world} rank={rank}")
    base, extra = divmod(n_items, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def max_over_ranks(x, world, device="cpu"):
    """Maximum of a float over all ranks of the default process group."""
    if world <= 1:
        return float(x)
    import torch.distributed as dist
    t = torch.tensor([float(x)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
