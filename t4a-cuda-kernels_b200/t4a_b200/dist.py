"""Multi-GPU composition of the path: one process per GPU over torch.distributed.

The per-GPU work is this library's CUDA kernels (the C ABI); this module only
partitions it and, for scatter_add, runs the one exchange that operation has:

* gather: index batches are sharded across ranks and the table is replicated, so every
  rank gathers its own output rows; no collective.
* reductions: a non-reduced axis is sharded into slabs, so every rank reduces its own
  slab to its own outputs; no collective.
* scatter_add: update batches are sharded.  Every rank adds its updates into a
  full-size partial destination (rank 0's holds the operand, the others start at zero),
  and one reduce-scatter (sum) leaves each rank the destination rows it owns.  The
  floating sums over colliding rows are order-dependent, as in the single-GPU
  operation (atomics).
* RRQR is not sharded: the reference's norm and dot chains fold each lane's rows in
  order, so splitting rows across GPUs would change the rounding; ranks run
  independent factorizations.
"""
import torch
import torch.distributed as dist

import t4a_b200 as _t4


def shard_range(n, world, rank):
    """Rows [start, stop) of rank `rank` when n rows are split into `world` contiguous,
    balanced shards (the first n % world shards hold one row more)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of world {world}")
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def _world(group):
    return dist.get_world_size(group), dist.get_rank(group)


def gather_rows_sharded(table, indices, group=None, out=None):
    """This rank's share of a gather of whole rows: `indices` holds all index rows;
    the rank gathers rows shard_range(len(indices)) of the output.  No collective."""
    world, rank = _world(group)
    start, stop = shard_range(indices.numel(), world, rank)
    return _t4.gather_rows(table, indices.reshape(-1)[start:stop], out=out)


def reduce_sharded(x, numpy_axis, op, shard_axis=0, group=None):
    """This rank's slab of a single-axis reduction: `x` is sharded along `shard_axis`
    (which must differ from the reduced axis); returns the reduction of this rank's
    slab.  No collective."""
    if shard_axis == numpy_axis:
        raise ValueError("the sharded axis must not be the reduced axis")
    world, rank = _world(group)
    start, stop = shard_range(x.shape[shard_axis], world, rank)
    return _t4.reduce(x.narrow(shard_axis, start, stop - start).contiguous(), numpy_axis, op)


def _reduce_scatter_rows(out, partial, group):
    """out = rows [rank*k, (rank+1)*k) of the sum of every rank's `partial`."""
    if dist.get_backend(group) == "gloo":
        # gloo has no reduce-scatter: all-reduce, then keep this rank's rows.
        world, rank = _world(group)
        summed = partial.clone()
        dist.all_reduce(summed, op=dist.ReduceOp.SUM, group=group)
        k = out.shape[0]
        out.copy_(summed[rank * k:(rank + 1) * k])
        return out
    dist.reduce_scatter_tensor(out, partial, op=dist.ReduceOp.SUM, group=group)
    return out


def scatter_partial(operand, group=None):
    """The full-size partial destination of this rank: the operand on rank 0, zeros
    elsewhere."""
    _, rank = _world(group)
    return operand.clone() if rank == 0 else torch.zeros_like(operand)


def scatter_add_rows_sharded(partial, indices, updates, group=None, workspace=None, out=None, local_add=None):
    """Sharded scatter_add of whole rows.  `indices` / `updates` are this rank's update
    batch; `partial` is this rank's full-size partial destination (scatter_partial()).
    Adds the batch into `partial`, then reduce-scatters the partials: returns the rows
    [rank*k, (rank+1)*k) of the global destination, k = rows / world (rows must divide
    evenly).  `local_add(partial, indices, updates, workspace)` is the per-rank step; the
    default is this library's CUDA scatter_add."""
    world, rank = _world(group)
    rows, cols = partial.shape
    if rows % world:
        raise ValueError(f"{rows} destination rows do not split evenly over {world} ranks")
    if local_add is None:
        _t4.scatter_add_rows(partial, indices, updates, workspace=workspace)
    else:
        local_add(partial, indices, updates, workspace)
    if out is None:
        out = torch.empty((rows // world, cols), dtype=partial.dtype, device=partial.device)
    return _reduce_scatter_rows(out, partial, group)
