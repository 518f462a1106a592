"""Multi-GPU composition of the path: one process per GPU over torch.distributed.

The per-GPU work is this library's CUDA kernels (the C ABI).  This module partitions
the work and, where the path has an exchange step, runs it:

* reductions: a non-reduced axis is sharded into slabs; every rank reduces the slab it
  holds (any strides: a compact local slab, or a view of a full tensor cut by
  `shard_view` without a copy) into its own outputs.  No collective.
* movement / permutation: the destination is sharded along the axis that is slowest in
  both it and the source view (`movement_shard_axis`); every rank writes its part,
  stored compactly, from the matching strided view of the source (`movement_slab`).
  No collective.
* gather: index batches are sharded and the table is replicated; every rank gathers
  its own output rows.  No collective.
* scatter_add: update batches are sharded.  Every rank adds its updates into a
  full-size partial destination (rank 0's holds the operand, the others start at
  zero), and one reduce-scatter (sum) leaves each rank the destination rows it owns.
  The floating sums over colliding rows are order-dependent, as in the single-GPU
  operation (atomics).
* RRQR: rows are sharded; every step exchanges the column norms and the reflector
  dots (`RrqrRowsSharded`: NCCL inside the library's C++ driver, t4a_dist_rrqr).
"""
import ctypes

import torch
import torch.distributed as dist

import t4a_b200 as _t4
from t4a_b200 import abi as _abi


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


def shard_view(x, shard_axis, world, rank):
    """The slab of `x` along NumPy axis `shard_axis` that rank `rank` of `world` owns, as a
    view (no copy)."""
    start, stop = shard_range(x.shape[shard_axis], world, rank)
    return x.narrow(shard_axis, start, stop - start)


def gather_rows_sharded(table, indices, group=None, out=None):
    """This rank's share of a gather of whole rows: `indices` holds all index rows;
    the rank gathers rows shard_range(len(indices)) of the output.  No collective."""
    world, rank = _world(group)
    start, stop = shard_range(indices.numel(), world, rank)
    return _t4.gather_rows(table, indices.reshape(-1)[start:stop], out=out)


def reduce_sharded(x_local, numpy_axis, op, out=None, workspace=None, stream=None):
    """This rank's part of a single-axis reduction whose input is sharded along another
    axis: reduces the slab `x_local` (any strides, e.g. a `shard_view`) along
    `numpy_axis` into this rank's outputs.  No collective, no copy of the slab."""
    return _t4.reduce(x_local, numpy_axis, op, out=out, workspace=workspace, stream=stream)


def movement_shard_axis(src_layout):
    """The destination axis (a t4a layout axis: 0 fastest) to shard a movement along: the
    one whose stride is largest in both the compact destination and the source view
    (the largest min(|source stride|, destination stride)), so that every rank reads and
    writes runs as long as the permutation allows; ties go to the slower destination
    axis."""
    strides = src_layout.strides_list()
    ext = src_layout.extents_list()
    best, best_key = src_layout.rank - 1, None
    dst_stride = 1
    for ax in range(src_layout.rank):
        key = (min(abs(strides[ax]), dst_stride), ax)
        if ext[ax] > 1 and (best_key is None or key > best_key):
            best, best_key = ax, key
        dst_stride *= ext[ax]
    return best


def movement_slab(src_layout, world, rank, axis=None):
    """Rank `rank`'s part of a movement whose destination is sharded along one of its
    axes (default movement_shard_axis).  `src_layout` is the source view that the whole
    destination is materialized from (strides may be negative).  Returns (source layout
    of the part, compact destination layout of the part, axis, start): the source part is
    the same view with that axis restricted to [start, stop); the destination part is
    stored compactly by the rank."""
    r = src_layout.rank
    axis = movement_shard_axis(src_layout) if axis is None else axis
    ext = src_layout.extents_list()
    strides = src_layout.strides_list()
    start, stop = shard_range(ext[axis], world, rank)
    part_ext = list(ext)
    part_ext[axis] = stop - start
    src = _abi.layout(part_ext, strides, src_layout.offset + start * strides[axis])
    return src, _abi.layout(part_ext), axis, start


def materialize_slab(stream_handle, dtype, dst_ptr, src_ptr, src_layout, src_len, world, rank, axis=None):
    """Writes rank `rank`'s destination part (movement_slab) from the source at
    `src_ptr` through the strided-copy entry.  Returns the destination part's layout."""
    src, dst, _, _ = movement_slab(src_layout, world, rank, axis)
    n = dst.count()
    _t4.copy_strided_raw(stream_handle, dtype, dst_ptr, dst, n, src_ptr, src, src_len)
    return dst


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


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr())


# ---- RRQR over row blocks ---------------------------------------------------------

class NcclComm:
    """This library's NCCL communicator over the ranks of a torch.distributed group: rank
    0's unique id reaches the others through the group (a one-off broadcast), then every
    rank joins.  Without an initialized process group it is a world of one."""

    def __init__(self, group=None):
        lib = _t4.lib()
        if dist.is_available() and dist.is_initialized():
            world, rank = _world(group)
        else:
            world, rank = 1, 0
        ident = torch.zeros(128, dtype=torch.uint8)
        if rank == 0:
            _t4.check(lib.t4a_dist_unique_id(_ptr(ident)), "dist_unique_id")
        if world > 1:
            carrier = ident.cuda() if dist.get_backend(group) == "nccl" else ident
            dist.broadcast(carrier, src=dist.get_global_rank(group, 0) if group is not None else 0, group=group)
            ident = carrier.cpu()
        handle = ctypes.c_void_p()
        _t4.check(lib.t4a_dist_comm_init(ctypes.byref(handle), _ptr(ident), world, rank), "dist_comm_init")
        self.handle, self.world, self.rank = handle, world, rank

    def close(self):
        if self.handle is not None and self.handle.value:
            _t4.check(_t4.lib().t4a_dist_comm_destroy(self.handle), "dist_comm_destroy")
        self.handle = None


class P2pComm:
    """This library's NVLink exchange for one rank (t4a_p2p_create / t4a_p2p_open): a
    region of this GPU's memory that every rank of the group maps through CUDA IPC, for
    a matrix of n columns.  The 64-byte IPC handles travel through the torch.distributed
    group once.  Without an initialized process group it is a world of one.  close()
    waits for every rank (a barrier), so no rank frees its region while another may
    still write into it."""

    def __init__(self, n, group=None):
        lib = _t4.lib()
        if dist.is_available() and dist.is_initialized():
            world, rank = _world(group)
        else:
            world, rank = 1, 0
        own = (ctypes.c_ubyte * 64)()
        handle = ctypes.c_void_p()
        _t4.check(lib.t4a_p2p_create(n, world, rank, ctypes.byref(handle), own), "p2p_create")
        handles = bytes(own)
        if world > 1:
            gathered = [None] * world
            dist.all_gather_object(gathered, bytes(own), group=group)
            handles = b"".join(gathered)
        _t4.check(lib.t4a_p2p_open(handle, ctypes.create_string_buffer(handles, len(handles))), "p2p_open")
        self.handle, self.world, self.rank, self.n, self.group = handle, world, rank, n, group

    def close(self):
        if self.handle is not None and self.handle.value:
            torch.cuda.synchronize()
            if self.world > 1:
                dist.barrier(group=self.group)
            _t4.check(_t4.lib().t4a_p2p_destroy(self.handle), "p2p_destroy")
        self.handle = None


class RrqrRowsSharded:
    """RRQR of a [m, n] F32/F64 matrix whose rows are split across the ranks of a group:
    this rank holds rows [row0, row0 + local_rows) as the column-major block `work`
    (a flat CUDA tensor of local_rows * n elements, or a 2-D tensor whose transpose is
    contiguous).  run() does `steps` steps of the reference loop.  exchange="p2p"
    (t4a_dist_rrqr_p2p): two launches per step, whose column pass stores each column's
    parts into every rank's memory over NVLink and waits on per-column flags;
    exchange="nccl" (t4a_dist_rrqr): three launches and two NCCL all-gathers per step.  Both give the same bits; perm, coeff, pivots and status come
    out identical on every rank, and a world of one gives t4a_rrqr's bits."""

    def __init__(self, work, m, n, row0, steps, comm=None, group=None, exchange="p2p"):
        if exchange not in ("p2p", "nccl"):
            raise ValueError(f"exchange {exchange!r}")
        flat = work.reshape(-1) if work.dim() == 1 else work.t().reshape(-1)
        self.work = flat
        self.m, self.n, self.row0, self.steps = m, n, row0, steps
        self.exchange = exchange
        self.rows = flat.numel() // n if n else 0
        self.dtype = _t4.torch_dtype_tag(flat)
        if comm is None:
            comm = P2pComm(n, group) if exchange == "p2p" else NcclComm(group)
            self.own_comm = True
        else:
            self.own_comm = False
        self.comm = comm
        self.layout = _abi.layout([self.rows, n], [1, max(self.rows, 1)])
        trailing_steps = sum(1 for s in range(steps) if n - s - 1 > 0)
        if exchange == "nccl":
            nbytes = ctypes.c_size_t(0)
            _t4.check(_t4.lib().t4a_dist_rrqr_workspace_bytes(self.dtype, n, self.comm.world, ctypes.byref(nbytes)),
                      "dist_rrqr_workspace_bytes")
            self.workspace = torch.empty(max(nbytes.value, 16), dtype=torch.uint8, device=flat.device)
            self.launches = 2 + steps + 2 * trailing_steps  # NCCL calls besides: 1 + 2 per step with trailing columns
        else:
            self.workspace = None
            self.launches = 3 + steps + trailing_steps if steps else 1  # init, first, swap + column per step, leave

    def run(self, stream_handle, perm, coeff, pivots, status):
        if self.exchange == "p2p":
            _t4.check(_t4.lib().t4a_dist_rrqr_p2p(self.comm.handle, stream_handle, self.dtype, _ptr(self.work),
                                                  ctypes.byref(self.layout), self.work.numel(), self.row0, self.m,
                                                  self.steps, _ptr(perm), _ptr(coeff), _ptr(pivots), _ptr(status)),
                      "dist_rrqr_p2p")
            return
        _t4.check(_t4.lib().t4a_dist_rrqr(self.comm.handle, stream_handle, self.dtype, _ptr(self.work),
                                          ctypes.byref(self.layout), self.work.numel(), self.row0, self.m, self.steps,
                                          _ptr(perm), _ptr(coeff), _ptr(pivots), _ptr(status),
                                          _ptr(self.workspace), self.workspace.numel()), "dist_rrqr")

    def close(self):
        if self.own_comm:
            self.comm.close()


def gather_rows_colmajor(local, m, n, row0, group=None):
    """The whole [m, n] column-major matrix (flat, m * n elements) on every rank, from each
    rank's row block (flat column-major, rows shard_range(m) of this rank)."""
    world, rank = _world(group)
    sizes = [shard_range(m, world, r) for r in range(world)]
    most = max(b - a for a, b in sizes)
    rows = local.numel() // n
    block = torch.zeros((n, most), dtype=local.dtype, device=local.device)
    block[:, :rows] = local.view(n, rows)
    parts = [torch.empty_like(block) for _ in range(world)]
    dist.all_gather(parts, block, group=group)
    full = torch.empty((n, m), dtype=local.dtype, device=local.device)
    for (a, b), part in zip(sizes, parts):
        full[:, a:b] = part[:, :b - a]
    return full.reshape(-1)
