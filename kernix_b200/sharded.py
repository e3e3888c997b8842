"""Row-sharded GEMM across the GPUs of one node, with the gathered output.

One process per GPU (torch.distributed, NCCL over NVLink/NVSwitch).  The M rows
of A are split block-cyclically into pieces of ``piece`` rows: global row block
``i * world + rank`` belongs to ``rank``.  Each rank multiplies its pieces with
its own replica of B (no data-path collective for the compute), and piece ``i``
of every rank is all-gathered straight into rows
``[i * world * piece, (i + 1) * world * piece)`` of the full C -- the gathered
layout is already C's row order.  The all-gather of piece ``i`` runs on a
communication stream while piece ``i + 1`` is being multiplied.

Three ways to gather on GPUs:

* ``PeerOutput`` + ``sharded_matmul_push`` (or symmetric memory +
  ``sharded_matmul_push_mc``, the bench's default where the node has NVLink
  multicast, NVLS): C lives in memory that every rank maps into every other
  rank (CUDA IPC over NVLink).  The library's ``kx_matmul_rows_sharded_f32``
  computes the rank's pieces and pushes each into the same rows of every
  peer's C: with the copy engines, one stream per peer, while the next piece
  multiplies, and the last piece with one NVLink multicast store (or an
  all-SM kernel); one 4-byte NCCL all-reduce at the end of the step tells
  every rank that all pushes into its C have landed.
* ``ReplicatedOutput`` + ``sharded_matmul_replicated``: C lives in symmetric
  memory bound to an NVLink multicast object; the GEMM's epilogue stores
  every output element once through the multicast address and the NVSwitch
  delivers it to every rank's C, and one small all-reduce closes the step.
* ``sharded_matmul`` with ``all_gather_into_tensor`` per piece (NCCL; also the
  gloo path the CPU tests use).

``gemm_sharded`` is the single-process form (``kx_gemm_sharded_f32``): one
handle per GPU in one process, a contiguous window of rows per handle, the
windows copied between the outputs by the copy engines.

This is the multi-worker counterpart of ``CpuExecutor::matmul_into``'s row
chunking (crates/kernix-ops/src/execution.rs:188-233), lifted from threads in
one process to GPUs in one node.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable


@dataclass(frozen=True)
class RowPlan:
    """Block-cyclic row plan: ``pieces`` pieces of ``piece`` rows per rank."""

    m: int
    world: int
    piece: int

    @property
    def pieces(self) -> int:
        return self.m // (self.world * self.piece)

    def rows_of(self, rank: int, i: int) -> tuple[int, int]:
        """Global [start, stop) rows of piece ``i`` on ``rank``."""
        start = (i * self.world + rank) * self.piece
        return start, start + self.piece

    def gathered_rows(self, i: int) -> tuple[int, int]:
        """Rows of C that the all-gather of piece ``i`` fills."""
        return i * self.world * self.piece, (i + 1) * self.world * self.piece

    def local_rows(self, rank: int) -> list[int]:
        """Global row indices owned by ``rank``, piece by piece."""
        rows = []
        for i in range(self.pieces):
            s, e = self.rows_of(rank, i)
            rows.extend(range(s, e))
        return rows


def plan_rows(m: int, world: int, target_piece: int = 512) -> RowPlan:
    """Largest piece <= target_piece that tiles M evenly across ranks
    (``kx_row_piece``)."""
    import ctypes as C

    from . import _abi
    if m % world:
        raise ValueError(f"M={m} is not divisible by world={world}")
    piece, pieces = C.c_uint64(), C.c_uint64()
    _abi.raise_for(_abi.lib.kx_row_piece(m, world, target_piece, C.byref(piece), C.byref(pieces)), None)
    return RowPlan(m, world, int(piece.value))


def shard_window(total: int, rank: int, world: int) -> tuple[int, int]:
    """The contiguous window (start, count) of ``total`` independent units that
    ``rank`` of ``world`` takes (``kx_shard_window``)."""
    import ctypes as C

    from . import _abi
    start, count = C.c_uint64(), C.c_uint64()
    _abi.raise_for(_abi.lib.kx_shard_window(total, rank, world, C.byref(start), C.byref(count)), None)
    return int(start.value), int(count.value)


def rows_sharded(a_local, b, out, plan: RowPlan, rank: int, peer_ptrs=None, out_mc: int = 0) -> None:
    """``kx_matmul_rows_sharded_f32``: this rank's pieces of ``out`` = A B,
    each pushed into the peers' outputs (``peer_ptrs``: every rank's output
    storage as mapped here; ``out_mc``: its multicast address, used for the
    last piece) -- enqueued on the current stream."""
    import ctypes as C

    from . import _abi, _bind, _descriptor
    h = _bind(out)
    da, db, do = _descriptor(a_local), _descriptor(b), _descriptor(out)
    peers = (C.c_void_p * plan.world)(*peer_ptrs) if peer_ptrs is not None else None
    err = _abi.KxError()
    rc = _abi.lib.kx_matmul_rows_sharded_f32(h.ptr, C.byref(da), C.byref(db), C.byref(do), rank, plan.world,
                                             plan.piece, peers, C.c_void_p(int(out_mc) or None), C.byref(err))
    _abi.raise_for(rc, err)


def gemm_sharded(handles, a_windows, b_replicas, outs, gather_out: bool = True) -> None:
    """``kx_gemm_sharded_f32``: the row-sharded product from one process over
    several handles (one per GPU).  ``a_windows[r]`` holds the rows
    ``shard_window(M, r, len(handles))`` of A on handle r's device,
    ``b_replicas[r]`` B there, ``outs[r]`` a C-contiguous [M, N] output there;
    with ``gather_out`` every output ends with the whole product once each
    handle's stream has completed (``Handle.synchronize``)."""
    import ctypes as C

    from . import _abi, _descriptor
    n = len(handles)
    if not (len(a_windows) == len(b_replicas) == len(outs) == n):
        raise ValueError("one A window, B replica and output per handle")
    hs = (C.c_void_p * n)(*[h.ptr for h in handles])
    da = (_abi.KxTensor * n)(*[_descriptor(t) for t in a_windows])
    db = (_abi.KxTensor * n)(*[_descriptor(t) for t in b_replicas])
    do = (_abi.KxTensor * n)(*[_descriptor(t) for t in outs])
    err = _abi.KxError()
    rc = _abi.lib.kx_gemm_sharded_f32(hs, n, da, db, do, int(bool(gather_out)), C.byref(err))
    _abi.raise_for(rc, err)


def sharded_matmul(a_pieces, b, c, plan: RowPlan, rank: int, group=None,
                   matmul_into: Callable | None = None, streams=None, scratch=None) -> None:
    """Compute this rank's pieces and all-gather them into ``c`` (M x N).

    ``a_pieces[i]`` is this rank's piece ``i`` of A (any strided view the
    matmul accepts); ``c`` receives the full product on every rank.  With
    ``world == 1`` the pieces are written straight into ``c``.
    ``matmul_into(a, b, out)`` defaults to the device kernel; CPU tests inject
    a host implementation with a gloo group.
    """
    import torch
    import torch.distributed as dist

    if matmul_into is None:
        from . import matmul_into as _mi
        matmul_into = _mi
    world = plan.world
    if world == 1:
        for i in range(plan.pieces):
            s, e = plan.rows_of(0, i)
            matmul_into(a_pieces[i], b, c[s:e])
        return
    cuda = c.is_cuda
    if scratch is None:
        scratch = [torch.empty((plan.piece, c.shape[1]), dtype=c.dtype, device=c.device) for _ in range(plan.pieces)]
    if cuda:
        compute, comm = streams if streams is not None else (torch.cuda.current_stream(), torch.cuda.Stream())
        comm.wait_stream(compute)
        works = []
        for i in range(plan.pieces):
            with torch.cuda.stream(compute):
                matmul_into(a_pieces[i], b, scratch[i])
                ev = torch.cuda.Event()
                ev.record(compute)
            comm.wait_event(ev)
            g0, g1 = plan.gathered_rows(i)
            with torch.cuda.stream(comm):
                works.append(dist.all_gather_into_tensor(c[g0:g1], scratch[i], group=group, async_op=True))
        for w in works:
            w.wait()
        compute.wait_stream(comm)
    else:
        for i in range(plan.pieces):
            matmul_into(a_pieces[i], b, scratch[i])
            g0, g1 = plan.gathered_rows(i)
            dist.all_gather_into_tensor(c[g0:g1], scratch[i], group=group)


class _CudaArray:
    """``__cuda_array_interface__`` view of library-owned device memory."""

    def __init__(self, ptr: int, shape: tuple[int, ...], typestr: str):
        self.__cuda_array_interface__ = {"shape": shape, "typestr": typestr, "data": (ptr, False),
                                         "version": 3, "strides": None}


class PeerOutput:
    """An M x N output allocated by the library on every rank of ``group``
    and mapped into every other rank, so that each rank can write its rows
    into all copies (``kx_ipc_export`` / ``kx_ipc_import``)."""

    def __init__(self, m: int, n: int, dtype, group, device: int):
        import ctypes as C

        import torch
        import torch.distributed as dist

        from . import _abi, handle
        self.h = handle(device)
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.dtype = dtype
        esize = torch.empty((), dtype=dtype).element_size()
        self.row_bytes = n * esize
        self.nbytes = m * n * esize
        lib = _abi.lib
        ptr = C.c_void_p()
        err = _abi.KxError()
        _abi.raise_for(lib.kx_alloc(self.h.ptr, self.nbytes, C.byref(ptr), C.byref(err)), err)
        self.ptr = int(ptr.value)
        typestr = {torch.float32: "<f4", torch.float64: "<f8"}[dtype]
        self._owner = _CudaArray(self.ptr, (m, n), typestr)
        self.tensor = torch.as_tensor(self._owner, device=f"cuda:{device}")
        hbuf = C.create_string_buffer(_abi.KX_IPC_HANDLE_BYTES)
        _abi.raise_for(lib.kx_ipc_export(self.h.ptr, C.c_void_p(self.ptr), hbuf, C.byref(err)), err)
        handles: list = [None] * self.world
        dist.all_gather_object(handles, bytes(hbuf.raw), group=group)
        self.peers: list[int] = []
        for r, hd in enumerate(handles):
            if r == self.rank:
                self.peers.append(self.ptr)
                continue
            pp = C.c_void_p()
            _abi.raise_for(lib.kx_ipc_import(self.h.ptr, hd, C.byref(pp), C.byref(err)), err)
            self.peers.append(int(pp.value))
        self.done = torch.zeros(1, dtype=torch.int32, device=f"cuda:{device}")

    def close(self) -> None:
        """Unmap the peers' buffers and free this rank's (collective: every
        rank calls it, after its last push has completed)."""
        import ctypes as C

        import torch
        import torch.distributed as dist

        from . import _abi
        if not self.peers:
            return
        torch.cuda.synchronize(self.h.device)
        dist.barrier(group=self.group)
        for r, p in enumerate(self.peers):
            if r != self.rank:
                _abi.lib.kx_ipc_close(self.h.ptr, C.c_void_p(p))
        dist.barrier(group=self.group)
        self.tensor = None
        _abi.lib.kx_free(self.h.ptr, C.c_void_p(self.ptr))
        self.peers = []


def sharded_matmul_push(a_local, b, out: PeerOutput, plan: RowPlan, rank: int, group=None,
                        streams: dict | None = None) -> None:
    """This rank's pieces into ``out.tensor``, each pushed into every peer's
    copy by the library (copy engines while a later piece computes, an all-SM
    kernel for the last piece), then a 4-byte all-reduce on ``streams["comm"]``
    that tells every rank all pushes into its C have landed.  ``a_local`` is
    this rank's rows of A in piece order.  On return the work is enqueued on
    the current stream."""
    import torch
    import torch.distributed as dist

    c = out.tensor
    compute = torch.cuda.current_stream(c.device)
    rows_sharded(a_local, b, c, plan, rank, peer_ptrs=out.peers)
    comm = streams["comm"] if streams else torch.cuda.Stream(c.device)
    comm.wait_stream(compute)
    with torch.cuda.stream(comm):
        dist.all_reduce(out.done, group=group)
    compute.wait_stream(comm)


class ReplicatedOutput:
    """An M x N output in symmetric memory, bound on every rank of ``group``
    to one NVLink multicast object (torch's symmetric-memory rendezvous).
    ``mc`` is the multicast address of the tensor's first element;
    ``available`` is False when the node offers no multicast (callers then
    use ``PeerOutput``)."""

    def __init__(self, m: int, n: int, dtype, group, device: int):
        import torch
        import torch.distributed._symmetric_memory as symm_mem

        self.tensor = symm_mem.empty((m, n), dtype=dtype, device=f"cuda:{device}")
        self.hdl = symm_mem.rendezvous(self.tensor, group)
        self.rank = self.hdl.rank
        mc = int(self.hdl.multicast_ptr) if self.hdl.has_multicast_support else 0
        base = int(self.hdl.buffer_ptrs[self.rank])
        off = self.tensor.data_ptr() - base
        # only the unambiguous layout: the tensor starts the symmetric buffer
        self.available = mc != 0 and off == 0 and int(self.hdl.buffer_size) >= self.tensor.numel() * \
            self.tensor.element_size()
        self.mc = mc if self.available else 0
        self.row_bytes = n * self.tensor.element_size()
        self.done = torch.zeros(1, dtype=torch.int32, device=f"cuda:{device}")

    def close(self) -> None:
        self.hdl = None
        self.tensor = None


def sharded_matmul_replicated(a_pieces, b, out: ReplicatedOutput, plan: RowPlan, rank: int, group=None) -> None:
    """Compute this rank's pieces with their stores going through the
    multicast address, then one all-reduce of a 4-byte flag: once it has
    completed on a rank, every rank's rows are in that rank's C."""
    import torch.distributed as dist

    from . import matmul_into_replicated
    c = out.tensor
    for i in range(plan.pieces):
        s, e = plan.rows_of(rank, i)
        matmul_into_replicated(a_pieces[i], b, c[s:e], out.mc + s * out.row_bytes)
    dist.all_reduce(out.done, group=group)


def sharded_matmul_push_mc(a_local, b, out: ReplicatedOutput, plan: RowPlan, rank: int, group=None,
                           streams: dict | None = None) -> None:
    """As ``sharded_matmul_push``, on symmetric memory: pieces before the last
    go to the peers' buffers on the copy engines while the next piece
    computes; the last piece is stored once through the NVLink multicast
    address (each rank sends its rows once, the NVSwitch fans them out)."""
    import torch
    import torch.distributed as dist

    c = out.tensor
    compute = torch.cuda.current_stream(c.device)
    rows_sharded(a_local, b, c, plan, rank, peer_ptrs=[int(p) for p in out.hdl.buffer_ptrs], out_mc=out.mc)
    comm = streams["comm"] if streams else torch.cuda.Stream(c.device)
    comm.wait_stream(compute)
    with torch.cuda.stream(comm):
        dist.all_reduce(out.done, group=group)
    compute.wait_stream(comm)
