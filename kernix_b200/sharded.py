"""Row-sharded GEMM across the GPUs of one node, with the gathered output.

One process per GPU (torch.distributed, NCCL over NVLink/NVSwitch).  The M rows
of A are split block-cyclically into pieces of ``piece`` rows: global row block
``i * world + rank`` belongs to ``rank``.  Each rank multiplies its pieces with
its own replica of B (no data-path collective for the compute), and piece ``i``
of every rank is all-gathered straight into rows
``[i * world * piece, (i + 1) * world * piece)`` of the full C -- the gathered
layout is already C's row order.  The all-gather of piece ``i`` runs on a
communication stream while piece ``i + 1`` is being multiplied.

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
    """Largest piece <= target_piece that tiles M evenly across ranks."""
    if m % world:
        raise ValueError(f"M={m} is not divisible by world={world}")
    per_rank = m // world
    piece = min(target_piece, per_rank)
    while per_rank % piece:
        piece -= 1
    return RowPlan(m, world, piece)


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
