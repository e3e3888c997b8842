"""Row-sharded GEMM schedule across ranks, on CPU with gloo (world size 2 and 3).

The device kernel is replaced by a host matmul (injected ``matmul_into``) so
the host-side logic -- block-cyclic piece plan, per-piece all-gather straight
into C's rows, strided A views -- is checked without a GPU.
"""
import os
import socket

import numpy as np
import pytest

from kernix_b200.sharded import plan_rows


def test_plan_covers_rows_once_and_gathers_in_order():
    for m, world, piece in [(8192, 8, 512), (8192, 2, 1024), (96, 3, 8), (10, 5, 100)]:
        plan = plan_rows(m, world, target_piece=piece)
        owned = sorted(r for rank in range(world) for r in plan.local_rows(rank))
        assert owned == list(range(m))
        for i in range(plan.pieces):
            g0, g1 = plan.gathered_rows(i)
            concat = [r for rank in range(world) for r in range(*plan.rows_of(rank, i))]
            assert concat == list(range(g0, g1))
    with pytest.raises(ValueError):
        plan_rows(10, 3)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, m, k, n, piece, q):
    import torch
    import torch.distributed as dist
    from kernix_b200.sharded import plan_rows, sharded_matmul

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        stride = k + 5
        rng = np.random.default_rng(0)
        abuf = rng.uniform(-1, 1, (m, stride)).astype(np.float32)    # A = abuf[:, :k]
        b = torch.from_numpy(rng.uniform(-1, 1, (k, n)).astype(np.float32))
        plan = plan_rows(m, world, target_piece=piece)
        mine = plan.local_rows(rank)
        local = torch.from_numpy(abuf[mine].reshape(-1).copy())
        # strided pieces of the local buffer (row stride k + 5), like the bench's TensorViews
        pieces = [torch.as_strided(local, (plan.piece, k), (stride, 1), i * plan.piece * stride)
                  for i in range(plan.pieces)]
        c = torch.full((m, n), float("nan"))

        def host_matmul_into(a, bb, out):
            out.copy_(a.double().matmul(bb.double()).float())

        sharded_matmul(pieces, b, c, plan, rank, matmul_into=host_matmul_into)
        want = abuf[:, :k].astype(np.float64) @ b.numpy().astype(np.float64)
        q.put((rank, float(np.max(np.abs(c.numpy() - want))), bool(np.isnan(c.numpy()).any())))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,m,piece", [(2, 96, 16), (3, 96, 8)])
def test_sharded_matmul_gathers_full_product(world, m, piece):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, m, 40, 24, piece, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, err, has_nan in results:
        assert not has_nan, rank
        assert err < 1e-5, (rank, err)


def test_stream_windows_reassemble_the_unsharded_inputs():
    """The batch-sharded attention and conv measurements have every rank
    generate its own window of the seeded streams; the windows of all ranks
    put together must be the single-process inputs."""
    from kernix_b200 import rng
    total, world = 12, 4            # values per batch element: 6 (even, as normal() pairs them)
    per = 6
    full = rng.normal(7, 3 * total * per, 1.0, np.float64)
    cnt = total // world * per
    for j in range(3):              # Q, K, V: consecutive segments of one stream
        parts = [rng.normal(7, cnt, 1.0, np.float64, start=j * cnt * world + r * cnt) for r in range(world)]
        assert np.array_equal(np.concatenate(parts), full[j * total * per:(j + 1) * total * per])
    full_u = rng.uniform(8, total * per, -1.0, 1.0, np.float32)
    parts = [rng.uniform(8, cnt, -1.0, 1.0, np.float32, start=r * cnt) for r in range(world)]
    assert np.array_equal(np.concatenate(parts), full_u)
    with pytest.raises(ValueError):
        rng.normal(7, 4, start=3)


def test_library_plans_partition_the_work():
    """kx_shard_window and kx_row_piece (host-only C entries): windows cover
    every unit once, in rank order, differing in size by at most one; row
    pieces tile M and are the largest divisor of the per-rank rows within the
    target."""
    from kernix_b200.sharded import shard_window
    for total in (0, 1, 5, 16, 64, 67):
        for world in (1, 2, 3, 4, 8):
            wins = [shard_window(total, r, world) for r in range(world)]
            assert sum(c for _, c in wins) == total
            assert all(wins[r][0] + wins[r][1] == wins[r + 1][0] for r in range(world - 1))
            assert max(c for _, c in wins) - min(c for _, c in wins) <= 1
    for m, world, target in ((8192, 8, 512), (8192, 2, 512), (96, 3, 10), (8192, 8, 768)):
        plan = plan_rows(m, world, target_piece=target)
        per_rank = m // world
        assert per_rank % plan.piece == 0 and plan.piece <= target
        assert all(per_rank % p for p in range(plan.piece + 1, min(target, per_rank) + 1))
