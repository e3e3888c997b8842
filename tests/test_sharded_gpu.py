"""kx_matmul_rows_sharded_f32 on one GPU, the other ranks' outputs stood in
for by local buffers (the copy engines and the push kernel write to them as to
a peer's memory): every piece of this rank lands in its rows of every output,
nothing else is written, and the values meet the f32 bound against the
compensated oracle -- for the plain schedule and for the split last piece
(two row halves, each one GEMM batched over its two K halves, and a sum)
that a large fan-out selects.
Restates the row-chunk contract of CpuExecutor::matmul_into
(execution.rs:188-233) for rows owned by one rank of a node.
"""
import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("world,rank,k,launches", [(4, 1, 2048, 6), (2, 0, 2048, 3)])
def test_rank_rows_reach_every_output(kx, torch_cuda, world, rank, k, launches):
    torch = torch_cuda
    from kernix_b200 import rng
    from kernix_b200.sharded import plan_rows, rows_sharded
    n, piece, pieces = 8192, 512, 2
    m = world * pieces * piece
    plan = plan_rows(m, world, piece)
    assert (plan.piece, plan.pieces) == (piece, pieces)
    pitch = k + 64                                       # A rows as a strided slice
    a_buf = rng.uniform(121, pieces * piece * pitch, -1, 1).reshape(pieces * piece, pitch)
    b_np = rng.uniform(122, k * n, -1, 1).reshape(k, n)
    a_local = torch.from_numpy(a_buf).cuda()[:, :k]
    b = torch.from_numpy(b_np).cuda()
    outs = [torch.full((m, n), float("nan"), device="cuda") for _ in range(world)]
    h = kx.handle(0)
    h.set_f32_variant(0)
    before = h.launches
    rows_sharded(a_local, b, outs[rank], plan, rank, peer_ptrs=[o.data_ptr() for o in outs])
    torch.cuda.synchronize()
    assert h.launches - before == launches
    mine = plan.local_rows(rank)
    mask = torch.zeros(m, dtype=torch.bool)
    mask[mine] = True
    for r, o in enumerate(outs):
        assert torch.equal(o[mine], outs[rank][mine]), r
        assert bool(torch.isnan(o[~mask.cuda()]).all()), r          # no other row written
    sample = [0, 300, 511, 512, 700, 767, 768, 1000, 1023]            # local rows: both pieces, both tail halves
    got = outs[rank][[mine[i] for i in sample]].cpu().numpy().astype(np.float64)
    want, absum = oracle.gemm_dot2(oracle.View(np.ascontiguousarray(a_buf[sample, :k]), (len(sample), k), (k, 1)),
                                   oracle.View.of(b_np))
    assert (np.abs(got - want) <= 2e-6 * absum).all()
