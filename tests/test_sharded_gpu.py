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


def _sharded_case(kx, torch, devices, m, k, n, gather, seed):
    """kx_gemm_sharded_f32 over handles on `devices` (one process): windows of
    A's rows per handle, B replicated, one output per handle on its own stream."""
    from kernix_b200.sharded import gemm_sharded, shard_window
    rs = np.random.default_rng(seed)
    a_np = rs.uniform(-1, 1, (m, k)).astype(np.float32)
    b_np = rs.uniform(-1, 1, (k, n)).astype(np.float32)
    handles = [kx.Handle(d) for d in devices]
    streams = []
    a_w, b_r, outs = [], [], []
    for r, (d, h) in enumerate(zip(devices, handles)):
        s0, c0 = shard_window(m, r, len(devices))
        a_w.append(torch.from_numpy(a_np[s0:s0 + c0]).to(f"cuda:{d}"))
        b_r.append(torch.from_numpy(b_np).to(f"cuda:{d}"))
        outs.append(torch.full((m, n), float("nan"), device=f"cuda:{d}"))
        s = torch.cuda.Stream(device=d)
        s.wait_stream(torch.cuda.current_stream(d))         # inputs written before the handle's work
        h.set_stream(s)
        streams.append(s)
    gemm_sharded(handles, a_w, b_r, outs, gather_out=gather)
    for h in handles:
        h.synchronize()
    return a_np, b_np, outs, handles


@pytest.mark.parametrize("m,k,n", [(1000, 768, 1024), (7, 33, 12), (3, 16, 8)])
@pytest.mark.parametrize("gather", [True, False])
def test_gemm_sharded_two_handles_one_process(kx, torch_cuda, m, k, n, gather):
    """Two handles on one GPU, each on its own stream, stand in for two GPUs
    (the window copies are then device-to-device on one GPU): with the gather
    every output holds the whole product, equal everywhere and within the f32
    bound of the compensated oracle; without it each output holds exactly its
    own window's rows."""
    torch = torch_cuda
    from kernix_b200.sharded import shard_window
    a_np, b_np, outs, handles = _sharded_case(kx, torch, [0, 0], m, k, n, gather, m + k + n)
    want, absum = oracle.gemm_dot2(oracle.View.of(a_np.astype(np.float64)), oracle.View.of(b_np.astype(np.float64)))
    for r, o in enumerate(outs):
        got = o.cpu().numpy().astype(np.float64)
        s0, c0 = shard_window(m, r, 2)
        rows = np.arange(m) if gather else np.arange(s0, s0 + c0)
        assert (np.abs(got[rows] - want[rows]) <= 2e-6 * absum[rows] + 1e-30).all(), r
        if not gather:
            others = np.setdiff1d(np.arange(m), rows)
            assert np.isnan(got[others]).all(), r
    if gather:
        assert torch.equal(outs[0], outs[1])
    for h in handles:
        h.close()


def test_gemm_sharded_across_gpus(kx, torch_cuda):
    """The same on two GPUs when the box has them (peer copies over NVLink)."""
    torch = torch_cuda
    if torch.cuda.device_count() < 2:
        pytest.skip("one GPU on this box")
    a_np, b_np, outs, handles = _sharded_case(kx, torch, [0, 1], 2048, 1024, 2048, True, 5)
    assert torch.equal(outs[0].cpu(), outs[1].cpu())
    rows = [0, 1023, 1024, 2047]
    want, absum = oracle.gemm_dot2(oracle.View.of(a_np[rows].astype(np.float64)),
                                   oracle.View.of(b_np.astype(np.float64)))
    assert (np.abs(outs[1].cpu().numpy()[rows].astype(np.float64) - want) <= 2e-6 * absum).all()
    for h in handles:
        h.close()
