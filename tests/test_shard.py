"""Multi-GPU partitioning logic, exercised with world_size 2 `gloo` ranks on CPU.

The compute step is the CPU oracle (the kernels need a GPU); what is tested is
that the per-rank pieces cover every unit exactly once and that the gather
reassembles the single-process result bit for bit."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import oracle as O
from triton_msl_b200 import shard


@pytest.mark.parametrize("n,world,align", [(10, 3, 1), (2048, 8, 1), (8192, 8, 128),
                                           (1000, 8, 128), (5, 8, 1), (0, 2, 1)])
def test_unit_ranges_partition(n, world, align):
    rs = [shard.unit_range(n, world, r, align) for r in range(world)]
    assert rs[0][0] == 0 and rs[-1][1] == n
    for (a0, a1), (b0, b1) in zip(rs, rs[1:]):
        assert a1 == b0 and a0 <= a1
    for a, b in rs:
        assert a % align == 0 or a == n
    sizes = [b - a for a, b in rs]
    assert max(sizes) - min(sizes) <= align


def test_unit_range_rejects_bad_args():
    with pytest.raises(ValueError):
        shard.unit_range(10, 2, 2)
    with pytest.raises(ValueError):
        shard.unit_range(10, 0, 0)


def test_attention_shard_views():
    q = torch.randn(2, 3, 16, 8)
    parts = [shard.attention_shard(q, q, q, 4, r) for r in range(4)]
    got = torch.cat([p[0][0] for p in parts], 0)
    assert torch.equal(got, q.reshape(6, 16, 8))
    assert parts[0][0].data_ptr() == q.data_ptr()   # a view, no copy


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(0)
        q, k, v = (torch.randn(2, 3, 40, 16, generator=g) for _ in range(3))
        ql, kl, vl, (lo, hi) = shard.attention_shard(q, k, v, world, rank)
        o_local = O.ref_attention(ql, kl, vl, causal=True)
        ranges = [shard.unit_range(6, world, r) for r in range(world)]
        o = shard.gather(o_local[0], ranges, 0).view(2, 3, 40, 16)
        ok_fa = torch.equal(o, O.ref_attention(q, k, v, causal=True))
        a = torch.randn(300, 64, generator=g)
        b = torch.randn(64, 32, generator=g)
        al, _ = shard.gemm_shard(a, world, rank)
        c = shard.gather(a.new_tensor(al @ b), [shard.unit_range(300, world, r, 128) for r in range(world)], 0)
        ok_gemm = torch.equal(c, a @ b)
        x = torch.randn(37, 50, generator=g)
        xl, _ = shard.rows_shard(x, world, rank)
        s = shard.gather(O.ref_argmax(xl), [shard.unit_range(37, world, r) for r in range(world)], 0)
        ok_rows = torch.equal(s, O.ref_argmax(x))
        results[rank] = (ok_fa, ok_gemm, ok_rows)
    finally:
        dist.destroy_process_group()


def test_two_rank_gather_reassembles_single_process_result():
    world = 2
    with mp.Manager() as m:
        results = m.dict()
        mp.spawn(_worker, args=(world, _free_port(), results), nprocs=world, join=True)
        assert dict(results) == {0: (True, True, True), 1: (True, True, True)}


def _failing_worker(rank, world, port, results):
    import datetime
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        results[rank] = "left"
        os._exit(0)   # this rank leaves between steps, before the gather
    try:
        local = torch.ones(3, 4)
        shard.gather(local, [(0, 3), (3, 6)], 0)
        results[rank] = "gather returned"
    except Exception as e:  # noqa: BLE001 - any collective error is the expected outcome
        results[rank] = f"error: {type(e).__name__}"


def test_surviving_rank_gets_an_error_not_a_hang():
    world = 2
    ctx = mp.get_context("spawn")
    with mp.Manager() as m:
        results = m.dict()
        procs = [ctx.Process(target=_failing_worker, args=(r, world, _free_port_shared[0], results))
                 for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=60)
        alive = [p for p in procs if p.is_alive()]
        for p in alive:
            p.kill()
        assert not alive, "a rank hung"
        assert results[1] == "left"
        assert results[0].startswith("error")


_free_port_shared = [_free_port()]


def test_host_pipeline_chunk_bounds():
    from triton_msl_b200.host_pipeline import _chunk_bounds
    # default: 10/16, 5/16, 1/16 of the (batch, head) slices, largest first
    assert _chunk_bounds(64, None) == [0, 40, 60, 64]
    assert _chunk_bounds(2048, None) == [0, 1280, 1920, 2048]
    # uploads overlapping the previous read-back: 2/3 and 1/3
    assert _chunk_bounds(64, None, True) == [0, 43, 64]
    for bh in range(1, 70):
        for chunks, ready in [(c, r) for c in (None, 1, 2, 3, 4, 64, 1000) for r in (False, True)]:
            b = _chunk_bounds(bh, chunks, ready)
            assert b[0] == 0 and b[-1] == bh
            assert all(x < y for x, y in zip(b, b[1:])), (bh, chunks, b)
            if chunks is not None:
                assert len(b) - 1 == min(chunks, bh)
