"""Multi-rank logic of bench.py on CPU ranks (gloo, world size 2): the barrier, the max over ranks
of the timed region, the whole-job rate from the slowest rank, and that a rank which dies before
the barrier makes the other rank fail with an error (short process-group timeout) instead of
waiting for good.  No GPU."""
from __future__ import annotations

import multiprocessing as mp
import os
import socket
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, mode: str, q) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    sys.path.insert(0, str(ROOT))
    try:
        import bench

        d = bench.Dist(world, backend="gloo", timeout_s=10.0)
        if mode == "die" and rank == 1:
            os._exit(3)  # leaves between steps, without joining the barrier
        if mode == "gather":
            import torch

            out = torch.empty((world, 3, 4), dtype=torch.float32)
            d.all_gather_into(out, torch.full((3, 4), float(rank)))
            ok = all(torch.equal(out[r], torch.full((3, 4), float(r))) for r in range(world))
            d.close()
            q.put((rank, "ok" if ok else "bad gather", 0.0, 0.0))
            return
        if mode == "shard":
            # strong scaling: the 512 heads of the fixed attention problem and the 8192 GEMM rows
            # split over the ranks; every unit is owned by exactly one rank
            import torch

            owned = torch.zeros(512 + 8192 + 4097, dtype=torch.int64)
            for off, total in ((0, 512), (512, 8192), (512 + 8192, 4097)):
                s0, cnt = bench.shard_range(total, d.world, rank)
                owned[off + s0: off + s0 + cnt] += 1
            d.dist.all_reduce(owned)
            ms = d.max(10.0 + 5.0 * rank)
            rate = bench.fixed_job_rate(8.8e12, ms)
            d.close()
            q.put((rank, "ok" if bool((owned == 1).all()) else "bad shard", ms, rate))
            return
        d.barrier()
        ms_local = 10.0 + 5.0 * rank  # rank 1 is the slow one
        ms = d.max(ms_local)
        rate = bench.whole_job_rate(1.0e9, d.world, ms)
        d.close()
        q.put((rank, "ok", ms, rate))
    except Exception as e:  # noqa: BLE001 -- reported to the parent
        q.put((rank, "error", type(e).__name__, str(e)[:200]))


def _run(world: int, mode: str, timeout: float):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
        p.join()
    out = []
    while not q.empty():
        out.append(q.get())
    return out, alive


def test_two_gloo_ranks_take_max_and_aggregate():
    out, alive = _run(2, "ok", 120)
    assert not alive
    res = {r[0]: r for r in out}
    assert set(res) == {0, 1}, out
    for r in (0, 1):
        assert res[r][1] == "ok", res[r]
        assert res[r][2] == pytest.approx(15.0)                  # max over ranks, on every rank
        assert res[r][3] == pytest.approx(2 * 1.0e9 / 15.0e-3)   # both ranks' work / slowest time


def test_dead_rank_makes_the_other_fail_not_hang():
    out, alive = _run(2, "die", 90)
    assert not alive, "a rank waited for good on a rank that died"
    res = {r[0]: r for r in out}
    assert 0 in res and res[0][1] == "error", out


def test_output_all_gather_two_ranks():
    """The sharded-output all-gather (bench.py --gather-outputs) on two gloo ranks: every rank ends up with every
    rank's shard in rank order."""
    out, alive = _run(2, "gather", 120)
    assert not alive
    assert sorted(r[:2] for r in out) == [(0, "ok"), (1, "ok")]


def test_strong_split_covers_every_unit_once():
    """The fixed problems split over two gloo ranks (bench.py strong scaling): every attention head,
    GEMM row and ragged flat range is owned by exactly one rank, and the job's rate is the whole
    problem's work over the slowest rank's time."""
    out, alive = _run(2, "shard", 120)
    assert not alive
    res = {r[0]: r for r in out}
    assert set(res) == {0, 1}, out
    for r in (0, 1):
        assert res[r][1] == "ok", res[r]
        assert res[r][3] == pytest.approx(8.8e12 / 15.0e-3)


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_shard_range_partitions(world):
    sys.path.insert(0, str(ROOT))
    import bench

    for total in (0, 1, 7, 512, 8192, 4096 * 8192):
        spans = [bench.shard_range(total, world, r) for r in range(world)]
        assert spans[0][0] == 0
        for (s0, c0), (s1, _) in zip(spans, spans[1:]):
            assert s0 + c0 == s1
        assert sum(c for _, c in spans) == total
        assert max(c for _, c in spans) - min(c for _, c in spans) <= 1
