"""Data-parallel host logic on CPU: two gloo ranks in spawned processes.

The forward shards pages across GPUs with no data-path collective; the only
cross-rank steps are the timing barrier and the max / sum reductions of the
bench.  These tests run that logic with world_size 2 on the CPU: reductions,
disjoint page shards per rank, the whole-job rate taken at the slowest rank,
and a rank that leaves before a collective (the survivor must get an error
within the process-group timeout instead of waiting).
"""
import os
import socket
import sys

import pytest
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _env(rank, world, port):
    os.environ.update({"RANK": str(rank), "WORLD_SIZE": str(world), "LOCAL_RANK": str(rank),
                       "MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port)})
    sys.path.insert(0, ROOT)


def _worker_reductions(rank, world, port, out):
    _env(rank, world, port)
    import hashlib
    import bench
    w, r, _, pg = bench.dist_setup(None, timeout_s=30)
    try:
        assert (w, r) == (world, rank)
        bench.barrier(pg)
        res = {"max": bench.max_over_ranks(pg, 10.0 + rank),
               "sum": bench.sum_over_ranks(pg, 1.0 + rank)}
        pages = bench._fwd_pages(rank, 2)
        res["digest"] = [hashlib.sha256(p.tobytes()).hexdigest() for p in pages]
        # rank 1 is the slow one: the job rate must use its time
        ms = bench.max_over_ranks(pg, 100.0 if rank == 0 else 250.0)
        res["rate"] = bench.job_rate(8, 10, w, ms)
        out[rank] = res
    finally:
        pg.destroy_process_group()


def _worker_dropout(rank, world, port, out):
    _env(rank, world, port)
    import bench
    _, _, _, pg = bench.dist_setup(None, timeout_s=5)
    bench.barrier(pg)
    if rank == 1:
        os._exit(0)  # leaves between steps, with nothing in flight
    try:
        bench.barrier(pg)
        out[rank] = "no error"
    except Exception as e:  # noqa: BLE001 - any collective error is the expected outcome
        out[rank] = "error: " + type(e).__name__


def _run(fn, world=2):
    ctx = mp.get_context("spawn")
    with ctx.Manager() as m:
        out = m.dict()
        port = _free_port()
        procs = [ctx.Process(target=fn, args=(r, world, port, out)) for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(120)
            if p.is_alive():
                p.kill()
                pytest.fail("a rank did not finish")
        return dict(out), [p.exitcode for p in procs]


def test_two_rank_reductions_shards_and_rate():
    out, codes = _run(_worker_reductions)
    assert codes == [0, 0]
    for r in (0, 1):
        assert out[r]["max"] == 11.0
        assert out[r]["sum"] == 3.0
        # 8 pages per rank per step, 10 steps, 2 ranks, slowest rank 250 ms
        assert out[r]["rate"] == pytest.approx(8 * 10 * 2 / 0.25)
    assert not set(out[0]["digest"]) & set(out[1]["digest"]), "ranks must see distinct pages"


def test_rank_that_leaves_fails_the_survivor_within_the_timeout():
    out, codes = _run(_worker_dropout)
    assert codes[1] == 0
    assert out.get(0, "").startswith("error"), out
