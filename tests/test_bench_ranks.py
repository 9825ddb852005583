"""bench.py's multi-process plumbing on two gloo ranks (CPU): the barrier,
the max over ranks of every timed quantity, and the whole-job aggregate the
driver reads for `--gpus N` (each rank's units over the slowest rank's
time).  The GPU work itself is not involved."""
import multiprocessing as mp
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _rank(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    sys.path.insert(0, ROOT)
    import bench
    bench._init_dist(world)
    bench._barrier(world)()
    # rank r "took" 1 + r seconds for 16 tokens x 3 steps
    slowest = bench._max_over_ranks(1.0 + rank, world)
    value = 16 * 3 * world / slowest
    bench._barrier(world)()
    bench._pg.destroy_process_group()
    out.put((rank, slowest, value))


def test_max_over_ranks_and_aggregate_on_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = 29000 + os.getpid() % 1000
    procs = [ctx.Process(target=_rank, args=(r, 2, port, out)) for r in range(2)]
    for p in procs:
        p.start()
    got = sorted(out.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert got == [(0, 2.0, 48.0), (1, 2.0, 48.0)]


def test_single_rank_needs_no_process_group():
    sys.path.insert(0, ROOT)
    import bench
    assert bench._max_over_ranks(3.5, 1) == 3.5
    bench._barrier(1)()  # no-op
