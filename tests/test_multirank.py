"""bench.py's multi-rank plumbing (one process per GPU, replicas, no
collective on the data path) on CPU: two gloo ranks on 127.0.0.1 take the
same collective steps the GPU run takes -- barrier, max of the timings,
sum of the units -- and rank 0's whole-job throughput is all units over the
slowest rank's time."""
import os
import socket
import sys

import pytest
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, q) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    sys.path.insert(0, ROOT)
    import bench

    d = bench.Dist(backend="gloo")
    try:
        d.barrier()
        ms = 100.0 * (rank + 1)        # rank 1 is the slow one
        units = 1000.0 * (rank + 1)
        t_max = d.max(ms)
        total = d.sum(units)
        q.put((rank, t_max, total, total / (t_max / 1e3)))
    finally:
        d.close()


def test_two_gloo_ranks_aggregate_like_the_gpu_run():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    res = sorted(q.get(timeout=10) for _ in range(world))
    for rank, t_max, total, value in res:
        assert t_max == 200.0 and total == 3000.0
        assert value == pytest.approx(3000.0 / 0.2)


def _failing_rank_main(rank: int, world: int, port: int, q) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank), Q3_DIST_TIMEOUT_S="10")
    sys.path.insert(0, ROOT)
    import bench

    d = bench.Dist(backend="gloo")
    if rank == 1:  # this replica fails before the barrier and leaves
        os._exit(3)
    try:
        d.barrier()
        d.max(1.0)
        q.put((rank, "no error"))
    except Exception as e:  # the failure reaches rank 0 as an error, not a hang
        q.put((rank, type(e).__name__))


def test_a_failed_replica_is_reported_not_hung_on():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_failing_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(90)
    alive = [p.is_alive() for p in procs]
    for p in procs:
        if p.is_alive():
            p.kill()
    assert not any(alive), "a rank still waits on the failed replica"
    assert procs[1].exitcode == 3
    rank, what = q.get(timeout=10)
    assert rank == 0 and what != "no error"


def test_aggregate_is_units_over_slowest_rank():
    sys.path.insert(0, ROOT)
    import bench

    v, t = bench.aggregate([100.0, 300.0], [50.0, 200.0])
    assert t == 200.0 and v == pytest.approx(400.0 / 0.2)


def test_single_process_dist_is_a_no_op():
    sys.path.insert(0, ROOT)
    import bench

    d = bench.Dist(backend="gloo")
    assert d.world == 1 and d.max(3.0) == 3.0 and d.sum(4.0) == 4.0
    d.barrier()
    d.close()


def test_step_roofline_is_the_per_step_fraction():
    """The headline roofline: algorithmic bytes of a step over the measured
    step time against the peak; the dominant kind from the live trace keeps
    its own figures; traffic per step only when every kind was captured."""
    import bench

    kern = {"fused_attn": {"total_us_per_step": 200.0, "achieved_gbs": 1000.0,
                           "launches_per_step": 28, "alg_bytes_per_launch": 7e6},
            "vocab": {"total_us_per_step": 50.0, "achieved_gbs": 6000.0, "launches_per_step": 1,
                      "alg_bytes_per_launch": 311e6}}
    r = bench.step_roofline(8e8, 0.4, kern, 6400.0, "measured", "fused", 57,
                            {"fused_attn": 7.1e6, "vocab": 3.12e8})
    assert r["achieved"] == pytest.approx(8e8 / 0.4e-3 / 1e9)
    assert r["frac"] == pytest.approx(r["achieved"] / 6400.0)
    assert r["dominant_kernel"]["name"] == "fused_attn"
    assert r["traffic"] == pytest.approx(28 * 7.1e6 + 3.12e8)
    r2 = bench.step_roofline(8e8, 0.4, kern, 6400.0, "measured", "fused", 57, {"vocab": 1.0})
    assert r2["traffic"] is None and r2["dominant_kernel"]["traffic"] is None


def test_kernel_bytes_count_weights_and_kv():
    import bench

    a0 = bench.kernel_alg_bytes("fused_attn", 0)
    a9 = bench.kernel_alg_bytes("fused_attn", 9)
    assert a9 - a0 == 9 * bench.KV_BYTES_W
    assert bench.kernel_alg_bytes("fused_ffn", 100) == bench.kernel_alg_bytes("fused_ffn", 0)
