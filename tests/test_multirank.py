"""The N>1 (replicas) path on CPU: two gloo ranks shard batches round-robin
and reduce their timings with max, exactly as bench.py does under torchrun."""
import os
import socket

import pytest

torch = pytest.importorskip("torch")


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, n_batches, times, q):
    import sys
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "..", "jammi-ai_b200"))
    import torch.distributed as dist
    from datetime import timedelta
    from jammi_b200.sharding import max_over_ranks, shard_batches, whole_job_rate
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    mine = shard_batches(n_batches, rank, world)
    gathered = [None] * world
    dist.all_gather_object(gathered, mine)
    t = max_over_ranks(times[rank])
    dist.barrier()
    if rank == 0:
        q.put((gathered, t, whole_job_rate(len(mine), world, t)))
    dist.destroy_process_group()


def test_two_rank_sharding_and_max_time():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, 9, [1.5, 2.5], q)) for r in range(2)]
    for p in procs:
        p.start()
    gathered, t, rate = q.get(timeout=120)
    for p in procs:
        p.join(60)
        assert p.exitcode == 0
    flat = sorted(b for shard in gathered for b in shard)
    assert flat == list(range(9)), "every batch exactly once"
    assert gathered[0] == [0, 2, 4, 6, 8] and gathered[1] == [1, 3, 5, 7]
    assert t == 2.5, "timing is the max over ranks"
    assert rate == pytest.approx(5 * 2 / 2.5)


def _failing_worker(rank, world, port, mode, q):
    import sys
    import time
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "..", "jammi-ai_b200"))
    import torch.distributed as dist
    from jammi_b200.sharding import init_replica_group, max_over_ranks
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world))
    if rank == 1 and mode == "never_joins":
        time.sleep(8)
        return
    t0 = time.monotonic()
    try:
        init_replica_group("gloo", timeout_s=3.0)
        if rank == 1:  # dies between steps, nothing in flight
            os._exit(1)
        max_over_ranks(1.0)
        dist.barrier()
        q.put((rank, "no error", time.monotonic() - t0))
    except Exception as e:  # noqa: BLE001
        q.put((rank, type(e).__name__, time.monotonic() - t0))


@pytest.mark.parametrize("mode", ["dies_after_init", "never_joins"])
def test_lost_rank_ends_the_others_with_an_error(mode):
    """Failure detection on the host: a rank that exits between steps, or
    never joins, makes rank 0's next collective (or the rendezvous) raise
    within the group's short timeout instead of hanging."""
    import queue as pyqueue

    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, 2, port, mode, q)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        rank, outcome, dt = q.get(timeout=60)
    except pyqueue.Empty:
        outcome, dt, rank = "hang", None, 0
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    assert rank == 0 and outcome != "no error" and outcome != "hang", outcome
    assert dt < 30
