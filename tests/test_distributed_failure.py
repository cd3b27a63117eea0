"""Failure detection across ranks, made on the host (CPU, gloo, spawned processes): a rank that
leaves between steps is seen by the survivors before their next launch (StepMonitor over a
TCPStore), a rank that never arrives turns into RankTimeout, and a collective that a peer never
joins ends with an error after the process group's short timeout instead of blocking."""
import multiprocessing as mp
import os
import socket
import time


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _monitor_worker(rank, world, port, q, mode):
    from datetime import timedelta

    import torch.distributed as dist
    from prismaquant_b200 import distributed as D
    store = dist.TCPStore("127.0.0.1", port, world, is_master=(rank == 0), timeout=timedelta(seconds=30))
    mon = D.StepMonitor(store, rank, world, timeout=3.0)
    try:
        mon.arrive(0)
        mon.check(0)
        if rank == 1:
            if mode == "leave":
                mon.leave()          # between steps: nothing of rank 1 in flight
            # mode "vanish": rank 1 just stops, without a word
            q.put((rank, "stopped", None))
            time.sleep(5.0)
            return
        mon.arrive(1)
        t0 = time.monotonic()
        try:
            mon.check(1)
            q.put((rank, "no error", None))
        except (D.RankLeft, D.RankTimeout) as e:
            q.put((rank, type(e).__name__, time.monotonic() - t0))
    except Exception as e:  # pragma: no cover - reported to the parent
        q.put((rank, f"unexpected {type(e).__name__}: {e}", None))


def _run(target, world, *args, timeout=60):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, world, port, q) + args) for r in range(world)]
    for p in procs:
        p.start()
    try:
        res = sorted(q.get(timeout=timeout) for _ in procs)
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    return res


def test_rank_that_leaves_between_steps_is_seen_on_the_host():
    res = _run(_monitor_worker, 2, "leave")
    assert res[0][1] == "RankLeft", res
    assert res[0][2] < 2.0            # seen at once, not after the timeout
    assert res[1][1] == "stopped"


def test_rank_that_vanishes_times_out_on_the_host():
    res = _run(_monitor_worker, 2, "vanish")
    assert res[0][1] == "RankTimeout", res
    assert 2.5 < res[0][2] < 10.0


def _pg_timeout_worker(rank, world, port, q):
    from datetime import timedelta

    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=2))
    if rank == 1:                     # never joins the collective
        q.put((rank, "absent", None))
        time.sleep(8.0)
        os._exit(0)
    t0 = time.monotonic()
    try:
        dist.all_reduce(torch.ones(4))
        q.put((rank, "no error", None))
    except Exception:
        q.put((rank, "raised", time.monotonic() - t0))
    os._exit(0)                       # the group is broken; do not wait on it


def test_collective_without_a_peer_ends_with_an_error():
    res = _run(_pg_timeout_worker, 2)
    assert res[0][1] == "raised", res
    assert res[0][2] < 7.0            # the 2 s group timeout, not the peer's 8 s
