"""Host-side dispatch of utterance batches over per-GPU workers
(voxcpm-cpp_b200/dispatch.py), on the CPU: a worker that fails gives its
batch back, the other workers finish it, and every utterance is done exactly
once -- with threads, and with two gloo ranks sharing a TCPStore."""
import os
import socket
import threading

import pytest

import dispatch as D


def double(batch):
    return [2 * u for u in batch]


def test_threads_requeue_a_failed_workers_batch():
    calls = {"bad": 0, "good": 0}
    seen = []
    lock = threading.Lock()

    def bad(batch):
        calls["bad"] += 1
        raise RuntimeError("vcpm_b200 error 5: injected")

    def good(batch):
        with lock:
            calls["good"] += 1
            seen.extend(batch)
        return double(batch)

    items = list(range(23))
    out = D.run_threads(items, [bad, good, good], batch=4)
    assert out == {u: 2 * u for u in items}
    assert sorted(seen) == items          # each utterance ran once on a live worker
    assert calls["bad"] == 1              # the failed worker took no more batches


def test_threads_fail_when_every_worker_fails():
    def bad(batch):
        raise RuntimeError("down")

    with pytest.raises(D.DispatchError):
        D.run_threads(list(range(5)), [bad, bad], batch=2)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank_main(rank, world, port, n_items, fail_rank, q):
    import datetime

    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    store = dist.distributed_c10d._get_default_store()
    state = {"n": 0}

    def fn(batch):
        state["n"] += 1
        if rank == fail_rank and state["n"] == 1:
            raise RuntimeError("vcpm_b200 error 5: injected device failure")
        return double(batch)

    mine = D.run_ranks(list(range(n_items)), fn, 3, store, rank, world, timeout_s=60)
    dist.barrier()
    q.put((rank, sorted(mine.items()), state["n"]))
    dist.destroy_process_group()


def test_gloo_ranks_requeue_a_failed_ranks_batch():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port, world, n_items = _free_port(), 2, 20
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, n_items, 1, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    got = {}
    for rank, items, n in res:
        for u, v in items:
            assert u not in got
            got[u] = v
        if rank == 1:
            assert n == 1 and not items       # failed on its first batch and stopped
    assert got == {u: 2 * u for u in range(n_items)}
