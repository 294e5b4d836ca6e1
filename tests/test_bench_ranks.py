"""Host-side logic of the multi-GPU bench on CPU: two `gloo` ranks (world
size 2, 127.0.0.1 rendezvous) run bench.py's max-over-ranks reduction, the
whole-job GB/s aggregation and the utterance sharding, as the torchrun ranks
of `bench.py --gpus 2` do over NCCL."""
import multiprocessing as mp
import os
import socket
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, q):
    try:
        sys.path.insert(0, ROOT)
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        import datetime
        import torch
        import bench
        torch.distributed.init_process_group("gloo", rank=rank, world_size=world,
                                             timeout=datetime.timedelta(seconds=60))
        # rank r reports (10 + r) ms for the step and (20 - r) ms for the e2e step
        ms, ms_e2e = bench.max_over_ranks([10.0 + rank, 20.0 - rank], world, device="cpu")
        gbs = bench.aggregate_gbs(bench.STEP_BYTES, 5, world, ms)
        shard = bench.utterances_per_rank(64, world)
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
        q.put((rank, ms, ms_e2e, gbs, shard))
    except Exception as e:  # surfaced by the parent
        q.put((rank, "error", repr(e), None, None))


def test_two_gloo_ranks_agree_on_max_and_aggregate():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    assert all(p.exitcode == 0 for p in procs)
    sys.path.insert(0, ROOT)
    import bench
    for rank, ms, ms_e2e, gbs, shard in out:
        assert ms != "error", ms_e2e
        assert ms == 11.0 and ms_e2e == 20.0          # the slowest rank of each
        assert gbs == pytest.approx(2 * bench.STEP_BYTES * 5 / 11e-3 / 1e9)
        assert shard == 32


def test_single_rank_helpers_need_no_process_group():
    sys.path.insert(0, ROOT)
    import bench
    assert bench.max_over_ranks([3.0, 4.0], 1, device="cpu") == [3.0, 4.0]
    assert bench.utterances_per_rank(64, 8) == 8 and bench.utterances_per_rank(3, 8) == 1
