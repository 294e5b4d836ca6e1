"""Host-side dispatch of independent utterances over per-GPU workers.

Utterances share nothing (each owns its KV slots, state rows and noise
stream, src/generate.h:155-212), so a multi-GPU host runs one worker per GPU
-- a thread with its own vb_ctx, or one process per GPU -- and hands each
worker batches of utterances from one queue.  A worker whose call fails (an
exception, or a non-zero vcpm_status raised as VBError) gives its batch back:
the batch goes to the other workers and the failed worker takes no more.
Only when no worker is left does the run fail.

Two forms:
  run_threads(items, workers, batch)   one process, one thread per worker
  run_ranks(items, fn, batch, store)   one process per GPU; the queue lives in
                                       a torch.distributed key-value store
                                       (TCPStore / the process group's store)
"""
from __future__ import annotations

import queue
import threading
import time


class DispatchError(RuntimeError):
    pass


def batches(items, batch):
    items = list(items)
    return [items[i:i + batch] for i in range(0, len(items), batch)]


def run_threads(items, workers, batch):
    """Runs every item through one of `workers` (callables taking a list of
    items and returning one result per item) in batches of `batch`.  Returns
    {item: result}.  A worker that raises returns its batch to the queue and
    stops; raises DispatchError if every worker has failed with work left."""
    q: queue.Queue = queue.Queue()
    for b in batches(items, batch):
        q.put(b)
    results, errors = {}, []
    lock = threading.Lock()
    live = [len(workers)]
    pending = [q.qsize()]
    done = threading.Event()
    if pending[0] == 0:
        return results

    def loop(i, fn):
        while not done.is_set():
            try:
                b = q.get(timeout=0.05)
            except queue.Empty:
                continue
            try:
                out = fn(b)
                if len(out) != len(b):
                    raise DispatchError(f"worker {i} returned {len(out)} results for {len(b)} items")
            except Exception as e:  # noqa: BLE001 -- any failure re-queues the batch
                with lock:
                    errors.append((i, e))
                    live[0] -= 1
                    q.put(b)
                    if live[0] == 0:
                        done.set()
                return
            with lock:
                results.update(zip(b, out))
                pending[0] -= 1
                if pending[0] == 0:
                    done.set()

    threads = [threading.Thread(target=loop, args=(i, fn), daemon=True) for i, fn in enumerate(workers)]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    if len(results) != len(list(items)):
        raise DispatchError(f"{len(items) - len(results)} items left, every worker failed: "
                            + "; ".join(f"worker {i}: {e}" for i, e in errors))
    return results


def run_ranks(items, fn, batch, store, rank, world, timeout_s=120.0, poll_s=0.01):
    """One process per GPU: every rank calls this with the same items.  A
    single counter in `store` hands out claims in order: claim i < nb is
    batch i; claim nb + k is the k-th re-queued batch, which the holder waits
    for.  A rank whose fn raises publishes its batch as the next re-queued
    entry and stops claiming.  Every batch is completed by exactly one rank
    (done markers are counted), and the call returns on every rank once all
    batches are done -- with the {item: result} of the batches this rank
    completed -- or raises DispatchError when they are not done within
    `timeout_s` (no live rank left)."""
    bs = batches(items, batch)
    nb = len(bs)
    mine = {}
    t0 = time.monotonic()

    def all_done():
        return store.add("dispatch/done_n", 0) >= nb

    def late():
        return time.monotonic() - t0 > timeout_s

    claim = None
    while not all_done():
        if claim is None:
            claim = store.add("dispatch/next", 1) - 1
        if claim < nb:
            i = claim
        else:
            k = claim - nb
            if store.add("dispatch/requeue_n", 0) <= k:
                if late():
                    raise DispatchError(f"rank {rank}: batches still open after {timeout_s} s")
                time.sleep(poll_s)
                continue
            i = int(store.get(f"dispatch/requeue/{k}").decode())
        claim = None
        try:
            out = fn(bs[i])
            if len(out) != len(bs[i]):
                raise DispatchError(f"rank {rank} returned {len(out)} results for {len(bs[i])} items")
        except Exception:  # noqa: BLE001 -- any failure re-queues the batch
            # publish the entry before counting it, so a holder that sees the
            # count finds the entry
            k = store.add("dispatch/requeue_pub", 1) - 1
            store.set(f"dispatch/requeue/{k}", str(i))
            store.add("dispatch/requeue_n", 1)
            while not all_done():
                if late():
                    raise DispatchError(f"rank {rank}: batches still open after {timeout_s} s")
                time.sleep(poll_s)
            return mine
        store.set(f"dispatch/done/{i}", str(rank))
        store.add("dispatch/done_n", 1)
        mine.update(zip(bs[i], out))
    return mine
