"""The request dispatcher (itts_gpt.serve) on CPU with fake engines: continuous
batching over a shared queue, and failure isolation by fault injection on the host (a
worker whose engine raises mid-run or at start-up).  The cross-process queue runs as two
gloo ranks sharing one torch.distributed store."""
import datetime
import os
import sys
import threading
import time
from pathlib import Path

import pytest
import torch.multiprocessing as mp

from itts_gpt import ValidationError
from itts_gpt.serve import Dispatcher, Request, RequestQueue, StoreQueue, Worker

BAD = {13, 77}  # requests whose admission the fake engine rejects

ROOT = Path(__file__).resolve().parent.parent


def _len(req):
    return 1 + (req.id * 37) % 23


def _codes(req):
    return [(req.id * 131 + i) % 8192 for i in range(_len(req))]


class FakeEngine:
    """Stands in for SlotEngine: request r needs _len(r) steps; decode() runs `chunk`
    steps at a time until one finishes; raises after `fail_after` decode calls."""

    def __init__(self, max_batch=4, chunk=3, fail_after=None, log=None):
        self.max_batch, self.chunk, self.fail_after = max_batch, chunk, fail_after
        self.live, self.calls, self.log = {}, 0, log if log is not None else []

    def admit(self, pairs):
        for s, r in pairs:
            if r.id in BAD:
                raise ValidationError(f"validation error on `text_tokens`: request {r.id}")
        for s, r in pairs:
            assert s not in self.live and 0 <= s < self.max_batch
            self.live[s] = [r, 0]
        self.log.append(("admit", [r.id for _, r in pairs]))

    def decode(self):
        time.sleep(0.001)  # a device step takes time: the other workers get to draw too
        self.calls += 1
        if self.fail_after is not None and self.calls > self.fail_after:
            raise RuntimeError("device error: injected fault")
        while True:
            done = [s for s, (r, n) in self.live.items() if n >= _len(r)]
            if done:
                return done
            for v in self.live.values():
                v[1] += self.chunk

    def collect(self, slot):
        r, _ = self.live.pop(slot)
        return _codes(r), r.id ^ 0x5555, 0


def _requests(n):
    return [Request(i, prompt=None, params=None, seed=i) for i in range(n)]


def _check_all(results, n):
    assert sorted(results) == list(range(n))
    for i, res in results.items():
        if i in BAD:  # rejected alone, with the library's message
            assert res.error and "ValidationError" in res.error and not res.codes, (i, res.error)
            continue
        assert res.error is None, (i, res.error)
        assert res.codes == _codes(Request(i, None, None, i))
        assert res.rng_state == i ^ 0x5555


def test_dispatcher_serves_every_request_once():
    d = Dispatcher([lambda: FakeEngine(max_batch=4), lambda: FakeEngine(max_batch=7),
                    lambda: FakeEngine(max_batch=1)])
    res = d.run(RequestQueue(_requests(200)))
    _check_all(res, 200)
    assert sum(w.served for w in d.workers) == 200 - len(BAD)
    assert all(w.served > 0 for w in d.workers)


def test_continuous_batching_refills_freed_slots():
    log = []
    eng = FakeEngine(max_batch=3, chunk=1, log=log)
    w = Worker(0, lambda: eng)
    q = RequestQueue(_requests(10))
    out = {}
    w.serve(q, lambda r: out.__setitem__(r.id, r))
    _check_all(out, 10)
    admits = [ids for kind, ids in log if kind == "admit"]
    assert admits[0] == [0, 1, 2]          # the first fill takes every slot
    assert all(len(a) <= 3 for a in admits) and sum(map(len, admits)) == 10
    assert len(admits) > 3                 # later requests enter as slots free up


def test_failed_worker_requests_are_requeued():
    d = Dispatcher([lambda: FakeEngine(max_batch=8, fail_after=2), lambda: FakeEngine(max_batch=4),
                    lambda: FakeEngine(max_batch=4)])
    res = d.run(RequestQueue(_requests(120)))
    _check_all(res, 120)
    assert d.workers[0].error and "injected fault" in d.workers[0].error
    assert d.workers[1].error is None and d.workers[2].error is None


def test_worker_failing_at_startup_is_isolated():
    def bad():
        raise RuntimeError("weight load error: missing tensor")

    d = Dispatcher([bad, lambda: FakeEngine(max_batch=5)])
    res = d.run(RequestQueue(_requests(40)))
    _check_all(res, 40)
    assert "weight load error" in d.workers[0].error


def test_all_workers_failing_reports_every_request():
    d = Dispatcher([lambda: FakeEngine(max_batch=4, fail_after=1), lambda: FakeEngine(max_batch=4, fail_after=3)])
    done = threading.Event()
    holder = {}

    def run():
        holder["res"] = d.run(RequestQueue(_requests(50)))
        done.set()

    threading.Thread(target=run, daemon=True).start()
    assert done.wait(30), "dispatcher hung after every worker failed"
    res = holder["res"]
    assert sorted(res) == list(range(50))
    failed = [r for r in res.values() if r.error and r.id not in BAD]
    assert failed and all("injected fault" in r.error for r in failed)
    for r in res.values():
        if r.error is None:
            assert r.codes == _codes(Request(r.id, None, None, r.id))


def _rank_main(rank, world, port, n, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    sys.path.insert(0, str(ROOT / "index-tts-rs_b200"))
    import torch.distributed as dist
    from itts_gpt.serve import Dispatcher as D, StoreQueue as SQ
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=60))
    try:
        store = dist.distributed_c10d._get_default_store()
        res = D([lambda: FakeEngine(max_batch=3 + rank)]).run(SQ(store, "test/next", _requests(n)))
        dist.barrier()
        q.put((rank, {i: (r.codes, r.error) for i, r in res.items()}))
    finally:
        dist.destroy_process_group()


def test_store_queue_two_ranks():
    """Two processes draw from one queue in the store: every request is served by exactly
    one of them."""
    import socket
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    n = 90
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, n, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(60)
        assert p.exitcode == 0
    by_rank = dict(got)
    assert not set(by_rank[0]) & set(by_rank[1])
    merged = {**by_rank[0], **by_rank[1]}
    assert sorted(merged) == list(range(n))
    assert all((err is not None) == (i in BAD) for i, (codes, err) in merged.items())
    assert all(codes == _codes(Request(i, None, None, i)) for i, (codes, err) in merged.items() if i not in BAD)
    assert by_rank[0] and by_rank[1]
