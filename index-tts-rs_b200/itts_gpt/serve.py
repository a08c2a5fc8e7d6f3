"""Request-level data parallelism: one decode worker per GPU, fed from one queue.

The reference runs every synthesis on a single engine actor that owns the GPU
(crates/core/src/engine/actor.rs:1227-1277): requests wait in its channel and go through
generate_codes_after (crates/core/src/models/sampler.rs:340-392) one at a time.  Here each
GPU has a worker thread that owns a decoder replica and a KV cache with up to `max_batch`
request slots (continuous batching, include/itts_gpt.h itts_batch_*): queued requests
enter free slots between decode chunks, every decode step advances all live requests,
and a request leaves at its own STOP.  No collective is involved; requests are
independent.

Failure isolation (the reference returns worker start-up errors through a bounded
channel and restarts the actor, actor.rs:1200, 1262-1277): a worker whose device call
fails puts its unfinished requests back at the head of the queue and stops; the other
workers serve them.  Requests that no live worker remains to serve are reported with the
error.

Across processes (one process per GPU under torchrun), StoreQueue hands out requests
from a shared counter in the torch.distributed store instead of an in-process queue.
"""
from __future__ import annotations

import threading
import time
from collections import deque
from dataclasses import dataclass, field
from typing import Callable, Sequence

from . import (CodePrompt, Gpt, KvCache, SamplerRng, SamplingParams, ValidationError, batch_admit,
               batch_collect, batch_decode)


@dataclass
class Request:
    """One sentence: generate_codes_after(prompt, params, SamplerRng(seed))."""

    id: int
    prompt: CodePrompt
    params: SamplingParams
    seed: int


@dataclass
class Result:
    id: int
    codes: list[int] = field(default_factory=list)
    rng_state: int = 0
    worker: int = -1
    error: str | None = None


class RequestQueue:
    """FIFO shared by the workers of one process.  `pending` counts requests taken and not
    yet finished, so an idle worker waits while another might still put some back."""

    def __init__(self, requests: Sequence[Request] = ()):
        self._q = deque(requests)
        self._lock = threading.Condition()
        self.pending = 0

    def take(self, k: int) -> list[Request]:
        with self._lock:
            out = [self._q.popleft() for _ in range(min(k, len(self._q)))]
            self.pending += len(out)
            return out

    def done(self, n: int) -> None:
        with self._lock:
            self.pending -= n
            self._lock.notify_all()

    def put_back(self, reqs: Sequence[Request]) -> None:
        with self._lock:
            self._q.extendleft(reversed(list(reqs)))
            self.pending -= len(reqs)
            self._lock.notify_all()

    def drained(self, timeout: float = 0.05) -> bool:
        """True when nothing is queued and nothing is in flight; waits up to `timeout`
        for a change otherwise."""
        with self._lock:
            if not self._q and self.pending == 0:
                return True
            if not self._q:
                self._lock.wait(timeout)
            return not self._q and self.pending == 0

    def __len__(self) -> int:
        with self._lock:
            return len(self._q)


class StoreQueue:
    """The queue over a torch.distributed store, for one process per GPU: every process
    holds the same request list, and take() claims the next indices with the store's
    atomic add.  Requests of a failed worker cannot move to another process; they are
    reported with the error."""

    def __init__(self, store, key: str, requests: Sequence[Request]):
        self.store, self.key, self.requests = store, key, list(requests)
        self.pending = 0
        self._exhausted = False

    def take(self, k: int) -> list[Request]:
        if self._exhausted or k <= 0:
            return []
        hi = int(self.store.add(self.key, k))
        lo = hi - k
        if lo >= len(self.requests):
            self._exhausted = True
            return []
        out = self.requests[lo:min(hi, len(self.requests))]
        self.pending += len(out)
        return out

    def done(self, n: int) -> None:
        self.pending -= n

    def put_back(self, reqs: Sequence[Request]) -> None:
        raise RuntimeError("requests cannot move between processes")

    def drained(self, timeout: float = 0.0) -> bool:
        return self._exhausted and self.pending == 0


class SlotEngine:
    """One device: a decoder replica and a KV cache of max_batch slots, driven through
    the continuous-batching calls of the C ABI."""

    def __init__(self, gpt: Gpt, cache: KvCache, chunk: int = 8):
        self.gpt, self.cache, self.chunk = gpt, cache, chunk
        self.max_batch = cache.max_batch()

    def admit(self, pairs: Sequence[tuple[int, Request]]) -> None:
        batch_admit(self.gpt, self.cache, [s for s, _ in pairs], [r.prompt for _, r in pairs],
                    [r.params for _, r in pairs], [SamplerRng(r.seed) for _, r in pairs])

    def decode(self) -> list[int]:
        finished, _ = batch_decode(self.gpt, self.cache, 1 << 30, self.chunk)
        return finished

    def collect(self, slot: int) -> tuple[list[int], int, int]:
        return batch_collect(self.gpt, self.cache, slot)

    def close(self) -> None:
        self.cache.close()
        self.gpt.close()


class Worker:
    """Serves requests from a queue on one engine until the queue is drained.  With
    keep_engine the engine outlives serve() and the next serve() reuses it (a warm-up run,
    then the real queue); close() frees it."""

    def __init__(self, index: int, make_engine: Callable[[], object], admit_max: int = 64,
                 keep_engine: bool = False):
        self.index, self.make_engine, self.admit_max = index, make_engine, admit_max
        self.keep_engine = keep_engine
        self.engine = None
        self.error: str | None = None
        self.served = 0
        self.busy_s = 0.0

    def close(self) -> None:
        if self.engine is not None and hasattr(self.engine, "close"):
            try:
                self.engine.close()
            except Exception:
                pass
        self.engine = None

    def _admit(self, engine, pairs, live, queue, sink) -> None:
        """Admits pairs; a request the library rejects (a Validation error, checked before
        any device work) is answered with that error alone, the others still enter."""
        try:
            engine.admit(pairs)
            return
        except ValidationError:
            pass
        for pair in pairs:
            try:
                engine.admit([pair])
            except ValidationError as e:
                live.pop(pair[0])
                sink(Result(pair[1].id, worker=self.index, error=f"ValidationError: {e}"))
                queue.done(1)

    def serve(self, queue, sink: Callable[[Result], None]) -> None:
        live: dict[int, Request] = {}
        engine = None
        try:
            if self.error is not None:
                raise RuntimeError(f"worker {self.index} failed earlier: {self.error}")
            engine = self.engine if self.engine is not None else self.make_engine()
            self.engine = engine
            t0 = time.perf_counter()
            while True:
                free = [s for s in range(engine.max_batch) if s not in live]
                if free:
                    reqs = queue.take(min(len(free), self.admit_max))
                    if reqs:
                        pairs = list(zip(free, reqs))
                        live.update(pairs)
                        self._admit(engine, pairs, live, queue, sink)
                if not live:
                    if queue.drained():
                        break
                    continue
                for slot in engine.decode():
                    codes, state, status = engine.collect(slot)
                    req = live.pop(slot)
                    sink(Result(req.id, codes, state, self.index,
                                None if status == 0 else "request outgrew the KV cache"))
                    queue.done(1)
                    self.served += 1
            self.busy_s = time.perf_counter() - t0
        except Exception as e:  # isolate this worker: its requests go back to the queue
            if self.error is None:
                self.error = f"{type(e).__name__}: {e}"
            reqs = list(live.values())
            try:
                queue.put_back(reqs)
            except Exception:
                for r in reqs:
                    sink(Result(r.id, worker=self.index, error=self.error))
                queue.done(len(reqs))
            self.close()  # a failed engine is not reused
        finally:
            if not self.keep_engine:
                self.close()


class Dispatcher:
    """Runs one Worker thread per engine factory over a shared queue and returns every
    request's Result.  make_engines[i]() is called on worker i's thread (each handle
    belongs to the thread that made it)."""

    def __init__(self, make_engines: Sequence[Callable[[], object]], admit_max: int = 64,
                 keep_engines: bool = False):
        self.workers = [Worker(i, f, admit_max, keep_engines) for i, f in enumerate(make_engines)]

    def close(self) -> None:
        for w in self.workers:
            w.close()

    def run(self, queue) -> dict[int, Result]:
        results: dict[int, Result] = {}
        lock = threading.Lock()

        def sink(r: Result) -> None:
            with lock:
                results[r.id] = r

        threads = [threading.Thread(target=w.serve, args=(queue, sink), daemon=True) for w in self.workers]
        for t in threads:
            t.start()
        for t in threads:
            t.join()
        # every worker failed: what is still queued cannot be served
        if isinstance(queue, RequestQueue):
            err = "; ".join(w.error for w in self.workers if w.error) or "no worker left"
            for r in queue.take(len(queue)):
                results[r.id] = Result(r.id, error=err)
            queue.done(0)
        return results


def gpu_engine_factory(weights: dict, device: int, max_batch: int, max_seq: int, chunk: int = 8):
    """A SlotEngine on `device`: a decoder replica from host tensors and its cache."""

    def make():
        gpt = Gpt.from_weights(weights, device=device)
        return SlotEngine(gpt, KvCache(gpt, max_seq=max_seq, max_batch=max_batch), chunk)

    return make
