"""Continuous batching over paged block tables: every running request advances in ONE decode step.

The reference's ``ContinuousBatchingScheduler`` (``microgen/scheduler/scheduler.py:17-255``) admits
requests by priority, prefills them, and then decodes each running request on its own at batch 1
(``scheduler.py:199-226``: one ``backend.decode`` + ``backend.sample`` per request and step). Here the
running set decodes as one batch through the B200 backend: each request owns a ``BlockTable`` in the
backend's ``PagedKVCacheAllocator``; a step hands the tables of all running requests (ragged contexts)
to one graph-replayed decode, and the attention kernel reads blocks that every table shares (a prompt
prefix prefilled once, or reused from the backend's prefix cache) once per batch.

Kept from the reference: ``add_request`` / ``step`` / ``run_until_complete``, admission of pending
requests by priority (higher first, then arrival) up to ``max_batch_size`` running, completion on EOS or
``max_new_tokens`` (``batch.py:101-129``), per-request sampling parameters, and the profiling counters
of ``get_profile_breakdown``. Requests are duck-typed: the reference's ``Request`` objects work, and so
do this module's ``Request``. Added: admission also waits for KV blocks — a request is admitted only
when the blocks of its prompt plus ``max_new_tokens`` fit beside those reserved by the running requests,
so a decode step never runs out of blocks.
"""

from __future__ import annotations

import heapq
import itertools
import threading
import time
from dataclasses import dataclass, field
from enum import Enum
from typing import Dict, List, Optional

import numpy as np
import torch

from .backends.b200 import PagedKVCache
from .runtime.paged_kv import BLOCK_SIZE


class RequestStatus(str, Enum):
    """Request lifecycle (the values of ``microgen/scheduler/queue.py:10-17``)."""
    PENDING = "pending"
    RUNNING = "running"
    COMPLETED = "completed"
    CANCELLED = "cancelled"
    FAILED = "failed"


@dataclass
class Request:
    """The request fields the scheduler reads and writes (those of ``queue.py:20-40``)."""
    request_id: str
    prompt: str
    prompt_ids: List[int]
    max_new_tokens: int = 128
    temperature: float = 1.0
    top_k: int = 0
    top_p: float = 0.0
    priority: int = 0
    status: RequestStatus = RequestStatus.PENDING
    arrival_time: float = field(default_factory=time.perf_counter)
    start_time: Optional[float] = None
    first_token_time: Optional[float] = None
    finish_time: Optional[float] = None
    generated_token_ids: List[int] = field(default_factory=list)
    generated_text: str = ""
    error_message: Optional[str] = None

    @property
    def num_prompt_tokens(self) -> int:
        return len(self.prompt_ids)

    @property
    def num_generated_tokens(self) -> int:
        return len(self.generated_token_ids)

    @property
    def is_finished(self) -> bool:
        return self.status in (RequestStatus.COMPLETED, RequestStatus.CANCELLED, RequestStatus.FAILED)


def _status(req, name: str):
    """The status value ``name`` in the enum the request itself uses (the reference's or this module's)."""
    return type(req.status)[name] if isinstance(req.status, Enum) else getattr(RequestStatus, name)


class PriorityQueue:
    """Pending requests ordered by priority (higher first), then arrival time, then submission order; a
    heap instead of the reference's lazily re-sorted id list (``queue.py:96-192``), same order."""

    def __init__(self) -> None:
        self._lock = threading.Lock()
        self._heap: list = []
        self._seq = itertools.count()

    def enqueue(self, req) -> None:
        with self._lock:
            heapq.heappush(self._heap, (-req.priority, req.arrival_time, next(self._seq), req))

    def pop_batch(self, n: int, admit=None) -> list:
        """Up to ``n`` pending requests in order; ``admit(req)`` False stops at that request (it stays
        queued, so a large request is not overtaken). Cancelled requests are dropped."""
        out = []
        with self._lock:
            while self._heap and len(out) < n:
                req = self._heap[0][3]
                if req.status != _status(req, "PENDING"):
                    heapq.heappop(self._heap)
                    continue
                if admit is not None and not admit(req):
                    break
                heapq.heappop(self._heap)
                req.status = _status(req, "RUNNING")
                req.start_time = time.perf_counter()
                out.append(req)
        return out

    def is_empty(self) -> bool:
        with self._lock:
            return not any(e[3].status == _status(e[3], "PENDING") for e in self._heap)

    def size(self) -> int:
        with self._lock:
            return sum(e[3].status == _status(e[3], "PENDING") for e in self._heap)


def _blocks(n_tokens: int) -> int:
    return (n_tokens + BLOCK_SIZE - 1) // BLOCK_SIZE


def _greedy(req) -> bool:
    t, k, p = req.temperature, req.top_k, req.top_p
    return t <= 0.0 or (k == 0 and p == 0.0 and t == 1.0)


class BatchedScheduler:
    """Continuous batching on a ``B200QuantizedBackend`` / ``B200TensorParallelBackend`` (loaded).

    ``step()`` admits pending requests while ``max_batch_size`` and the KV blocks allow, prefills them
    (prompts of equal length together, so a shared prompt prefix is computed once), samples their first
    token, then runs one batched decode step for every running request and samples each request's next
    token with its own parameters. Returns the requests that finished in this step; their blocks go back
    to the allocator."""

    def __init__(self, backend, max_batch_size: int = 8, eos_token_id: Optional[int] = None,
                 pad_token_id: int = 0) -> None:
        eng = backend._need_model()
        if max_batch_size > eng.max_batch:
            raise ValueError(f"max_batch_size {max_batch_size} > the backend's max_batch {eng.max_batch}")
        self.backend = backend
        self.max_batch_size = max_batch_size
        self.eos_token_id = eos_token_id
        self.pad_token_id = pad_token_id
        self.request_queue = PriorityQueue()
        self.running_requests: list = []
        self._tables: Dict[str, object] = {}
        self._reserved: Dict[str, int] = {}
        self._batch = PagedKVCache(backend.allocator)
        self._shared_key = None
        self._n_shared = 0
        self._admitting = 0
        self.decode_batch_sizes: List[int] = []
        self.reset_profiling()

    # ---- the reference's surface ------------------------------------------------------------------
    def reset_profiling(self) -> None:
        self.profiling_stats = {"queue_pop_ms": 0.0, "kv_manage_ms": 0.0, "backend_cuda_ms": 0.0,
                                "python_loop_ms": 0.0, "total_steps": 0.0}

    def get_profile_breakdown(self) -> Dict[str, float]:
        s = self.profiling_stats
        overhead = s["queue_pop_ms"] + s["kv_manage_ms"] + s["python_loop_ms"]
        total = overhead + s["backend_cuda_ms"]
        return {"queue_pop_ms": s["queue_pop_ms"], "kv_manage_ms": s["kv_manage_ms"],
                "backend_cuda_ms": s["backend_cuda_ms"], "python_loop_ms": s["python_loop_ms"],
                "total_scheduler_ms": total, "scheduler_overhead_ms": overhead,
                "scheduler_overhead_ratio": overhead / total if total > 0 else 0.0,
                "total_steps": s["total_steps"]}

    def add_request(self, request) -> None:
        if request.num_prompt_tokens < 1:
            raise ValueError("a request needs at least one prompt token")
        need = _blocks(request.num_prompt_tokens + request.max_new_tokens)
        if need > self.backend.engine.max_blocks or need > self.backend.allocator.num_blocks:
            raise ValueError(f"request {request.request_id}: {need} KV blocks exceed the backend's capacity")
        self.request_queue.enqueue(request)

    def step(self) -> list:
        self.profiling_stats["total_steps"] += 1.0
        done = []
        room = self.max_batch_size - len(self.running_requests)
        if room > 0 and not self.request_queue.is_empty():
            t0 = time.perf_counter()
            self._admitting = 0
            new = self.request_queue.pop_batch(room, admit=self._fits)
            self.profiling_stats["queue_pop_ms"] += (time.perf_counter() - t0) * 1e3
            if new:
                done += self._prefill(new)
        if self.running_requests:
            done += self._decode(self.running_requests)
        t0 = time.perf_counter()
        self.running_requests = [r for r in self.running_requests if r.status == _status(r, "RUNNING")]
        self.profiling_stats["python_loop_ms"] += (time.perf_counter() - t0) * 1e3
        return done

    def run_until_complete(self) -> list:
        out = []
        while not self.request_queue.is_empty() or self.running_requests:
            out += self.step()
        return out

    # ---- internals -------------------------------------------------------------------------------
    def _fits(self, req) -> bool:
        """KV admission: the request's blocks (prompt + max_new_tokens) must fit in the allocator's free
        blocks minus those the running requests may still append and those of requests admitted in this
        step. A prompt prefix shared with other requests is counted as private (conservative). With
        nothing running and nothing admitted the request is let through (blocks held elsewhere, e.g. by
        the prefix cache, then surface as the allocator's MemoryError instead of a queue that never
        drains)."""
        need = _blocks(req.num_prompt_tokens + req.max_new_tokens)
        if not self.running_requests and not self._admitting:
            self._admitting += need
            return True
        free = self.backend.allocator.get_num_free_blocks()
        future = sum(max(0, self._reserved[rid] - t.num_blocks()) for rid, t in self._tables.items())
        if need > free - future - self._admitting:
            return False
        self._admitting += need
        return True

    def _sample_rows(self, reqs, logits: torch.Tensor) -> List[int]:
        be = self.backend
        if all(_greedy(r) for r in reqs):
            return be.sample(logits)[:, 0].tolist()
        greedy = None
        out = []
        for i, r in enumerate(reqs):
            if _greedy(r):
                if greedy is None:
                    greedy = be.sample(logits)[:, 0].tolist()
                out.append(greedy[i])
            else:
                out.append(int(be.sample(logits[i:i + 1].clone(), temperature=r.temperature, top_k=r.top_k,
                                         top_p=r.top_p).reshape(-1)[0]))
        return out

    def _finish(self, reqs, tokens: List[int]) -> list:
        """Append the sampled tokens; EOS or max_new_tokens completes a request and frees its blocks
        (``batch.py:101-129``)."""
        now = time.perf_counter()
        done = []
        for r, tok in zip(reqs, tokens):
            if r.is_finished:
                continue
            if r.first_token_time is None:
                r.first_token_time = now
            r.generated_token_ids.append(int(tok))
            if (self.eos_token_id is not None and tok == self.eos_token_id) or \
                    r.num_generated_tokens >= r.max_new_tokens:
                r.status = _status(r, "COMPLETED")
                r.finish_time = now
                done.append(r)
        t0 = time.perf_counter()
        for r in done:
            self._release(r)
        self.profiling_stats["kv_manage_ms"] += (time.perf_counter() - t0) * 1e3
        return done

    def _release(self, r) -> None:
        t = self._tables.pop(r.request_id, None)
        if t is not None:
            self.backend.allocator.free_sequence(t)
        self._reserved.pop(r.request_id, None)

    def _prefill(self, new) -> list:
        done = []
        groups: Dict[int, list] = {}
        for r in new:
            groups.setdefault(r.num_prompt_tokens, []).append(r)
        for reqs in groups.values():
            t0 = time.perf_counter()
            ids = torch.tensor([list(r.prompt_ids) for r in reqs], dtype=torch.long)
            logits, cache = self.backend.prefill(ids)
            toks = self._sample_rows(reqs, logits)
            self.profiling_stats["backend_cuda_ms"] += (time.perf_counter() - t0) * 1e3
            t0 = time.perf_counter()
            for r, tab in zip(reqs, cache.tables):
                self._tables[r.request_id] = tab
                self._reserved[r.request_id] = _blocks(r.num_prompt_tokens + r.max_new_tokens)
            if cache.prefix is not None:  # the requests' tables hold their own references to its blocks
                self.backend.allocator.free_sequence(cache.prefix)
                cache.prefix = None
            self.profiling_stats["kv_manage_ms"] += (time.perf_counter() - t0) * 1e3
            finished = self._finish(reqs, toks)
            done += finished
            self.running_requests += [r for r in reqs if r not in finished]
        return done

    def _shared_blocks(self, reqs, tables) -> int:
        """Leading blocks every table holds by id (a shared prompt prefix): the attention kernel reads
        them once for the whole batch. Fixed while the batch keeps its members, so computed on change."""
        key = tuple(r.request_id for r in reqs)
        if key != self._shared_key:
            n = 0
            if len(tables) > 1:
                width = min(t.num_blocks() for t in tables) - 1  # the newest block of each stays private
                if width > 0:
                    ids = np.array([[b.block_id for b in t.physical_blocks[:width]] for t in tables])
                    same = (ids == ids[0]).all(0)
                    n = int(width if same.all() else np.argmin(same))
            self._shared_key, self._n_shared = key, n
        return self._n_shared

    def _decode(self, reqs) -> list:
        t0 = time.perf_counter()
        tables = [self._tables[r.request_id] for r in reqs]
        self._batch.tables = tables
        self._batch.n_shared_blocks = self._shared_blocks(reqs, tables)
        toks = torch.tensor([[r.generated_token_ids[-1]] for r in reqs], dtype=torch.long)
        self.profiling_stats["python_loop_ms"] += (time.perf_counter() - t0) * 1e3
        t0 = time.perf_counter()
        logits, _ = self.backend.decode(toks, cache=self._batch)
        nxt = self._sample_rows(reqs, logits)
        self.profiling_stats["backend_cuda_ms"] += (time.perf_counter() - t0) * 1e3
        self.decode_batch_sizes.append(len(reqs))
        return self._finish(reqs, nxt)
