"""Request bookkeeping and admission control (host side).

Follows reference src/microserve/scheduler.py: FCFS / SJF / LIFO priority,
continuous or static batching, preemption by recomputation, and the
speculative ``tokens_per_step`` reservation (gamma + 1 slots per running
request).  It owns no tensors.  ``Request.rng_step`` is new: the request's
Philox draw-step counter, advanced once per engine iteration it takes part
in.
"""

from __future__ import annotations

import enum
import itertools
from dataclasses import dataclass, field

from .cache import PagedKVCache
from .config import SamplingConfig, SchedulerConfig


class RequestStatus(enum.Enum):
    WAITING = "waiting"
    RUNNING = "running"
    PREEMPTED = "preempted"
    FINISHED = "finished"
    ABORTED = "aborted"


@dataclass
class Request:
    """One generation request (reference scheduler.py:41-115)."""

    request_id: int
    prompt_ids: list[int]
    sampling: SamplingConfig
    arrival_time: float = 0.0

    output_ids: list[int] = field(default_factory=list)
    status: RequestStatus = RequestStatus.WAITING
    num_computed: int = 0

    schedule_time: float | None = None
    first_token_time: float | None = None
    finish_time: float | None = None

    num_preemptions: int = 0
    num_draft_proposed: int = 0
    num_draft_accepted: int = 0
    rng_step: int = 0

    @property
    def all_ids(self) -> list[int]:
        return self.prompt_ids + self.output_ids

    @property
    def num_tokens(self) -> int:
        return len(self.prompt_ids) + len(self.output_ids)

    def tail(self, start: int) -> list[int]:
        """``all_ids[start:]`` without concatenating the whole history."""
        n_prompt = len(self.prompt_ids)
        if start >= n_prompt:
            return self.output_ids[start - n_prompt :]
        return self.prompt_ids[start:] + self.output_ids

    @property
    def num_uncomputed(self) -> int:
        return self.num_tokens - self.num_computed

    @property
    def is_prefill(self) -> bool:
        return self.num_uncomputed > 1

    @property
    def finished(self) -> bool:
        return self.status in (RequestStatus.FINISHED, RequestStatus.ABORTED)

    def should_stop(self) -> bool:
        if len(self.output_ids) >= self.sampling.max_new_tokens:
            return True
        stop = self.sampling.stop_token
        return stop is not None and bool(self.output_ids) and self.output_ids[-1] == stop

    def reset_for_recompute(self) -> None:
        self.num_computed = 0
        self.status = RequestStatus.PREEMPTED
        self.num_preemptions += 1

    def ttft(self) -> float | None:
        if self.first_token_time is None:
            return None
        return self.first_token_time - self.arrival_time

    def tpot(self) -> float | None:
        if self.finish_time is None or self.first_token_time is None:
            return None
        extra = len(self.output_ids) - 1
        if extra <= 0:
            return None
        return (self.finish_time - self.first_token_time) / extra

    def latency(self) -> float | None:
        if self.finish_time is None:
            return None
        return self.finish_time - self.arrival_time


@dataclass
class SchedulerOutput:
    scheduled: list[Request] = field(default_factory=list)
    preempted: list[Request] = field(default_factory=list)

    @property
    def is_empty(self) -> bool:
        return not self.scheduled

    @property
    def num_tokens(self) -> int:
        return sum(r.num_uncomputed for r in self.scheduled)


class Scheduler:
    """Priority queueing, admission control and preemption (reference scheduler.py:134-258)."""

    def __init__(self, cfg: SchedulerConfig, cache: PagedKVCache) -> None:
        self.cfg = cfg
        self.cache = cache
        self.waiting: list[Request] = []
        self.running: list[Request] = []
        self.finished: list[Request] = []
        self._ids = itertools.count()
        self.total_preemptions = 0
        self.tokens_per_step = 1

    def add(self, request: Request) -> Request:
        request.status = RequestStatus.WAITING
        self.waiting.append(request)
        return request

    def next_request_id(self) -> int:
        return next(self._ids)

    @property
    def num_unfinished(self) -> int:
        return len(self.waiting) + len(self.running)

    def priority(self, request: Request) -> tuple[float, int]:
        if self.cfg.policy == "fcfs":
            key = request.arrival_time
        elif self.cfg.policy == "lifo":
            key = -request.arrival_time
        else:
            key = float(len(request.prompt_ids) + request.sampling.max_new_tokens)
        return (key, request.request_id)

    def schedule(self, now: float) -> SchedulerOutput:
        out = SchedulerOutput()
        if self.cfg.batching == "static" and self.running:
            self._ensure_room(self.running, out)
            out.scheduled = list(self.running)
            return out
        self._ensure_room(self.running, out)
        out.scheduled = list(self.running)
        self._admit(out, now)
        return out

    def _need(self, r: Request) -> int:
        return self.cache.blocks_needed(r.request_id, max(self.tokens_per_step, r.num_uncomputed))

    def _ensure_room(self, running: list[Request], out: SchedulerOutput) -> None:
        """Preempt lowest-priority requests until every running one can step."""
        while running:
            needed = sum(self._need(r) for r in running)
            if needed <= self.cache.num_free_blocks or len(running) == 1:
                return
            victim = max(running, key=self.priority)
            running.remove(victim)
            self.cache.free(victim.request_id)
            victim.reset_for_recompute()
            self.waiting.append(victim)
            out.preempted.append(victim)
            self.total_preemptions += 1

    def _admit(self, out: SchedulerOutput, now: float) -> None:
        """Admit waiting requests while the token and block budgets allow,
        debiting blocks locally because nothing is allocated until the batch
        is built."""
        token_budget = self.cfg.max_batched_tokens - out.num_tokens
        reserve = int(self.cache.allocator.num_blocks * self.cfg.watermark)
        free_blocks = self.cache.num_free_blocks - sum(self._need(r) for r in out.scheduled)
        for request in sorted(self.waiting, key=self.priority):
            if len(self.running) >= self.cfg.max_batch_size:
                break
            need = request.num_uncomputed
            if need > token_budget and out.scheduled:
                continue
            blocks = self.cache.blocks_needed(request.request_id, max(need, self.tokens_per_step))
            headroom = free_blocks - (reserve if out.scheduled else 0)
            if blocks > headroom:
                continue
            self.waiting.remove(request)
            request.status = RequestStatus.RUNNING
            if request.schedule_time is None:
                request.schedule_time = now
            self.running.append(request)
            out.scheduled.append(request)
            token_budget -= need
            free_blocks -= blocks

    def finish(self, request: Request, now: float) -> None:
        request.status = RequestStatus.FINISHED
        request.finish_time = now
        if request in self.running:
            self.running.remove(request)
        self.cache.free(request.request_id)
        self.finished.append(request)
