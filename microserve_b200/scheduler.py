"""Which requests take part in the next engine iteration (host side).

The policy is MicroServe's (reference src/microserve/scheduler.py): FCFS,
LIFO or shortest-job-first priority with the request id as tie-break,
continuous or static batching, admission under a token budget, a batch-size
cap and a block watermark, preemption by recomputation of the
lowest-priority running request while the running set's next step does not
fit, and the speculative reservation of ``tokens_per_step`` (gamma + 1)
slots per request.  It decides exactly what the reference decides, so token
streams and step counts match it.

How it is organised here:

* ``waiting`` stays ordered by priority (each request is inserted at its
  place), so admission is one ordered scan instead of a sort per step;
* the running set's block demand is one batched computation
  (``PagedKVCache.blocks_needed_each``); a request's demand depends only on
  its own table, so preemption takes victims in descending priority and
  subtracts each victim's demand instead of re-summing the set per victim;
* a request's stop condition is an explicit ``finish_reason`` ("length" or
  "stop"), and ``Request.extend_until_stop`` appends a step's tokens up to
  it in one slice;
* with ``SchedulerConfig.prefill_chunk`` (chunked prefill, not in the
  reference) a prefilling request is charged only the chunk it processes
  next, for the token budget and for its blocks.

``Request.rng_step`` (not in the reference) counts the engine iterations a
request took part in; it is the counter of the request's Philox stream.
"""

from __future__ import annotations

import bisect
import enum
from dataclasses import dataclass, field

import numpy as np

from .cache import PagedKVCache
from .config import SamplingConfig, SchedulerConfig


class RequestStatus(enum.Enum):
    WAITING = "waiting"
    RUNNING = "running"
    PREEMPTED = "preempted"
    FINISHED = "finished"
    ABORTED = "aborted"


@dataclass(eq=False)
class Request:
    """One generation request (the reference's ``Request`` fields, scheduler.py:41-115).

    ``num_computed`` counts the leading tokens whose K/V is in the cache;
    the timing fields are engine-clock seconds.  Requests compare by
    identity.
    """

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

    # -- tokens ------------------------------------------------------------
    @property
    def all_ids(self) -> list[int]:
        return [*self.prompt_ids, *self.output_ids]

    @property
    def num_tokens(self) -> int:
        return len(self.prompt_ids) + len(self.output_ids)

    def tail(self, start: int) -> list[int]:
        """``all_ids[start:]``, built from the part of the history it needs."""
        past_prompt = start - len(self.prompt_ids)
        if past_prompt >= 0:
            return self.output_ids[past_prompt:]
        return [*self.prompt_ids[start:], *self.output_ids]

    @property
    def num_uncomputed(self) -> int:
        return self.num_tokens - self.num_computed

    @property
    def is_prefill(self) -> bool:
        """More than one token to process in the next pass."""
        return self.num_uncomputed > 1

    # -- stopping ----------------------------------------------------------
    def finish_reason(self) -> str | None:
        """"length" once the budget is spent, "stop" after the stop token, else None."""
        out = self.output_ids
        if len(out) >= self.sampling.max_new_tokens:
            return "length"
        stop = self.sampling.stop_token
        if stop is not None and out and out[-1] == stop:
            return "stop"
        return None

    def should_stop(self) -> bool:
        return self.finish_reason() is not None

    def extend_until_stop(self, tokens: list[int]) -> int:
        """Append ``tokens`` up to the stop condition; returns how many were
        taken.  Equal to appending one at a time while ``should_stop()`` is
        false: the budget caps the count and the first stop token is the
        last one taken."""
        if self.should_stop():
            return 0
        take = tokens[: self.sampling.max_new_tokens - len(self.output_ids)]
        stop = self.sampling.stop_token
        if stop is not None and stop in take:
            take = take[: take.index(stop) + 1]
        self.output_ids.extend(take)
        return len(take)

    @property
    def finished(self) -> bool:
        return self.status in (RequestStatus.FINISHED, RequestStatus.ABORTED)

    def reset_for_recompute(self) -> None:
        """Preempted: nothing is cached any more; generated tokens are kept
        and will be prefilled again with the prompt."""
        self.num_computed = 0
        self.status = RequestStatus.PREEMPTED
        self.num_preemptions += 1

    # -- latency metrics -----------------------------------------------------
    def ttft(self) -> float | None:
        t = self.first_token_time
        return None if t is None else t - self.arrival_time

    def tpot(self) -> float | None:
        """Mean time per output token after the first (None below two tokens)."""
        t0, t1, n = self.first_token_time, self.finish_time, len(self.output_ids)
        if t0 is None or t1 is None or n < 2:
            return None
        return (t1 - t0) / (n - 1)

    def latency(self) -> float | None:
        t = self.finish_time
        return None if t is None else t - self.arrival_time


@dataclass
class SchedulerOutput:
    """The plan of one engine iteration: who runs, who was evicted for it."""

    scheduled: list[Request] = field(default_factory=list)
    preempted: list[Request] = field(default_factory=list)

    @property
    def is_empty(self) -> bool:
        return len(self.scheduled) == 0

    @property
    def num_tokens(self) -> int:
        return sum(r.num_uncomputed for r in self.scheduled)


class Scheduler:
    """Priority queue, admission control and preemption over one paged cache."""

    def __init__(self, cfg: SchedulerConfig, cache: PagedKVCache) -> None:
        self.cfg = cfg
        self.cache = cache
        self.waiting: list[Request] = []  # ordered by ``priority``
        self.running: list[Request] = []
        self.finished: list[Request] = []
        self.total_preemptions = 0
        self.tokens_per_step = 1
        self._issued_ids = 0

    # -- queue ----------------------------------------------------------------
    def priority(self, request: Request) -> tuple[float, int]:
        """Sort key, smallest first; the id breaks ties."""
        policy = self.cfg.policy
        if policy == "fcfs":
            key = request.arrival_time
        elif policy == "lifo":
            key = -request.arrival_time
        else:  # shortest job first: prompt plus output budget
            key = float(len(request.prompt_ids) + request.sampling.max_new_tokens)
        return key, request.request_id

    def _enqueue(self, request: Request) -> None:
        bisect.insort(self.waiting, request, key=self.priority)

    def add(self, request: Request) -> Request:
        request.status = RequestStatus.WAITING
        self._enqueue(request)
        return request

    def next_request_id(self) -> int:
        rid = self._issued_ids
        self._issued_ids += 1
        return rid

    @property
    def num_unfinished(self) -> int:
        return len(self.waiting) + len(self.running)

    # -- one iteration's plan -------------------------------------------------------
    def step_len(self, request: Request) -> int:
        """Tokens a request processes in its next pass: all its uncomputed
        ones, or at most ``prefill_chunk`` of them with chunked prefill."""
        n = request.num_uncomputed
        chunk = self.cfg.prefill_chunk
        return n if chunk is None else min(n, chunk)

    def _step_tokens(self, request: Request) -> int:
        """Slots a request needs for its next step (gamma + 1 when speculating)."""
        return max(self.tokens_per_step, self.step_len(request))

    def schedule(self, now: float) -> SchedulerOutput:
        plan = SchedulerOutput()
        # static batching admits only when the previous batch has drained
        admit = not (self.cfg.batching == "static" and self.running)
        demand = self._make_room(plan)
        plan.scheduled = list(self.running)
        if admit:
            self._admit(plan, now, demand)
        return plan

    def _make_room(self, plan: SchedulerOutput) -> int:
        """Preempt until the running set's next step fits the free blocks (a
        lone request is never preempted); returns the survivors' block demand."""
        running = self.running
        if not running:
            return 0
        need = self.cache.blocks_needed_each([r.request_id for r in running],
                                             [self._step_tokens(r) for r in running])
        total = int(need.sum())
        free = self.cache.num_free_blocks
        if total <= free or len(running) == 1:
            return total
        evicted = np.zeros(len(running), dtype=bool)
        left = len(running)
        for i in sorted(range(len(running)), key=lambda j: self.priority(running[j]), reverse=True):
            if total <= free or left == 1:
                break
            victim = running[i]
            self.cache.free(victim.request_id)
            free = self.cache.num_free_blocks
            total -= int(need[i])
            evicted[i] = True
            left -= 1
            victim.reset_for_recompute()
            self._enqueue(victim)
            plan.preempted.append(victim)
            self.total_preemptions += 1
        self.running = [r for r, gone in zip(running, evicted, strict=True) if not gone]
        return total

    def _admit(self, plan: SchedulerOutput, now: float, demand: int) -> None:
        """Admit waiting requests in priority order under the token budget,
        the batch cap and the free blocks (minus the watermark reserve once
        something is scheduled).  Blocks are debited locally: nothing is
        allocated until the batch is built."""
        tokens_left = self.cfg.max_batched_tokens - sum(self.step_len(r) for r in plan.scheduled)
        blocks_left = self.cache.num_free_blocks - demand
        reserve = int(self.cache.allocator.num_blocks * self.cfg.watermark)
        admitted: list[Request] = []
        for request in self.waiting:
            if len(self.running) >= self.cfg.max_batch_size:
                break
            n = self.step_len(request)
            busy = bool(plan.scheduled)
            if busy and n > tokens_left:
                continue
            blocks = self.cache.blocks_needed(request.request_id, max(n, self.tokens_per_step))
            if blocks > blocks_left - (reserve if busy else 0):
                continue
            admitted.append(request)
            request.status = RequestStatus.RUNNING
            if request.schedule_time is None:
                request.schedule_time = now
            self.running.append(request)
            plan.scheduled.append(request)
            tokens_left -= n
            blocks_left -= blocks
        if admitted:
            taken = {id(r) for r in admitted}
            self.waiting = [r for r in self.waiting if id(r) not in taken]

    def finish(self, request: Request, now: float) -> None:
        request.status = RequestStatus.FINISHED
        request.finish_time = now
        self.running = [r for r in self.running if r is not request]
        self.cache.free(request.request_id)
        self.finished.append(request)
