"""The serving loop around the device round: ``LLMEngine`` (host side).

Public surface: MicroServe's ``LLMEngine`` (reference src/microserve/engine.py:
``add_request`` / ``step`` / ``run`` / ``generate`` / ``reset``, with
``EngineStats`` and ``RequestOutput``), so callers switch without changes.
The behaviour that decides token streams is the reference's:

* an iteration is one speculative round for every scheduled request when
  none of them is prefilling and the cache can take gamma + 1 more tokens
  for each (engine.py:167-174), otherwise one ordinary paged pass that
  samples one token per request (engine.py:204-262);
* a request's generated tokens are appended up to its budget or stop
  token, and a finished request releases its blocks in both caches;
* each request's random stream is keyed by ``sampling.seed`` or, when that
  is unset, ``config.seed + request_id`` (engine.py:144-147).

The iteration itself is organised around the device: ``_ordinary_pass``
packs a pass's metadata and sampling parameters into two pinned uploads,
runs one forward that computes logits only for each request's last row,
draws on the device, and reads the tokens back in one copy; the speculative
round is ``SpeculativeDecoder.step`` (three uploads, one read-back).
``_commit`` then applies the stop rules to each request's tokens in one
slice (``Request.extend_until_stop``).
"""

from __future__ import annotations

import time
from collections.abc import Callable, Sequence
from dataclasses import dataclass, field
from statistics import fmean
from typing import Any

import numpy as np
import torch

from . import _lib
from .batching import HostStaging, batch_from_host, host_batch_arrays, pack_int32
from .cache import OutOfCacheMemory, PagedKVCache
from .config import CacheConfig, EngineConfig, SamplingConfig
from .model import PagedBatch, Transformer
from .sampling import make_params, validate
from .scheduler import Request, RequestStatus, Scheduler, SchedulerOutput


@dataclass
class RequestOutput:
    """A finished request as the caller receives it.  ``finish_reason`` ("length"
    or "stop") is an addition; the other fields are the reference's."""

    request_id: int
    prompt_ids: list[int]
    output_ids: list[int]
    text: str | None = None
    ttft: float | None = None
    tpot: float | None = None
    latency: float | None = None
    num_preemptions: int = 0
    acceptance_rate: float | None = None
    finish_reason: str | None = None


@dataclass
class EngineStats:
    """Lifetime counters of an engine (the reference's fields, plus the
    number of speculative rounds run)."""

    num_steps: int = 0
    num_prefill_tokens: int = 0
    num_decode_tokens: int = 0
    num_generated_tokens: int = 0
    num_preemptions: int = 0
    num_draft_proposed: int = 0
    num_draft_accepted: int = 0
    num_spec_rounds: int = 0
    utilization_samples: list[float] = field(default_factory=list)
    batch_size_samples: list[int] = field(default_factory=list)

    def record_step(self, batch_size: int, utilization: float) -> None:
        self.num_steps += 1
        self.batch_size_samples.append(batch_size)
        self.utilization_samples.append(utilization)

    @property
    def mean_utilization(self) -> float:
        return fmean(self.utilization_samples) if self.utilization_samples else 0.0

    @property
    def peak_utilization(self) -> float:
        return max(self.utilization_samples, default=0.0)

    @property
    def mean_batch_size(self) -> float:
        return fmean(self.batch_size_samples) if self.batch_size_samples else 0.0

    @property
    def acceptance_rate(self) -> float | None:
        if self.num_draft_proposed == 0:
            return None
        return self.num_draft_accepted / self.num_draft_proposed


class LLMEngine:
    """Continuous batching over a paged KV cache on one CUDA device, with
    optional speculative decoding (``config.speculative`` plus a draft model)."""

    def __init__(
        self,
        model: Transformer,
        config: EngineConfig | None = None,
        tokenizer: Any | None = None,
        draft_model: Transformer | None = None,
        clock: Callable[[], float] = time.perf_counter,
    ) -> None:
        self.config = config if config is not None else EngineConfig(model=model.cfg)
        self.model = model.eval()
        self.tokenizer = tokenizer
        self.clock = clock
        self.device = _lib.require_cuda(self.config.device)
        # the device cache holds K/V in the model's dtype
        c = self.config.cache
        self._cache_cfg = CacheConfig(c.block_size, c.num_blocks, model.cfg.dtype)
        self.cache = PagedKVCache(model.cfg, self._cache_cfg, self.device)
        self.stats = EngineStats()
        self._generators: dict[int, torch.Generator] = {}
        self._meta_upload = HostStaging(self.device)
        self._param_upload = HostStaging(self.device)
        self._q_start = np.zeros(1, dtype=np.int32)  # the last built pass's row offsets
        self.lookahead = True  # let the decoder draft the next round ahead (same streams)
        self._no_rows = torch.zeros(0, dtype=torch.int32, device=self.device)  # no logits
        self.spec = None
        if draft_model is not None and self.config.speculative.enabled:
            from .speculative import SpeculativeDecoder

            self.spec = SpeculativeDecoder(target=self.model, draft=draft_model,
                                           cache_cfg=self._cache_cfg,
                                           gamma=self.config.speculative.gamma,
                                           device=self.device)
        self.scheduler = self._new_scheduler()

    def _new_scheduler(self) -> Scheduler:
        sched = Scheduler(self.config.scheduler, self.cache)
        if self.spec is not None:
            sched.tokens_per_step = self.config.speculative.gamma + 1  # reserve a round's slots
        return sched

    # -- requests --------------------------------------------------------------------
    def add_request(
        self,
        prompt_ids: Sequence[int] | str,
        sampling: SamplingConfig | None = None,
        request_id: int | None = None,
        arrival_time: float | None = None,
    ) -> Request:
        """Queue a request given token ids (or text, with a tokenizer).

        Raises ``ValueError`` for an empty prompt, text without a tokenizer,
        invalid sampling settings, a prompt plus budget beyond
        ``max_seq_len``, or a request the whole pool could never hold."""
        if isinstance(prompt_ids, str):
            if self.tokenizer is None:
                raise ValueError("text prompts need a tokenizer")
            prompt_ids = self.tokenizer.encode(prompt_ids)
        ids = [int(t) for t in prompt_ids]
        if len(ids) == 0:
            raise ValueError("prompt must contain at least one token")
        sampling = sampling if sampling is not None else SamplingConfig()
        validate(sampling)
        # the id is taken before the length checks, so a refused request
        # consumes one as in the reference (later seeds depend on it)
        rid = request_id if request_id is not None else self.scheduler.next_request_id()
        longest = len(ids) + sampling.max_new_tokens
        if longest > self.model.cfg.max_seq_len:
            raise ValueError("prompt plus max_new_tokens exceeds max_seq_len")
        if -(-longest // self.cache.block_size) > self.cache.allocator.num_blocks:
            raise ValueError(
                f"request needs up to {longest} tokens of KV cache but the pool holds only "
                f"{self.config.cache.num_slots}; it could never be served")
        seed = sampling.seed if sampling.seed is not None else self.config.seed + rid
        self._generators[rid] = torch.Generator().manual_seed(seed)
        arrived = arrival_time if arrival_time is not None else self.clock()
        return self.scheduler.add(Request(rid, ids, sampling, arrival_time=arrived))

    @property
    def has_unfinished(self) -> bool:
        return self.scheduler.num_unfinished > 0

    # -- one iteration -----------------------------------------------------------------
    def step(self) -> list[RequestOutput]:
        """Schedule, run one pass or round on the device, retire finished
        requests; returns their outputs."""
        plan = self.scheduler.schedule(self.clock())
        self.stats.num_preemptions = self.scheduler.total_preemptions
        if plan.is_empty:
            return []
        if self.spec is not None:
            for victim in plan.preempted:
                self.spec.free(victim.request_id)
        batch = plan.scheduled
        if self._round_fits(plan):
            assert self.spec is not None
            # drafting the next round ahead pays off only if the batch stays
            # the same, which requests still waiting for admission make unlikely
            self.spec.lookahead = self.lookahead and not self.scheduler.waiting
            tokens = self.spec.step(batch, self.cache, self._generators)
            self.stats.num_spec_rounds += 1
            self.stats.num_draft_proposed = self.spec.num_proposed
            self.stats.num_draft_accepted = self.spec.num_accepted
        else:
            tokens = self._ordinary_pass(batch)
        return self._commit(batch, tokens, self.clock())

    def _round_fits(self, plan: SchedulerOutput) -> bool:
        """A speculative round needs every request decoding (one uncomputed
        token) and room for gamma + 1 tokens per request."""
        if self.spec is None:
            return False
        width = self.config.speculative.gamma + 1
        return all(not r.is_prefill and self.cache.can_append(r.request_id, width)
                   for r in plan.scheduled)

    def _commit(self, batch: list[Request], tokens: list[list[int]], now: float
                ) -> list[RequestOutput]:
        done: list[RequestOutput] = []
        for request, new in zip(batch, tokens, strict=True):
            taken = request.extend_until_stop(new)
            if taken:
                self.stats.num_generated_tokens += taken
                if request.first_token_time is None:
                    request.first_token_time = now
            if request.should_stop():
                self.scheduler.finish(request, now)
                if self.spec is not None:
                    self.spec.free(request.request_id)
                done.append(self.make_output(request))
        self.stats.record_step(len(batch), self.cache.utilization)
        return done

    def _ordinary_pass(self, batch: list[Request]) -> list[list[int]]:
        """One paged forward over every request's uncomputed tokens (or the
        next chunk of them), then one draw from the last row of each request
        whose tokens are now all computed (reference engine.py:204-220).  A
        request whose prefill continues in a later chunk draws nothing and
        keeps its round counter, so its stream equals the unchunked one."""
        meta = self.build_batch(batch)
        done = [i for i, r in enumerate(batch) if r.num_uncomputed == 0]
        out: list[list[int]] = [[] for _ in batch]
        if not done:
            self.model.forward_paged(meta, self.cache, logit_rows=self._no_rows)  # K/V only
            return out
        fin = [batch[i] for i in done]
        last_rows = (self._q_start[1:] - 1).astype(np.int32)[done]
        seeds = [self._generators[r.request_id].initial_seed() for r in fin]
        params = make_params([r.sampling for r in fin], seeds, [r.rng_step for r in fin])
        blob, spans = pack_int32([params.view(np.int32), last_rows])
        dev = self._param_upload.upload(blob)
        (p_off, _), (r_off, r_len) = spans
        rows = dev[r_off : r_off + r_len]
        logits = self.model.forward_paged(meta, self.cache, logit_rows=rows)
        V = self.model.cfg.vocab_size
        drawn = torch.empty(len(fin), dtype=torch.int32, device=self.device)
        _lib.call("ms_sample", logits.data_ptr(), V, len(fin), V, dev[p_off:].data_ptr(), None,
                  _lib.LANE_SAMPLE, drawn.data_ptr(), None, None, None, None,
                  _lib.stream_ptr(self.device))
        for r in fin:
            r.rng_step += 1
        for i, t in zip(done, drawn.cpu().tolist(), strict=True):
            out[i] = [t]
        return out

    def build_batch(self, batch: list[Request]) -> PagedBatch:
        """Reserve cache slots for every request's uncomputed tokens and upload
        the flattened pass (reference engine.py:222-262).  Raises
        ``RuntimeError`` for a request with nothing to do and
        ``OutOfCacheMemory`` when a request's tokens do not fit."""
        ids = [r.request_id for r in batch]
        todo = [self.scheduler.step_len(r) for r in batch]
        for r, n in zip(batch, todo, strict=True):
            if n <= 0:
                raise RuntimeError(f"request {r.request_id} has nothing to do")
            if not self.cache.can_append(r.request_id, n):
                raise OutOfCacheMemory(
                    f"request {r.request_id} needs {self.cache.blocks_needed(r.request_id, n)} "
                    f"blocks, {self.cache.num_free_blocks} free; raise cache.num_blocks")
        starts = [r.num_computed for r in batch]
        try:
            parts, width, max_q, n_tokens = host_batch_arrays(
                self.cache, ids, [r.tail(s)[:n] for r, s, n in zip(batch, starts, todo,
                                                                   strict=True)], starts)
        except OutOfCacheMemory as e:
            raise OutOfCacheMemory(f"{e}; raise cache.num_blocks") from e
        for r, n in zip(batch, todo, strict=True):
            if n > 1:
                self.stats.num_prefill_tokens += n
            else:
                self.stats.num_decode_tokens += n
            r.num_computed += n
            r.status = RequestStatus.RUNNING
        self._q_start = parts[3]
        blob, spans = pack_int32(parts)
        return batch_from_host(self._meta_upload.upload(blob), spans, len(ids), width, max_q,
                               n_tokens, int(parts[4].max()))

    # -- results -------------------------------------------------------------------
    def make_output(self, request: Request) -> RequestOutput:
        proposed = request.num_draft_proposed
        text = None if self.tokenizer is None else self.tokenizer.decode(request.output_ids)
        return RequestOutput(
            request_id=request.request_id, prompt_ids=request.prompt_ids,
            output_ids=request.output_ids, text=text, ttft=request.ttft(),
            tpot=request.tpot(), latency=request.latency(),
            num_preemptions=request.num_preemptions,
            acceptance_rate=request.num_draft_accepted / proposed if proposed else None,
            finish_reason=request.finish_reason())

    def run(self, max_steps: int | None = None) -> list[RequestOutput]:
        """Step until every queued request has finished (or ``max_steps``)."""
        outputs: list[RequestOutput] = []
        taken = 0
        while self.has_unfinished and (max_steps is None or taken < max_steps):
            outputs += self.step()
            taken += 1
        return outputs

    def generate(
        self,
        prompts: Sequence[str] | Sequence[Sequence[int]],
        sampling: SamplingConfig | None = None,
    ) -> list[RequestOutput]:
        """Queue every prompt, run to completion, return outputs in prompt order."""
        order = [self.add_request(p, sampling).request_id for p in prompts]
        by_id = {o.request_id: o for o in self.run()}
        return [by_id[i] for i in order]

    def reset(self) -> None:
        """Drop every request and cached token; the weights stay."""
        self.cache.reset()
        if self.spec is not None:
            self.spec.reset()
        self.scheduler = self._new_scheduler()
        self.stats = EngineStats()
        self._generators.clear()


__all__ = ["EngineStats", "LLMEngine", "RequestOutput"]
