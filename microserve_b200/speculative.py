"""Speculative decoding on the device: draft gamma tokens, verify, accept, roll back.

Reference: src/microserve/speculative.py.  Same API (``SpeculativeDecoder``
with ``step``/``free``/``reset``/``generate``, ``verify_proposals``,
``VerificationResult``) and the same Leviathan et al. accept/reject rule:

    accept x ~ q with probability min(1, p(x) / q(x)); on the first reject
    resample from normalise(max(0, p - q)) (p if that mass is <= 1e-9);
    if all gamma proposals survive, draw a bonus token from p[gamma].

One round (``step``) is, on one stream: gamma draft passes (each a paged
forward that computes logits only for each request's last row, then a draw
that writes the proposal straight into the next pass's inputs and into the
verify batch), one target verify pass over ``[uncached tokens] + proposals``
with logits for the last gamma+1 rows of each request, and the fused
accept/resample/bonus kernel.  The metadata goes up in at most three pinned
copies, planned while earlier passes run, and the accepted tokens come back
in one; the host then rolls both caches back with ``truncate`` as the
reference does (speculative.py:213-226).  When the next round's requests are
known to continue, its draft side is planned on the device and launched
before the host reads the results (round chaining; see SpeculativeDecoder).

Random draws use Philox uniforms keyed by the request generator's seed and
``Request.rng_step`` (see sampling.py), one step per round: draft draw j on
lane j, accept roll i on lane 64+i, the residual/bonus draw on lane 128.
"""

from __future__ import annotations

import itertools
from dataclasses import dataclass, field

import numpy as np
import torch

from . import _lib
from .batching import HostStaging, batch_from_host, pack_int32
from .cache import OutOfCacheMemory, PagedKVCache
from .config import CacheConfig, SamplingConfig
from .model import PagedBatch, Transformer
from .sampling import generator_seed_and_step, make_params, validate
from .scheduler import Request


@dataclass
class VerificationResult:
    """Outcome of verifying one sequence's proposals."""

    tokens: list[int]  # accepted drafts followed by exactly one extra token
    num_accepted: int
    num_proposed: int


def _tails(requests: list[Request], counts: np.ndarray) -> list[list[int]]:
    """The last ``counts[b]`` token ids of each request (its uncached suffix)."""
    out = []
    for r, k in zip(requests, counts.tolist(), strict=True):
        o = r.output_ids
        if k <= len(o):
            out.append(o[len(o) - k :] if k else [])
        else:
            out.append(r.prompt_ids[len(r.prompt_ids) - (k - len(o)) :] + o)
    return out


def _u64_tensor(values: list[int], device: torch.device) -> torch.Tensor:
    """uint64 values carried in an int64 device tensor (same bits)."""
    arr = np.asarray([v & 0xFFFFFFFFFFFFFFFF for v in values], dtype=np.uint64)
    return torch.from_numpy(arr.view(np.int64)).to(device)


def _philox_device(seed: int, step: int, lanes: list[int], device: torch.device) -> torch.Tensor:
    out = torch.empty(len(lanes), dtype=torch.float32, device=device)
    seeds = _u64_tensor([seed], device)
    steps = _u64_tensor([step], device)
    for i, lane in enumerate(lanes):
        _lib.call("ms_philox_uniforms", seeds.data_ptr(), steps.data_ptr(), 1, lane,
                  out[i:].data_ptr(), _lib.stream_ptr(device))
    return out


def verify_proposals(
    draft_probs: torch.Tensor,
    target_probs: torch.Tensor,
    proposals: list[int],
    generator: torch.Generator | None = None,
) -> VerificationResult:
    """Accept/reject test for one sequence (reference speculative.py:44-86).

    ``draft_probs`` is ``(gamma, vocab)``, ``target_probs`` ``(gamma+1, vocab)``.
    """
    gamma = len(proposals)
    if draft_probs.shape[0] != gamma or target_probs.shape[0] != gamma + 1:
        raise ValueError("probability tensors do not match the proposal length")
    dev = draft_probs.device if draft_probs.device.type == "cuda" else torch.device("cuda")
    _lib.require_cuda(dev)
    vocab = int(target_probs.shape[-1])
    q = draft_probs.to(device=dev, dtype=torch.float32).contiguous()
    p = target_probs.to(device=dev, dtype=torch.float32).contiguous()
    x = torch.tensor(proposals, dtype=torch.int32, device=dev)
    seed, step = generator_seed_and_step(generator)
    u = _philox_device(seed, step, [_lib.LANE_ACCEPT + i for i in range(gamma)]
                       + [_lib.LANE_RESAMPLE], dev)
    out = torch.empty(gamma + 1, dtype=torch.int32, device=dev)
    nacc = torch.empty(1, dtype=torch.int32, device=dev)
    _lib.call("ms_verify_probs", p.data_ptr(), q.data_ptr(), x.data_ptr(), u.data_ptr(),
              u[gamma:].data_ptr(), 1, gamma, vocab, out.data_ptr(), nacc.data_ptr(),
              _lib.stream_ptr(dev))
    n = int(nacc.item())
    return VerificationResult(out[: n + 1].tolist(), n, gamma)


class _Buffers:
    """Grow-only flat device (and pinned host) buffers, viewed at the exact
    shape of each round so position-major rows are exactly B apart."""

    def __init__(self, device: torch.device) -> None:
        self.device = device
        self._store: dict[str, torch.Tensor] = {}

    def get(self, name: str, numel: int, dtype: torch.dtype, pinned: bool = False) -> torch.Tensor:
        t = self._store.get(name)
        if t is None or t.numel() < numel:
            cap = max(numel, 2 * (0 if t is None else t.numel()))
            if pinned:
                t = torch.empty(cap, dtype=dtype, pin_memory=True)
            else:
                t = torch.empty(cap, dtype=dtype, device=self.device)
            self._store[name] = t
        return t[:numel]

    def round_views(self, B: int, G: int, V: int) -> None:
        f32, i32 = torch.float32, torch.int32
        self.dlogits = self.get("dlogits", G * B * V, f32).view(G, B, V)
        self.vlogits = self.get("vlogits", B * (G + 1) * V, f32).view(B * (G + 1), V)
        self.dstats = self.get("dstats", G * B * 4, i32).view(G, B, 4)
        self.proposals = self.get("proposals", G * B, i32).view(G, B)
        self.out = self.get("out", B * (G + 2), i32)
        self.out_host = self.get("out_host", B * (G + 2), i32, pinned=True)


def _empty(dtype: type = np.int64) -> np.ndarray:
    return np.zeros(0, dtype)


@dataclass
class _RoundPlan:
    """What a round's three host phases compute.  :meth:`SpeculativeDecoder._plan`
    fills the first group (draft pass 0, before any launch), ``_plan_draft``
    the second (while pass 0 runs), ``_plan_verify`` the third (while the
    draft passes run).  Each ``blob*`` is one pinned upload, ``spans*`` the
    (offset, size) of its parts."""

    blob: np.ndarray
    spans: list[tuple[int, int]]
    B: int
    dw: int
    T0: int
    max_q0: int
    ctx0: int
    kv_draft0: int
    ids: list[int]
    requests: list[Request]
    gens: list[torch.Generator]
    configs: list[SamplingConfig] | None
    n_tok: np.ndarray
    n0: np.ndarray
    npre: np.ndarray
    d_cached: np.ndarray
    t_cached: np.ndarray
    trows: np.ndarray | None
    drows: np.ndarray | None
    dslots: np.ndarray
    dstart: np.ndarray
    tails: np.ndarray
    tail_end: np.ndarray
    # later draft passes, verify token ids, sampling parameters
    blob_d: np.ndarray = field(default_factory=lambda: _empty(np.int32))
    spans_d: list[tuple[int, int]] = field(default_factory=list)
    Tv: int = 0
    max_qv: int = 0
    ctx_j: list[int] = field(default_factory=list)
    qv: np.ndarray = field(default_factory=_empty)
    segv: np.ndarray = field(default_factory=_empty)
    withinv: np.ndarray = field(default_factory=_empty)
    kv_draft: int = 0
    # the verify batch
    blob_v: np.ndarray = field(default_factory=lambda: _empty(np.int32))
    spans_v: list[tuple[int, int]] = field(default_factory=list)
    tw: int = 0
    ctxv: int = 0
    kv_verify: int = 0
    # device views the verify side reads: sampling parameters, verify token ids
    dev_params: torch.Tensor | None = None
    dev_idsv: torch.Tensor | None = None
    # the next round's chain: inputs appended to the verify blob (n_tok,
    # last token, draft tables covering n_tok + 2 gamma tokens)
    chain_reserved: bool = False
    chain_span: int = -1
    chain_dw: int = 0
    dev_blob_v: torch.Tensor | None = None
    v_slot: int = 0  # which of the decoder's two verify-blob buffers holds it
    target_cache: PagedKVCache | None = None


@dataclass
class _Lookahead:
    """The next round's draft passes, launched on the device right after a
    round's accept kernel (planned there by ``ms_spec_chain_plan``), and what
    they assumed about the caller's next ``step`` call."""

    ids: tuple[int, ...]
    requests: list[Request]
    gens: list[torch.Generator]
    configs: list[SamplingConfig] | None
    samplings: list[SamplingConfig]
    seeds: list[int]
    target_cache: PagedKVCache
    max_ctx: int  # an upper bound of the next round's draft contexts
    params: torch.Tensor  # the next round's sampling parameters (device)
    idsv: torch.Tensor  # the next round's verify token ids (device)
    events: tuple[torch.cuda.Event, torch.cuda.Event] | None
    # filled once the round's results are read
    n_tok: np.ndarray = field(default_factory=_empty)  # token counts with the round's tokens
    last: list[int] = field(default_factory=list)  # last tokens then
    t_cached: np.ndarray = field(default_factory=_empty)  # target counts after the rollback


class SpeculativeDecoder:
    """Batched draft-then-verify over decoding requests (reference speculative.py:89-261).

    Lookahead (``lookahead = True``, the default): when no request can stop
    in a round (its budget exceeds the round's gamma + 1 tokens, no stop
    token), the next round's draft side is planned on the device from the
    accepted counts (``ms_spec_chain_plan``) and its draft passes are
    launched right after the accept kernel, before the host reads the
    results: while they run, the host reads this round's tokens, rolls the
    caches back, returns, and the caller's next ``step`` plans and launches
    the verify pass, so the GPU does not wait for the host between rounds.
    The draft cache reserves the blocks those passes write (its token count
    moves only when the host confirms them).  The next ``step`` uses the
    passes only if its requests are the same, in the same order, each with
    exactly the round's tokens appended (and the same sampling settings,
    seeds and target cache state); otherwise they are ignored and the round
    is planned on the host.  Draws are a function of (seed, round counter,
    lane), so the token streams are the same either way.  The target cache,
    which the scheduler's admission reads, is never touched ahead of time."""

    def __init__(
        self,
        target: Transformer,
        draft: Transformer,
        cache_cfg: CacheConfig,
        gamma: int = 4,
        device: str | torch.device = "cuda",
    ) -> None:
        if gamma < 1:
            raise ValueError("gamma must be at least 1")
        if target.cfg.vocab_size != draft.cfg.vocab_size:
            raise ValueError("draft and target must share a vocabulary")
        self.target = target.eval()
        self.draft = draft.eval()
        self.gamma = gamma
        self.device = _lib.require_cuda(device)
        # The draft keeps its own pool, sized by the same CacheConfig as the target's.
        dcfg = CacheConfig(cache_cfg.block_size, cache_cfg.num_blocks, draft.cfg.dtype)
        self.draft_cache = PagedKVCache(draft.cfg, dcfg, self.device)
        self.num_proposed = 0
        self.num_accepted = 0
        self._staging = HostStaging(self.device)
        self._staging_d = HostStaging(self.device)  # later draft passes, verify ids, params
        # The verify batch's blob (phase B), in two buffers used alternately:
        # a round's blob goes up on a copy stream while its draft passes run.
        # Its readers are that round's verify and accept kernels and, when
        # the next round is chained, the next round's chain plan and draft
        # passes (whose block tables it holds); `_v_free[k]` is recorded on
        # the current stream after the last of them was enqueued, and the
        # next upload into buffer k waits for it.
        self._staging_v = [HostStaging(self.device), HostStaging(self.device)]
        self._v_slot = 0
        self._v_free: list[torch.cuda.Event | None] = [None, None]
        self._copy_stream = torch.cuda.Stream(self.device)
        self._v_fence = torch.zeros(1, device=self.device)
        self._buf = _Buffers(self.device)
        self.last_round_launches = 0
        self._row_cache: tuple | None = None  # see _rows_for
        # Measurement hooks (set by benchmarks): when ``round_events`` is a
        # list, each round appends a (start, end) CUDA event pair around its
        # kernels; the last round's shapes and copy sizes are kept below.
        self.round_events: list[tuple[torch.cuda.Event, torch.cuda.Event]] | None = None
        # and when ``verify_events`` is a list, a pair around each verify pass
        self.verify_events: list[tuple[torch.cuda.Event, torch.cuda.Event]] | None = None
        self.last_round_shape: dict[str, int] = {}
        self.last_h2d_bytes = 0
        self.last_d2h_bytes = 0
        self.lookahead = True
        self._pending: _Lookahead | None = None
        self._scat: torch.Tensor | None = None
        self._scat_key: tuple[int, int] | None = None
        self.lookahead_hits = 0
        self.lookahead_misses = 0

    # -- one round ------------------------------------------------------------
    def step(
        self,
        requests: list[Request],
        target_cache: PagedKVCache,
        generators: dict[int, torch.Generator],
    ) -> list[list[int]]:
        """Advance every request by one speculative round; returns the emitted
        tokens (1..gamma+1) per request.  The caller appends them."""
        if not requests:
            return []
        G, B = self.gamma, len(requests)
        configs = list({id(r.sampling): r.sampling for r in requests}.values())
        for cfg in configs:
            validate(cfg)
        launches0 = _lib.launch_count()
        ahead, self._pending = self._pending, None
        plan = None
        if ahead is not None:
            if self._lookahead_holds(ahead, requests, target_cache, generators):
                plan, ev = self._chained_plan(ahead, target_cache), ahead.events
                self.lookahead_hits += 1
            else:
                self.lookahead_misses += 1
        if plan is None:
            plan = self._plan(requests, target_cache, generators, configs)
            ev = self._round_start_events()
            self._launch_draft(plan)
        chain = self.lookahead and self._no_request_can_stop(requests)
        try:
            self._launch_verify(plan, target_cache, ev, chain)
        except OutOfCacheMemory:
            self._drop_draft_slots(plan.ids, plan.d_cached)
            raise
        buf = self._buf
        n_out = B * (G + 2)
        buf.out_host[:n_out].copy_(buf.out[:n_out], non_blocking=True)
        copied = torch.cuda.Event()
        copied.record(torch.cuda.current_stream(self.device))
        if plan.chain_reserved:
            self._pending = self._launch_chain(plan)
        self.last_round_launches = _lib.launch_count() - launches0
        copied.synchronize()
        res = buf.out_host[:n_out].numpy()
        tokens = res[: B * (G + 1)].reshape(B, G + 1)
        nacc = res[B * (G + 1) : B * (G + 2)].astype(np.int64)
        results = self._finish(requests, target_cache, plan, tokens, nacc)
        if self._pending is not None:
            la = self._pending
            la.n_tok = plan.n_tok + nacc + 1
            la.last = [row[-1] for row in results]
            la.t_cached = plan.n_tok + nacc
        return results

    # -- lookahead -----------------------------------------------------------------
    def _no_request_can_stop(self, requests: list[Request]) -> bool:
        """No request can finish with this round's tokens (at most gamma + 1)."""
        room = self.gamma + 1
        return all(r.sampling.stop_token is None
                   and len(r.output_ids) + room < r.sampling.max_new_tokens for r in requests)

    def _launch_chain(self, plan: _RoundPlan) -> _Lookahead:
        """Plan the next round's draft side on the device from this round's
        accepted counts and launch its draft passes (same requests)."""
        G, V = self.gamma, self.target.cfg.vocab_size
        B = plan.B
        buf = self._buf
        stream = _lib.stream_ptr(self.device)
        ev = self._round_start_events()
        chain, params, scat = self._chain_buffers(B)
        o, n = plan.spans_v[plan.chain_span]
        cin = plan.dev_blob_v[o : o + n]
        n_tok, last, dtab = cin[:B], cin[B : 2 * B], cin[2 * B :]
        dc = self.draft_cache
        _lib.call("ms_spec_chain_plan", buf.out.data_ptr(), buf.out[B * (G + 1):].data_ptr(),
                  n_tok.data_ptr(), last.data_ptr(), dtab.data_ptr(), plan.chain_dw, dc.block_size,
                  dc.cfg.num_blocks, plan.dev_params.data_ptr(), B, G, chain.data_ptr(),
                  params.data_ptr(), stream)
        off = 0

        def take(k: int) -> torch.Tensor:
            nonlocal off
            v = chain[off : off + k]
            off += k
            return v

        ids0, pos0, slots0 = take(2 * B), take(2 * B), take(2 * B)
        qs0, ctx0, ql0, rows0 = take(B + 1), take(B), take(B), take(B)
        pos, slots, ctx = take((G - 1) * B), take((G - 1) * B), take((G - 1) * B)
        unit_qs, ones, idsv = take(B + 1), take(B), take((G + 1) * B)
        tables = dtab.view(B, plan.chain_dw)
        max_ctx = int(plan.n_tok.max()) + G + 1
        b0 = PagedBatch(input_ids=ids0, positions=pos0, slot_mapping=slots0, q_start=qs0,
                        context_lens=ctx0, q_lens=ql0, block_tables=tables, max_q=2,
                        n_tokens=2 * B, max_context=max_ctx)
        self.draft.forward_paged(b0, dc, logit_rows=rows0, out=buf.dlogits[0], out_row_stride=V)
        for j in range(G):
            out = buf.dlogits[j]
            if j:
                bj = PagedBatch(input_ids=buf.proposals[j - 1], positions=pos[(j - 1) * B : j * B],
                                slot_mapping=slots[(j - 1) * B : j * B], block_tables=tables,
                                context_lens=ctx[(j - 1) * B : j * B], q_lens=ones,
                                q_start=unit_qs, max_q=1, n_tokens=B, max_context=max_ctx + j)
                self.draft.forward_paged(bj, dc, out=out, out_row_stride=V)
            _lib.call("ms_sample", out.data_ptr(), V, B, V, params.data_ptr(), None,
                      _lib.LANE_DRAFT + j, buf.proposals[j].data_ptr(), None,
                      buf.dstats[j].data_ptr(), idsv.data_ptr(), scat[j].data_ptr(), stream)
        self._release_blob_v(plan)  # the draft passes read their block tables from it
        return _Lookahead(
            ids=tuple(plan.ids), requests=plan.requests, gens=plan.gens, configs=plan.configs,
            samplings=[r.sampling for r in plan.requests],
            seeds=[g.initial_seed() for g in plan.gens], target_cache=plan.target_cache,
            max_ctx=max_ctx, params=params, idsv=idsv, events=ev)

    def _chain_buffers(self, B: int) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        """Device buffers of the chained round: its metadata, its sampling
        parameters, and where each draft pass's proposals go in the verify
        ids (constant: request b's verify rows start at b * (gamma + 1))."""
        G = self.gamma
        n = int(_lib.load().ms_spec_chain_size(B, G))
        chain = self._buf.get("chain", n, torch.int32)
        params = self._buf.get("chain_params", B * _lib.SAMPLING_PARAMS_DTYPE.itemsize,
                               torch.uint8)
        key = (B, G)
        if self._scat_key != key:
            idx = (np.arange(B)[None, :] * (G + 1) + 1 + np.arange(G)[:, None]).astype(np.int32)
            self._scat = torch.from_numpy(idx).to(self.device)
            self._scat_key = key
        return chain, params, self._scat

    def _chained_plan(self, ahead: _Lookahead, target_cache: PagedKVCache) -> _RoundPlan:
        """The host's side of a round whose draft passes ran ahead: the draft
        cache takes the tokens those passes wrote (inside the reserved
        blocks, so the slots are the ones the device used), and the verify
        batch is laid out as the device did (one uncached token per request,
        then the proposals)."""
        G = self.gamma
        ids = list(ahead.ids)
        B = len(ids)
        trows, drows = self._rows_for(ids, target_cache)
        dc = self.draft_cache
        d_cached = dc.num_tokens_many(ids, drows)
        n_tok = ahead.n_tok
        grow = n_tok + G - 1 - d_cached
        if dc.blocks_needed_many(ids, grow, drows) != 0:
            raise RuntimeError("lookahead: the draft passes ran outside the reserved blocks")
        dc.append_many(ids, grow, drows)
        t_cached = target_cache.num_tokens_many(ids, trows)
        npre = n_tok - t_cached
        qv = np.arange(B + 1, dtype=np.int64) * (G + 1)
        segv = np.repeat(np.arange(B), G + 1)
        withinv = np.tile(np.arange(G + 1), B)
        n0 = n_tok - d_cached
        empty = _empty(np.int32)
        plan = _RoundPlan(
            blob=empty, spans=[], B=B, dw=0, T0=2 * B, max_q0=2, ctx0=ahead.max_ctx,
            kv_draft0=int(n_tok.sum()), ids=ids, requests=ahead.requests, gens=ahead.gens,
            configs=ahead.configs, n_tok=n_tok, n0=n0, npre=npre, d_cached=d_cached,
            t_cached=t_cached, trows=trows, drows=drows, dslots=_empty(), dstart=_empty(),
            tails=empty, tail_end=_empty(),
        )
        plan.Tv, plan.max_qv = B * (G + 1), G + 1
        plan.qv, plan.segv, plan.withinv = qv, segv, withinv
        plan.kv_draft = int(n_tok.sum()) * G + B * (G - 1) * G // 2
        plan.dev_params, plan.dev_idsv = ahead.params, ahead.idsv
        return plan

    def _lookahead_holds(self, ahead: _Lookahead, requests: list[Request],
                         target_cache: PagedKVCache,
                         generators: dict[int, torch.Generator]) -> bool:
        """Did the caller do what the lookahead assumed?"""
        if target_cache is not ahead.target_cache or len(requests) != len(ahead.ids):
            return False
        for i, r in enumerate(requests):
            if r.request_id != ahead.ids[i] or r.sampling is not ahead.samplings[i]:
                return False
            if len(r.prompt_ids) + len(r.output_ids) != ahead.n_tok[i]:
                return False
            last = r.output_ids[-1] if r.output_ids else r.prompt_ids[-1]
            if last != ahead.last[i]:
                return False
            gen = generators.get(r.request_id)
            if gen is None or gen.initial_seed() != ahead.seeds[i]:
                return False
        rows = target_cache.rows_if_all_present(list(ahead.ids))
        drows = self.draft_cache.rows_if_all_present(list(ahead.ids))
        if rows is None or drows is None:
            return False
        return bool(np.array_equal(target_cache.num_tokens_many(list(ahead.ids), rows),
                                   ahead.t_cached))

    def _drop_draft_slots(self, ids: list[int], d_cached: np.ndarray) -> None:
        """Give back the draft slots a round took before it failed."""
        keep = [(s, int(n)) for s, n in zip(ids, d_cached.tolist(), strict=True)
                if s in self.draft_cache.tables and self.draft_cache.num_tokens(s) >= n]
        if keep:
            self.draft_cache.truncate_many([s for s, _ in keep], [n for _, n in keep])

    def _round_start_events(self) -> tuple[torch.cuda.Event, torch.cuda.Event] | None:
        if self.round_events is None:
            return None
        ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
        ev[0].record()
        return ev

    def _rows_for(self, ids: list[int], target_cache: PagedKVCache
                  ) -> tuple[np.ndarray | None, np.ndarray | None]:
        """Both caches' table rows of ``ids``, kept from round to round while
        the request list and the caches' row assignments are unchanged; (None,
        None) while a sequence has no row yet (its first round)."""
        key = tuple(ids)
        c = self._row_cache
        if (c is not None and c[0] is target_cache and c[2] == target_cache.generation
                and c[3] == self.draft_cache.generation and c[1] == key):
            return c[4], c[5]
        self._row_cache = None
        if len(set(key)) != len(key):
            return None, None  # append_many reports the duplicate
        trows = target_cache.rows_if_all_present(ids)
        drows = self.draft_cache.rows_if_all_present(ids)
        if trows is None or drows is None:
            return None, None
        self._row_cache = (target_cache, key, target_cache.generation,
                           self.draft_cache.generation, trows, drows)
        return trows, drows

    def _plan(
        self,
        requests: list[Request],
        target_cache: PagedKVCache,
        generators: dict[int, torch.Generator],
        configs: list[SamplingConfig] | None = None,
    ) -> _RoundPlan:
        """What the draft passes need, packed into one blob (phase A).

        The round stays all-or-nothing: the target cache's room for the round
        is checked here, before the draft cache reserves anything, and its
        slots are taken in :meth:`_plan_verify` while the draft passes run.
        """
        G, B = self.gamma, len(requests)
        ids = [r.request_id for r in requests]
        gens = [generators[i] for i in ids]  # a missing generator fails before any change
        dcache = self.draft_cache
        trows, drows = self._rows_for(ids, target_cache)
        d_cached = dcache.num_tokens_many(ids, drows)
        t_cached = target_cache.num_tokens_many(ids, trows)
        n_tok = np.fromiter((len(r.prompt_ids) + len(r.output_ids) for r in requests),
                            np.int64, B)
        n0 = n_tok - d_cached
        npre = n_tok - t_cached
        if np.any(npre < 1):
            raise ValueError("every request needs at least one uncomputed token")
        need = target_cache.blocks_needed_many(ids, npre + G, trows)
        if need > target_cache.num_free_blocks:
            raise OutOfCacheMemory(f"need {need} blocks, {target_cache.num_free_blocks} free")
        # One walk over the token lists: the longer of the two suffixes, split
        # into the draft's catch-up tokens and the target's uncomputed ones.
        kmax = np.maximum(n0, npre)
        tails = np.fromiter(itertools.chain.from_iterable(_tails(requests, kmax)), np.int32,
                            int(kmax.sum()))
        tail_end = np.cumsum(kmax)

        # The draft's slots for the whole round (all-or-nothing).
        dslots = dcache.append_many(ids, n0 + (G - 1), drows)
        dtab, _, dw = dcache.table_rows(ids, drows)

        # Draft pass 0: the catch-up tokens (usually 1 or 2 per request).
        dstart = np.zeros(B + 1, np.int64)
        np.cumsum(n0 + (G - 1), out=dstart[1:])
        q0 = np.zeros(B + 1, np.int64)
        np.cumsum(n0, out=q0[1:])
        T0 = int(q0[-1])
        seg0 = np.repeat(np.arange(B), n0)
        within0 = np.arange(T0) - q0[:-1][seg0]
        ids0 = tails[tail_end[seg0] - n0[seg0] + within0]
        pos0 = d_cached[seg0] + within0
        slots0 = dslots[dstart[:-1][seg0] + within0]
        ctx0 = d_cached + n0
        rows0 = q0[1:] - 1
        parts = [ids0, pos0, slots0, q0, ctx0, n0, dtab, rows0]  # order matches batch_from_host
        blob, spans = pack_int32([np.ascontiguousarray(p).astype(np.int32, copy=False) for p in parts])
        return _RoundPlan(
            blob=blob, spans=spans, B=B, dw=dw, T0=T0, max_q0=int(n0.max()),
            ctx0=int(ctx0.max()), kv_draft0=int(ctx0.sum()), ids=ids, requests=requests,
            gens=gens, configs=configs, n_tok=n_tok, n0=n0, npre=npre, d_cached=d_cached,
            t_cached=t_cached, trows=trows, drows=drows, dslots=dslots, dstart=dstart,
            tails=tails, tail_end=tail_end,
        )

    def _plan_draft(self, plan: _RoundPlan) -> None:
        """Phase A, second part, run on the host while draft pass 0 executes:
        the later draft passes' metadata, the verify token ids with the places
        the proposals go, and the sampling parameters, packed into a second
        blob."""
        G = self.gamma
        B = plan.B
        requests = plan.requests
        gens = plan.gens
        configs = plan.configs
        d_cached = plan.d_cached
        n0 = plan.n0
        npre = plan.npre
        dslots = plan.dslots
        dstart = plan.dstart
        tails = plan.tails
        tail_end = plan.tail_end
        # Draft passes 1..G-1: one token per request (the previous proposal).
        unit_qs = np.arange(B + 1)
        ones = np.ones(B, np.int64)
        pos_j = [d_cached + n0 + j - 1 for j in range(1, G)]
        slots_j = [dslots[dstart[:-1] + n0 + j - 1] for j in range(1, G)]
        ctx_j = [d_cached + n0 + j for j in range(1, G)]

        # Target verify tokens: [uncached tokens] + G proposals per request;
        # the draft samplers write the proposals into their places.
        qv = np.zeros(B + 1, np.int64)
        np.cumsum(npre + G, out=qv[1:])
        Tv = int(qv[-1])
        segv = np.repeat(np.arange(B), npre + G)
        withinv = np.arange(Tv) - qv[:-1][segv]
        idsv = np.zeros(Tv, np.int32)
        is_prefix = withinv < npre[segv]
        segp = segv[is_prefix]
        idsv[is_prefix] = tails[tail_end[segp] - npre[segp] + withinv[is_prefix]]
        scat = [qv[:-1] + npre + j for j in range(G)]

        seeds = [g.initial_seed() for g in gens]
        steps = [r.rng_step for r in requests]
        if configs is not None and len(configs) == 1:  # one config shared by every request
            params = make_params(configs, [0], [0]).repeat(B)
            params["seed"] = seeds
            params["step"] = steps
        else:
            params = make_params([r.sampling for r in requests], seeds, steps)

        parts = [
            params.view(np.int32),
            # shared unit batch arrays for passes >= 1
            unit_qs, ones,
            *[a for j in range(G - 1) for a in (pos_j[j], slots_j[j], ctx_j[j])],
            # verify token ids and where each draft pass's proposals go
            idsv,
            *scat,
        ]
        blob, spans = pack_int32([np.ascontiguousarray(p).astype(np.int32, copy=False) for p in parts])
        plan.blob_d, plan.spans_d, plan.Tv = blob, spans, Tv
        plan.max_qv = int((npre + G).max())
        plan.ctx_j = [int(c.max()) for c in ctx_j]
        plan.qv, plan.segv, plan.withinv = qv, segv, withinv
        plan.kv_draft = plan.kv_draft0 + sum(int(c.sum()) for c in ctx_j)

    def _plan_verify(self, plan: _RoundPlan, target_cache: PagedKVCache,
                     chain: bool = False) -> None:
        """Phase B, run on the host while the draft passes execute: the target
        cache's slots (room checked in :meth:`_plan`) and the verify batch's
        metadata, packed into a third blob.  With ``chain``, the draft cache
        reserves blocks for every request's next round (n_tok + 2 gamma
        tokens) and the blob carries what ``ms_spec_chain_plan`` reads."""
        G = self.gamma
        ids = plan.ids
        npre = plan.npre
        t_cached = plan.t_cached
        qv = plan.qv
        segv = plan.segv
        withinv = plan.withinv
        trows = plan.trows
        tslots = target_cache.append_many(ids, npre + G, trows)
        ttab, _, tw = target_cache.table_rows(ids, trows)
        posv = t_cached[segv] + withinv
        ctxv = t_cached + npre + G
        rowsv = (qv[1:, None] - (G + 1) + np.arange(G + 1)[None, :]).reshape(-1)
        parts = [posv, tslots, qv, ctxv, npre + G, ttab, rowsv]
        plan.target_cache = target_cache
        plan.chain_reserved = chain and self.draft_cache.reserve_many(
            ids, plan.n_tok + 2 * G, plan.drows)
        if plan.chain_reserved:
            dtab, _, dw = self.draft_cache.table_rows(ids, plan.drows)
            last = plan.tails[plan.tail_end - 1] if plan.tails.size else self._last_tokens(plan)
            parts.append(np.concatenate([plan.n_tok.astype(np.int32), last.astype(np.int32),
                                         dtab.reshape(-1)]))
            plan.chain_span, plan.chain_dw = len(parts) - 1, dw
        blob, spans = pack_int32([np.ascontiguousarray(p).astype(np.int32, copy=False) for p in parts])
        plan.blob_v, plan.spans_v, plan.tw = blob, spans, tw
        plan.ctxv, plan.kv_verify = int(ctxv.max()), int(ctxv.sum())

    def _last_tokens(self, plan: _RoundPlan) -> np.ndarray:
        """Every request's last token (a chained round keeps no tails)."""
        return np.fromiter(((r.output_ids[-1] if r.output_ids else r.prompt_ids[-1])
                            for r in plan.requests), np.int32, plan.B)

    def _launch_draft(self, plan: _RoundPlan) -> None:
        """Upload phase A, launch draft pass 0, plan the rest of the draft side
        while it runs, then the later passes and every pass's draw (which
        writes the proposal into the next pass and into the verify batch)."""
        G, V = self.gamma, self.target.cfg.vocab_size
        B = plan.B
        self._buf.round_views(B, G, V)
        buf = self._buf
        dev_blob = self._staging.upload(plan.blob)
        spans = plan.spans
        stream = _lib.stream_ptr(self.device)
        b0 = batch_from_host(dev_blob, spans[0:7], B, plan.dw, plan.max_q0,
                             plan.T0, plan.ctx0)
        dtab = b0.block_tables
        o, n = spans[7]
        rows0 = dev_blob[o : o + n]
        self.draft.forward_paged(b0, self.draft_cache, logit_rows=rows0, out=buf.dlogits[0],
                                 out_row_stride=V)
        # The rest of the draft side is planned while draft pass 0 runs.
        self._plan_draft(plan)
        dblob = self._staging_d.upload(plan.blob_d)
        w = [dblob[o : o + n] for o, n in plan.spans_d]
        params = w[0]
        unit_qs, ones = w[1], w[2]
        k = 3
        batches: list[PagedBatch | None] = [None]
        for j in range(1, G):
            pos, slots, ctx = w[k], w[k + 1], w[k + 2]
            k += 3
            batches.append(PagedBatch(
                input_ids=buf.proposals[j - 1], positions=pos, slot_mapping=slots,
                block_tables=dtab, context_lens=ctx, q_lens=ones, q_start=unit_qs, max_q=1,
                n_tokens=B, max_context=plan.ctx_j[j - 1],
            ))
        idsv = w[k]
        k += 1
        scat = w[k : k + G]
        for j, bj in enumerate(batches):
            out = buf.dlogits[j]
            if bj is not None:
                self.draft.forward_paged(bj, self.draft_cache, out=out, out_row_stride=V)
            _lib.call(
                "ms_sample", out.data_ptr(), V, B, V, params.data_ptr(), None, _lib.LANE_DRAFT + j,
                buf.proposals[j].data_ptr(), None, buf.dstats[j].data_ptr(),
                idsv.data_ptr(), scat[j].data_ptr(), stream,
            )
        plan.dev_params, plan.dev_idsv = params, idsv

    def _launch_verify(self, plan: _RoundPlan, target_cache: PagedKVCache,
                       ev: tuple[torch.cuda.Event, torch.cuda.Event] | None,
                       chain: bool = False) -> None:
        """Plan the target side (its slots are taken here), then the verify pass
        and the fused accept kernel."""
        G, V = self.gamma, self.target.cfg.vocab_size
        B = plan.B
        buf = self._buf
        stream = _lib.stream_ptr(self.device)
        self._plan_verify(plan, target_cache, chain)
        k = self._v_slot
        self._v_slot ^= 1
        vblob = self._staging_v[k].upload_on(plan.blob_v, self._copy_stream, self._v_free[k])
        # A kernel launched without programmatic serialisation after the wait
        # for the copy: the verify pass's first kernel then overlaps this
        # one only, never the copy.
        self._v_fence.zero_()
        plan.dev_blob_v = vblob
        plan.v_slot = k
        w = [vblob[o : o + n] for o, n in plan.spans_v]
        tw = plan.tw
        bv = PagedBatch(
            input_ids=plan.dev_idsv, positions=w[0], slot_mapping=w[1], q_start=w[2],
            context_lens=w[3], q_lens=w[4], block_tables=w[5].view(B, tw), max_q=plan.max_qv,
            n_tokens=plan.Tv, max_context=plan.ctxv,
        )
        rowsv = w[6]
        self.last_round_shape = {"B": B, "T0": plan.T0, "Tv": plan.Tv,
                                 "gamma": G,
                                 # keys each pass's attention reads, summed over requests
                                 "kv_tokens_verify": plan.kv_verify,
                                 "kv_tokens_draft": plan.kv_draft}
        self.last_h2d_bytes = plan.blob.nbytes + plan.blob_d.nbytes + plan.blob_v.nbytes
        self.last_d2h_bytes = B * (G + 2) * 4
        vev = None
        if self.verify_events is not None:
            vev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            vev[0].record()
        self.target.forward_paged(bv, target_cache, logit_rows=rowsv, out=buf.vlogits,
                                  out_row_stride=V)
        if vev is not None and self.verify_events is not None:
            vev[1].record()
            self.verify_events.append(vev)
        _lib.call(
            "ms_spec_accept", buf.vlogits.data_ptr(), V, buf.dlogits.data_ptr(), V,
            buf.dstats.data_ptr(), 0, buf.proposals.data_ptr(), plan.dev_params.data_ptr(), B,
            G, V, buf.out.data_ptr(), buf.out[B * (G + 1) :].data_ptr(), stream,
        )
        self._release_blob_v(plan)
        if ev is not None and self.round_events is not None:
            ev[1].record()
            self.round_events.append(ev)

    def _release_blob_v(self, plan: _RoundPlan) -> None:
        """Every reader of the round's verify blob has been enqueued."""
        done = torch.cuda.Event()
        done.record(torch.cuda.current_stream(self.device))
        self._v_free[plan.v_slot] = done

    def _finish(
        self,
        requests: list[Request],
        target_cache: PagedKVCache,
        plan: _RoundPlan,
        tokens: np.ndarray,
        nacc: np.ndarray,
    ) -> list[list[int]]:
        G = self.gamma
        ids = plan.ids
        n_tok = plan.n_tok
        keep = n_tok + nacc
        target_cache.truncate_many(ids, keep, plan.trows)
        d_len = plan.d_cached + plan.n0 + (G - 1)
        # with a chained round in flight its draft passes write into the
        # blocks reserved for it: keep them
        self.draft_cache.truncate_many(ids, np.minimum(d_len, keep), plan.drows,
                                       keep_blocks=plan.chain_reserved)
        rows = tokens.tolist()
        nacc_l = nacc.tolist()
        keep_l = keep.tolist()
        results: list[list[int]] = []
        for r, row, n, kp in zip(requests, rows, nacc_l, keep_l, strict=True):
            r.num_computed = kp
            r.num_draft_proposed += G
            r.num_draft_accepted += n
            r.rng_step += 1
            del row[n + 1 :]
            results.append(row)
        self.num_proposed += G * len(requests)
        self.num_accepted += int(nacc.sum())
        return results

    # -- lifecycle ----------------------------------------------------------------
    def free(self, seq_id: int) -> None:
        self.draft_cache.free(seq_id)

    def reset(self) -> None:
        self._pending = None
        self._row_cache = None
        self.draft_cache.reset()
        self.num_proposed = 0
        self.num_accepted = 0

    def generate(
        self,
        prompt_ids: list[int],
        sampling: SamplingConfig,
        seq_id: int = 0,
        generator: torch.Generator | None = None,
        target_cache: PagedKVCache | None = None,
    ) -> list[int]:
        """Single-sequence speculative generation (reference speculative.py:237-261)."""
        ccfg = CacheConfig(self.draft_cache.cfg.block_size, self.draft_cache.cfg.num_blocks,
                           self.target.cfg.dtype)
        cache = target_cache or PagedKVCache(self.target.cfg, ccfg, self.device)
        gen = generator or torch.Generator().manual_seed(0)
        request = Request(request_id=seq_id, prompt_ids=list(prompt_ids), sampling=sampling)
        generators = {seq_id: gen}
        try:
            while len(request.output_ids) < sampling.max_new_tokens:
                for token in self.step([request], cache, generators)[0]:
                    if request.should_stop():
                        break
                    request.output_ids.append(token)
                if request.should_stop():
                    break
            return request.output_ids
        finally:
            cache.free(seq_id)
            self.draft_cache.free(seq_id)
