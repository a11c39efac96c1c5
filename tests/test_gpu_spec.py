"""The speculative step and engine on the device against the reference and the oracle."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle.model import OracleModel
from oracle.spec import OracleRequest, spec_round

from .conftest import tiny_dims, tiny_state
from .spec_check import RequestRound, explain
from .test_gpu_model import device_model

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _cache_cfg(block_size=8, num_blocks=32):
    from microserve_b200.config import CacheConfig

    return CacheConfig(block_size, num_blocks)


@pytest.mark.parametrize("i", [0, 1, 2])
def test_greedy_generate_matches_reference(golden, i: int) -> None:
    from microserve_b200.config import SamplingConfig
    from microserve_b200.speculative import SpeculativeDecoder

    target, draft = device_model(golden, "target"), device_model(golden, "draft")
    prompt = golden[f"greedy/{i}/prompt"].tolist()
    assert golden[f"greedy/{i}/dense"].tolist() == golden[f"greedy/{i}/spec1"].tolist()
    for gamma in (1, 2, 3, 5):
        dec = SpeculativeDecoder(target, draft, _cache_cfg(), gamma=gamma)
        got = dec.generate(prompt, SamplingConfig(temperature=0.0, max_new_tokens=20))
        assert got == golden[f"greedy/{i}/spec{gamma}"].tolist()
        assert [dec.num_accepted, dec.num_proposed] == golden[f"greedy/{i}/spec{gamma}_counts"].tolist()
        assert dec.draft_cache.num_free_blocks == dec.draft_cache.cfg.num_blocks


@pytest.mark.parametrize("gamma", [1, 3, 5])
def test_engine_speculative_matches_reference(golden, gamma: int) -> None:
    from microserve_b200.config import (CacheConfig, EngineConfig, SamplingConfig,
                                        SchedulerConfig, SpeculativeConfig)
    from microserve_b200.engine import LLMEngine

    from .test_gpu_model import tiny_model_cfg

    target, draft = device_model(golden, "target"), device_model(golden, "draft")
    cfg = EngineConfig(model=tiny_model_cfg(golden, "target"),
                       cache=CacheConfig(block_size=8, num_blocks=128),
                       scheduler=SchedulerConfig(max_batch_size=3),
                       speculative=SpeculativeConfig(enabled=True, gamma=gamma))
    eng = LLMEngine(target, cfg, draft_model=draft)
    reqs = [eng.add_request(golden[f"engine/prompt/{j}"].tolist(),
                            SamplingConfig(temperature=0.0, max_new_tokens=16)) for j in range(3)]
    outs = {o.request_id: o.output_ids for o in eng.run()}
    for j, r in enumerate(reqs):
        assert outs[r.request_id] == golden[f"engine/g{gamma}/{j}"].tolist()
    assert [eng.stats.num_draft_accepted, eng.stats.num_draft_proposed] == \
        golden[f"engine/g{gamma}/counts"].tolist()
    assert eng.cache.num_free_blocks == cfg.cache.num_blocks
    assert eng.spec.draft_cache.num_free_blocks == cfg.cache.num_blocks
    eng.cache.allocator.check_invariants()


def test_rollback_restores_the_engine_invariant(golden) -> None:
    from microserve_b200.cache import PagedKVCache
    from microserve_b200.config import SamplingConfig
    from microserve_b200.scheduler import Request
    from microserve_b200.speculative import SpeculativeDecoder

    target, draft = device_model(golden, "target"), device_model(golden, "draft")
    dec = SpeculativeDecoder(target, draft, _cache_cfg(), gamma=4)
    cache = PagedKVCache(target.cfg, _cache_cfg(), DEV)
    request = Request(0, [1, 2, 3, 4], SamplingConfig(temperature=0.0, max_new_tokens=40))
    gens = {0: torch.Generator().manual_seed(0)}
    for _ in range(5):
        tokens = dec.step([request], cache, gens)[0]
        request.output_ids.extend(tokens)
        assert cache.num_tokens(0) == request.num_tokens - 1
        assert request.num_computed == request.num_tokens - 1
    cache.free(0)
    dec.free(0)
    cache.allocator.check_invariants()
    assert dec.draft_cache.num_free_blocks == dec.draft_cache.cfg.num_blocks


def test_exact_token_budgets(golden) -> None:
    from microserve_b200.config import (CacheConfig, EngineConfig, SamplingConfig,
                                        SchedulerConfig, SpeculativeConfig)
    from microserve_b200.engine import LLMEngine

    from .test_gpu_model import tiny_model_cfg

    target, draft = device_model(golden, "target"), device_model(golden, "draft")
    cfg = EngineConfig(model=tiny_model_cfg(golden, "target"), cache=CacheConfig(8, 128),
                       scheduler=SchedulerConfig(max_batch_size=2),
                       speculative=SpeculativeConfig(enabled=True, gamma=5))
    eng = LLMEngine(target, cfg, draft_model=draft)
    budgets = {}
    for b in (1, 2, 3, 7, 13):
        r = eng.add_request([1, 2, 3], SamplingConfig(temperature=0.0, max_new_tokens=b))
        budgets[r.request_id] = b
    for out in eng.run():
        assert len(out.output_ids) == budgets[out.request_id]


@pytest.mark.parametrize("setting", [(0.8, None, None), (1.0, 5, 0.9), (0.8, None, 0.9)])
def test_sampled_rounds_match_oracle_draw_for_draw(golden, setting) -> None:
    """Sampled streams are exact given shared uniforms: proposals, accepted
    lengths and emitted tokens per round, for a batch of requests."""
    from microserve_b200.cache import PagedKVCache
    from microserve_b200.config import SamplingConfig
    from microserve_b200.scheduler import Request
    from microserve_b200.speculative import SpeculativeDecoder

    t, k, p = setting
    gamma = 3
    target, draft = device_model(golden, "target"), device_model(golden, "draft")
    o_t = OracleModel(tiny_dims(golden, "target"), tiny_state(golden, "target"))
    o_d = OracleModel(tiny_dims(golden, "draft"), tiny_state(golden, "draft"))
    dec = SpeculativeDecoder(target, draft, _cache_cfg(8, 64), gamma=gamma)
    dec.lookahead = False  # the round's proposals are read back out of its buffers
    cache = PagedKVCache(target.cfg, _cache_cfg(8, 64), DEV)
    rng = np.random.default_rng(4)
    sc = SamplingConfig(temperature=t, top_k=k, top_p=p, max_new_tokens=64)
    prompts = [rng.integers(0, 32, int(n)).tolist() for n in (5, 12, 3, 9)]
    reqs = [Request(i, pr, sc) for i, pr in enumerate(prompts)]
    gens = {i: torch.Generator().manual_seed(500 + i) for i in range(len(reqs))}
    oreqs = [OracleRequest(i, pr, t, k, p, seed=500 + i) for i, pr in enumerate(prompts)]
    diverged: dict[int, str] = {}
    for _ in range(6):
        live = [i for i in range(len(reqs)) if i not in diverged]
        if not live:
            break
        steps = [oreqs[i].step for i in live]
        got = dec.step([reqs[i] for i in live], cache, gens)
        props = dec._buf.proposals.cpu().numpy()
        tr = spec_round(o_t, o_d, gamma, [oreqs[i] for i in live])
        for j, i in enumerate(live):
            if got[j] != tr.emitted[j] or props[:, j].tolist() != tr.proposals[j]:
                # only at a decision boundary, within the 1e-4 relative
                # tolerance of the float32 logits each side computes
                rr = RequestRound(oreqs[i].seed, steps[j], tr.draft_rows[j], tr.target_rows[j],
                                  tr.proposals[j], tr.emitted[j], tr.num_accepted[j])
                why = explain(rr, props[:, j].tolist(), got[j], tol=1e-4)
                assert why is not None, (i, got[j], tr.emitted[j])
                diverged[i] = why
                continue
            reqs[i].output_ids.extend(got[j])
            oreqs[i].output_ids.extend(tr.emitted[j])
            assert cache.num_tokens(i) == reqs[i].num_tokens - 1
    assert len(diverged) <= 1, diverged


def test_streams_do_not_depend_on_how_requests_are_sharded(golden) -> None:
    """Eight sampled requests served by one decoder, and split over two
    decoders by the longest-processing-time partition of two ranks: every
    request's stream is the same, because its Philox stream is keyed by its
    own generator seed and round counter, never by its batch or rank."""
    from microserve_b200 import distributed
    from microserve_b200.cache import PagedKVCache
    from microserve_b200.config import SamplingConfig
    from microserve_b200.scheduler import Request
    from microserve_b200.speculative import SpeculativeDecoder

    target, draft = device_model(golden, "target"), device_model(golden, "draft")
    rng = np.random.default_rng(12)
    prompts = [rng.integers(0, 32, int(n)).tolist() for n in rng.integers(2, 30, 8)]
    sc = SamplingConfig(temperature=0.8, top_p=0.95, max_new_tokens=64)

    def serve(ids: list[int]) -> dict[int, list[int]]:
        dec = SpeculativeDecoder(target, draft, _cache_cfg(8, 96), gamma=3)
        cache = PagedKVCache(target.cfg, _cache_cfg(8, 96), DEV)
        reqs = [Request(g, list(prompts[g]), sc) for g in ids]
        gens = {g: torch.Generator().manual_seed(700 + g) for g in ids}
        for _ in range(5):
            for r, toks in zip(reqs, dec.step(reqs, cache, gens), strict=True):
                r.output_ids.extend(toks)
        return {r.request_id: r.output_ids for r in reqs}

    one = serve(list(range(8)))
    two: dict[int, list[int]] = {}
    for rank in range(2):
        two.update(serve(distributed.shard_requests([float(len(p)) for p in prompts], 2, rank)))
    assert two == one


def test_lookahead_keeps_the_streams_and_gives_back_its_slots(golden) -> None:
    """The next round's draft passes launched ahead of the caller (lookahead)
    change nothing observable: streams equal a decoder without it, also when
    the caller's next call differs from what the lookahead assumed (a request
    dropped, a request added); the draft pool is whole again after free()."""
    from microserve_b200.cache import PagedKVCache
    from microserve_b200.config import SamplingConfig
    from microserve_b200.scheduler import Request
    from microserve_b200.speculative import SpeculativeDecoder

    target, draft = device_model(golden, "target"), device_model(golden, "draft")
    rng = np.random.default_rng(21)
    prompts = [rng.integers(0, 32, int(n)).tolist() for n in rng.integers(2, 20, 6)]
    sc = SamplingConfig(temperature=0.9, top_k=20, max_new_tokens=200)
    # call pattern: the batch changes at calls 3 (request 5 leaves) and 5 (it returns)
    batches = [[0, 1, 2, 3, 4, 5]] * 3 + [[0, 1, 2, 3, 4]] * 2 + [[0, 1, 2, 3, 4, 5]] * 3

    def serve(lookahead: bool):
        dec = SpeculativeDecoder(target, draft, _cache_cfg(8, 128), gamma=3)
        dec.lookahead = lookahead
        cache = PagedKVCache(target.cfg, _cache_cfg(8, 128), DEV)
        reqs = [Request(i, list(p), sc) for i, p in enumerate(prompts)]
        gens = {i: torch.Generator().manual_seed(900 + i) for i in range(len(prompts))}
        for ids in batches:
            for i, toks in zip(ids, dec.step([reqs[i] for i in ids], cache, gens), strict=True):
                reqs[i].output_ids.extend(toks)
        outs = [r.output_ids for r in reqs]
        for i in range(len(prompts)):
            cache.free(i)
            dec.free(i)
        assert dec.draft_cache.num_free_blocks == dec.draft_cache.cfg.num_blocks
        assert cache.num_free_blocks == cache.cfg.num_blocks
        return outs, dec

    plain, _ = serve(False)
    ahead, dec = serve(True)
    assert ahead == plain
    assert dec.lookahead_hits >= 4 and dec.lookahead_misses >= 2
