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


def test_chain_plan_kernel_matches_a_host_restatement() -> None:
    """ms_spec_chain_plan through the C ABI against the next round's draft-side
    metadata computed here on the host, request by request: after a round
    with n accepted of gamma proposals, a request that had T tokens holds
    T + n + 1; draft pass 0 takes its last two tokens (the first to a spare
    reserved slot unless n == gamma), pass j its token at T + n + j, the
    verify batch starts with the emitted token at T + n, and the sampling
    step advances by one."""
    from microserve_b200 import _lib
    from microserve_b200.config import SamplingConfig
    from microserve_b200.sampling import make_params, params_to_device

    rng = np.random.default_rng(3)
    B, G, bs, nb = 7, 4, 8, 200
    T = rng.integers(1, 60, B)
    nacc = rng.integers(0, G + 1, B)
    nacc[0], nacc[1] = 0, G  # both ends
    out_tok = rng.integers(0, 1000, (B, G + 1)).astype(np.int32)
    last = rng.integers(0, 1000, B).astype(np.int32)
    width = int(((T + 2 * G + bs - 1) // bs).max())
    tables = rng.permutation(nb)[: B * width].reshape(B, width).astype(np.int32)
    params = make_params([SamplingConfig(temperature=0.8)] * B, np.arange(B) + 11,
                         np.arange(B) * 3 + 5)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a, dtype=np.int32)).to(DEV)  # noqa: E731
    d_out, d_nacc, d_T, d_last, d_tab = dev(out_tok), dev(nacc), dev(T), dev(last), dev(tables)
    p_in = params_to_device(params, torch.device(DEV))
    p_out = torch.empty_like(p_in)
    n = int(_lib.load().ms_spec_chain_size(B, G))
    chain = torch.full((n,), -7, dtype=torch.int32, device=DEV)
    _lib.call("ms_spec_chain_plan", d_out.data_ptr(), d_nacc.data_ptr(), d_T.data_ptr(),
              d_last.data_ptr(), d_tab.data_ptr(), width, bs, nb, p_in.data_ptr(), B, G,
              chain.data_ptr(), p_out.data_ptr(), _lib.stream_ptr())
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    got = chain.cpu().numpy()
    slot = lambda b, p: int(tables[b, p // bs]) * bs + p % bs  # noqa: E731
    want = {k: [] for k in ("ids0", "pos0", "slots0", "pos", "slots", "ctx", "ctx0")}
    idsv_first = []
    pos_j = np.zeros((G - 1, B), np.int64)
    slots_j = np.zeros((G - 1, B), np.int64)
    ctx_j = np.zeros((G - 1, B), np.int64)
    for b in range(B):
        n_b, t = int(nacc[b]), int(T[b])
        ntok = t + n_b + 1
        tok_a = int(out_tok[b, n_b - 1]) if n_b >= 1 else int(last[b])
        want["ids0"] += [tok_a, int(out_tok[b, n_b])]
        want["pos0"] += [ntok - 2, ntok - 1]
        want["slots0"] += [slot(b, ntok - 2 if n_b == G else t + 2 * G - 1), slot(b, ntok - 1)]
        want["ctx0"].append(ntok)
        idsv_first.append(int(out_tok[b, n_b]))
        for j in range(1, G):
            pos_j[j - 1, b] = ntok + j - 1
            slots_j[j - 1, b] = slot(b, ntok + j - 1)
            ctx_j[j - 1, b] = ntok + j
    o = 0

    def take(k: int) -> np.ndarray:
        nonlocal o
        v = got[o : o + k]
        o += k
        return v

    assert take(2 * B).tolist() == want["ids0"]
    assert take(2 * B).tolist() == want["pos0"]
    assert take(2 * B).tolist() == want["slots0"]
    assert take(B + 1).tolist() == [2 * b for b in range(B + 1)]
    assert take(B).tolist() == want["ctx0"]
    assert take(B).tolist() == [2] * B
    assert take(B).tolist() == [2 * b + 1 for b in range(B)]
    assert take((G - 1) * B).tolist() == pos_j.reshape(-1).tolist()
    assert take((G - 1) * B).tolist() == slots_j.reshape(-1).tolist()
    assert take((G - 1) * B).tolist() == ctx_j.reshape(-1).tolist()
    assert take(B + 1).tolist() == list(range(B + 1))
    assert take(B).tolist() == [1] * B
    verify_ids = take((G + 1) * B).reshape(B, G + 1)
    assert verify_ids[:, 0].tolist() == idsv_first
    assert (verify_ids[:, 1:] == -7).all()  # left for the samplers' scatter
    assert o == n
    po = np.frombuffer(p_out.cpu().numpy().tobytes(), dtype=_lib.SAMPLING_PARAMS_DTYPE)
    assert po["step"].tolist() == (params["step"] + 1).tolist()
    assert po["seed"].tolist() == params["seed"].tolist()
