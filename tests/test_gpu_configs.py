"""Parity at the benchmark configurations' shapes, through the public API.

* config 0 (character-level fp32 target and draft, 8 requests, gamma 3):
  the engine's greedy token streams and acceptance counts against the
  unmodified reference engine's (``config_fixtures.npz``), and its sampled
  streams at temperature 0.8 against the oracle draw for draw;
* config 2 (the same models, continuous batching): a 64-request subset of
  the workload at gamma 1/2/3/5, greedy, against the reference engine, and
  24 requests in a 64-block pool, where the reference preempts between
  speculative rounds;
* config 1 (acceptance microbenchmark): one ``ms_spec_accept`` launch at the
  full 4096 x gamma 5 x 32000, a fixed subset of 256 requests checked
  against the oracle;
* configs 3 and 4 (Llama-1.1B and Llama-3-8B widths in bf16, layer counts
  reduced): speculative rounds whose draft and verify logits are checked
  against the float32 oracle on the same bf16-rounded weights and K/V
  histories, and whose every sampling decision is checked against the
  oracle's on the device's own logits.
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import philox
from oracle.model import Dims, OracleModel
from oracle.sampling import filter_row, near_boundary
from oracle.spec import OracleRequest, prefill, spec_round

from .spec_check import RequestRound, decide, explain, pool_history
from .test_gpu_model import assert_bf16_close

pytestmark = pytest.mark.gpu

DEV = "cuda"
GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.fixture(scope="module")
def cfgfix() -> dict[str, np.ndarray]:
    with np.load(GOLDEN / "config_fixtures.npz") as z:
        return {k: z[k] for k in z.files}


def _wl():
    import sys

    if str(GOLDEN) not in sys.path:
        sys.path.insert(0, str(GOLDEN))
    import workloads

    return workloads


def _model_cfg(shape, dtype: str = "float32", **kw):
    from microserve_b200.config import ModelConfig

    return ModelConfig(vocab_size=shape.vocab_size, n_layers=shape.n_layers,
                       d_model=shape.d_model, n_heads=shape.n_heads,
                       n_kv_heads=shape.n_kv_heads, d_ff=shape.d_ff,
                       max_seq_len=shape.max_seq_len, rope_theta=shape.rope_theta, dtype=dtype,
                       **kw)


def _dims(cfg) -> Dims:
    return Dims(cfg.vocab_size, cfg.d_model, cfg.n_layers, cfg.n_heads, cfg.kv_heads,
                cfg.ffn_hidden, cfg.max_seq_len, cfg.rope_theta, cfg.norm_eps)


def _char_models(amp: float):
    from microserve_b200.model import Transformer

    wl = _wl()
    ts, ds = wl.init_state(wl.CHAR_TARGET, 0, amp), wl.init_state(wl.CHAR_DRAFT, 1, amp)
    tcfg, dcfg = _model_cfg(wl.CHAR_TARGET), _model_cfg(wl.CHAR_DRAFT)
    return (Transformer.from_state_dict(tcfg, ts, DEV), Transformer.from_state_dict(dcfg, ds, DEV),
            (tcfg, ts), (dcfg, ds))


def _engine(target, draft, gamma: int, blocks: int, max_batch: int, max_tokens: int):
    from microserve_b200.config import (CacheConfig, EngineConfig, SchedulerConfig,
                                        SpeculativeConfig)
    from microserve_b200.engine import LLMEngine

    cfg = EngineConfig(model=target.cfg, cache=CacheConfig(block_size=16, num_blocks=blocks),
                       scheduler=SchedulerConfig(max_batch_size=max_batch,
                                                 max_batched_tokens=max_tokens),
                       speculative=SpeculativeConfig(enabled=True, gamma=gamma))
    return LLMEngine(target, cfg, draft_model=draft)


def _greedy_run(eng, prompts, budgets):
    from microserve_b200.config import SamplingConfig

    reqs = [eng.add_request(p, SamplingConfig(temperature=0.0, max_new_tokens=int(b)))
            for p, b in zip(prompts, budgets, strict=True)]
    outs = {o.request_id: o.output_ids for o in eng.run()}
    counts = [eng.stats.num_draft_accepted, eng.stats.num_draft_proposed, eng.stats.num_steps]
    return [outs[r.request_id] for r in reqs], counts


# -- config 0 ---------------------------------------------------------------------
@pytest.mark.parametrize("amp", [1, 20])
def test_config0_engine_greedy_matches_reference(cfgfix, amp: int) -> None:
    """8 requests, prompts lognormal(100, 50) in [8, 256], 50 new tokens, gamma 3,
    block 16 x 256 blocks: token streams, acceptance counts and the number of
    engine steps equal the reference engine's.  ``amp`` 20 scales the residual
    projections as the reference's test fixture does, so the two models disagree."""
    target, draft, _, _ = _char_models(float(amp))
    w = _wl().config0()
    eng = _engine(target, draft, 3, 256, 8, 2048)
    got, counts = _greedy_run(eng, w.prompts, w.max_new_tokens)
    for j, toks in enumerate(got):
        assert toks == cfgfix[f"cfg0/a{amp}/g3/{j}"].tolist(), f"request {j}"
    assert counts == cfgfix[f"cfg0/a{amp}/g3/counts"].tolist()
    assert eng.cache.num_free_blocks == 256


def test_config0_engine_sampled_matches_oracle() -> None:
    """Config 0 at temperature 0.8: every request's stream, round by round,
    equals the oracle's given the shared Philox uniforms.  A differing
    request must sit at a decision boundary within the 1e-4 relative logit
    tolerance of float32 (each side computes its own logits); at most one may."""
    from microserve_b200.config import SamplingConfig

    target, draft, (tcfg, ts), (dcfg, ds) = _char_models(20.0)
    o_t, o_d = OracleModel(_dims(tcfg), ts), OracleModel(_dims(dcfg), ds)
    w = _wl().config0()
    eng = _engine(target, draft, 3, 256, 8, 2048)
    sc = SamplingConfig(temperature=0.8, max_new_tokens=50)
    reqs = [eng.add_request(p, sc) for p in w.prompts]
    seeds = [eng.config.seed + r.request_id for r in reqs]
    oreqs = [OracleRequest(i, list(p), 0.8, None, None, seed=s)
             for i, (p, s) in enumerate(zip(w.prompts, seeds, strict=True))]
    # engine step 1 prefills every request (one token each on lane 0)
    eng.step()
    first = prefill(o_t, oreqs)
    for r, o, t in zip(reqs, oreqs, first, strict=True):
        assert r.output_ids == [t]
        o.output_ids.append(t)
    diverged: dict[int, str] = {}
    live = list(range(len(reqs)))
    while eng.has_unfinished:
        before = [len(r.output_ids) for r in reqs]
        step = {i: oreqs[i].step for i in live}
        tr = spec_round(o_t, o_d, 3, [oreqs[i] for i in live])
        eng.step()
        still = []
        for j, i in enumerate(live):
            got = reqs[i].output_ids[before[i]:]
            want = tr.emitted[j][: 50 - before[i]]
            if got != want:
                rr = RequestRound(oreqs[i].seed, step[i], tr.draft_rows[j], tr.target_rows[j],
                                  tr.proposals[j], tr.emitted[j], tr.num_accepted[j])
                why = explain(rr, None, got, tol=1e-4)
                assert why is not None, (i, got, want)
                diverged[i] = why
                continue
            oreqs[i].output_ids.extend(want)
            if len(oreqs[i].output_ids) < 50:
                still.append(i)
        live = still
    assert len(diverged) <= 1, diverged
    assert eng.stats.num_draft_proposed > 0


# -- config 2 ---------------------------------------------------------------------
@pytest.mark.parametrize("gamma,amp", [(1, 1), (2, 1), (3, 1), (5, 1), (3, 20)])
def test_config2_engine_subset_matches_reference(cfgfix, gamma: int, amp: int) -> None:
    """64 concurrent requests of the continuous-batching workload (prompts
    lognormal(100, 50) in [8, 512], outputs uniform 1..50, block 16), greedy:
    streams, acceptance counts and engine steps equal the reference's."""
    target, draft, _, _ = _char_models(float(amp))
    w = _wl().config2(64)
    eng = _engine(target, draft, gamma, 4096, 64, 64 * 600)
    got, counts = _greedy_run(eng, w.prompts, w.max_new_tokens)
    for j, toks in enumerate(got):
        assert toks == cfgfix[f"cfg2/a{amp}/g{gamma}/{j}"].tolist(), f"request {j}"
    assert counts == cfgfix[f"cfg2/a{amp}/g{gamma}/counts"].tolist()
    eng.cache.allocator.check_invariants()


@pytest.mark.parametrize("amp", [1, 20])
def test_config2_engine_under_memory_pressure_matches_reference(cfgfix, amp: int) -> None:
    """24 requests of the continuous-batching workload in a pool of 64 blocks
    of 16: running requests are preempted between speculative rounds and
    recomputed by prefill.  Streams, acceptance counts, engine steps and the
    number of preemptions equal the reference engine's."""
    target, draft, _, _ = _char_models(float(amp))
    w = _wl().config2(24, seed=5)
    eng = _engine(target, draft, 3, 64, 24, 4096)
    got, counts = _greedy_run(eng, w.prompts, w.max_new_tokens)
    for j, toks in enumerate(got):
        assert toks == cfgfix[f"cfg2p/a{amp}/g3/{j}"].tolist(), f"request {j}"
    want = cfgfix[f"cfg2p/a{amp}/g3/counts"].tolist()
    assert counts + [eng.stats.num_preemptions] == want
    assert want[3] > 0
    eng.cache.allocator.check_invariants()
    assert eng.cache.num_free_blocks == eng.cache.allocator.num_blocks


# -- config 1 ---------------------------------------------------------------------
@pytest.mark.parametrize("setting", [(1.0, None, None), (1.0, 50, None), (1.0, None, 0.9)])
def test_config1_accept_full_size(setting) -> None:
    """One ms_spec_accept launch over 4096 requests x gamma 5 x vocab 32000
    (target logits N(0, 2^2), draft = target + N(0, 0.5^2), seed 1234); the
    proposals are drawn from the draft rows by ms_sample.  Every 16th request
    (256 of them) is checked against the oracle on the same rows and uniforms."""
    from microserve_b200 import _lib
    from microserve_b200.config import SamplingConfig
    from microserve_b200.sampling import make_params, params_to_device

    t, k, p = setting
    B, G, V = 4096, 5, 32000
    gen = torch.Generator(device=DEV).manual_seed(1234)
    target = torch.randn(B, G + 1, V, device=DEV, generator=gen) * 2.0
    draft = (target[:, :G, :] + torch.randn(B, G, V, device=DEV, generator=gen) * 0.5)
    draft = draft.permute(1, 0, 2).contiguous()  # position-major: row i*B + b
    target = target.reshape(B * (G + 1), V)
    seeds = np.arange(B, dtype=np.uint64) + np.uint64(1234)
    steps = np.zeros(B, dtype=np.uint64)
    params = params_to_device(make_params([SamplingConfig(temperature=t, top_k=k, top_p=p)] * B,
                                          seeds, steps), torch.device(DEV))
    props = torch.empty((G, B), dtype=torch.int32, device=DEV)
    stats = torch.empty((G * B, 4), dtype=torch.int32, device=DEV)
    pidx = (torch.arange(G * B, device=DEV, dtype=torch.int32) % B).contiguous()
    for j in range(G):  # draft pass j draws on lane j, as the round does
        _lib.call("ms_sample", draft[j].data_ptr(), V, B, V, params.data_ptr(), None, j,
                  props[j].data_ptr(), None, stats[j * B:].data_ptr(), None, None,
                  _lib.stream_ptr())
    _ = pidx
    out = torch.empty(B * (G + 1), dtype=torch.int32, device=DEV)
    nacc = torch.empty(B, dtype=torch.int32, device=DEV)
    _lib.call("ms_spec_accept", target.data_ptr(), V, draft.data_ptr(), V, stats.data_ptr(), 0,
              props.data_ptr(), params.data_ptr(), B, G, V, out.data_ptr(), nacc.data_ptr(),
              _lib.stream_ptr())
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    check = np.arange(0, B, 16)
    idx = torch.from_numpy(check).to(DEV)
    tl = target.view(B, G + 1, V).index_select(0, idx).cpu().numpy()
    dl = draft.index_select(1, idx).permute(1, 0, 2).cpu().numpy()  # (n, G, V)
    got_props = props.index_select(1, idx).cpu().numpy().T
    got_tok = out.view(B, G + 1).index_select(0, idx).cpu().numpy()
    got_n = nacc.index_select(0, idx).cpu().numpy()
    odd: dict[int, str] = {}
    accepted = 0
    for c, b in enumerate(check.tolist()):
        seed = int(seeds[b])
        rr = decide(seed, 0, dl[c], tl[c], t, k, p)
        emitted = got_tok[c, : got_n[c] + 1].tolist()
        accepted += int(got_n[c])
        if got_props[c].tolist() != rr.proposals or emitted != rr.emitted:
            why = explain(rr, got_props[c].tolist(), emitted, tol=1e-5)
            assert why is not None, (b, got_props[c].tolist(), rr.proposals, emitted, rr.emitted)
            odd[b] = why
    assert len(odd) <= 2, odd
    assert 0 < accepted < len(check) * G  # accepts and rejects both occur


# -- configs 3 and 4: real widths in bf16 ------------------------------------------
def _bf16_state(cfg, seed: int, amp: float) -> dict[str, torch.Tensor]:
    """Reference-format weights drawn on the device in bf16 (the reference's
    init rule, o_proj and down_proj scaled by ``amp``)."""
    g = torch.Generator(device=DEV).manual_seed(seed)
    d, hq, hkv, dh, ff, L = (cfg.d_model, cfg.n_heads, cfg.kv_heads, cfg.d_head, cfg.ffn_hidden,
                             cfg.n_layers)
    res = 0.02 / np.sqrt(2 * L) * amp

    def n(rows: int, cols: int, std: float) -> torch.Tensor:
        return (torch.randn(rows, cols, device=DEV, generator=g) * std).bfloat16()

    st = {"embed.weight": n(cfg.vocab_size, d, 0.02),
          "norm.weight": torch.ones(d, device=DEV)}
    for i in range(L):
        p = f"blocks.{i}."
        st[p + "attn.q_proj.weight"] = n(hq * dh, d, 0.02)
        st[p + "attn.k_proj.weight"] = n(hkv * dh, d, 0.02)
        st[p + "attn.v_proj.weight"] = n(hkv * dh, d, 0.02)
        st[p + "attn.o_proj.weight"] = n(d, hq * dh, res)
        st[p + "ffn.gate_proj.weight"] = n(ff, d, 0.02)
        st[p + "ffn.up_proj.weight"] = n(ff, d, 0.02)
        st[p + "ffn.down_proj.weight"] = n(d, ff, res)
        st[p + "attn_norm.weight"] = torch.ones(d, device=DEV)
        st[p + "ffn_norm.weight"] = torch.ones(d, device=DEV)
    return st


class _Setup:
    """Target + draft at real widths, caches holding synthetic K/V histories
    (N(0, 1), the benchmark's contexts), requests one token short of cached."""

    def __init__(self, tshape: dict, dshape: dict, gamma: int, ctx: list[int], amp: float,
                 sampling, seed: int) -> None:
        from microserve_b200.cache import PagedKVCache
        from microserve_b200.config import CacheConfig, ModelConfig
        from microserve_b200.model import Transformer
        from microserve_b200.scheduler import Request
        from microserve_b200.speculative import SpeculativeDecoder

        tcfg = ModelConfig(**tshape, dtype="bfloat16")
        dcfg = ModelConfig(**dshape, dtype="bfloat16")
        tst, dst = _bf16_state(tcfg, seed, amp), _bf16_state(dcfg, seed + 1, amp)
        self.target = Transformer.from_state_dict(tcfg, tst, DEV)
        self.draft = Transformer.from_state_dict(dcfg, dst, DEV)
        host = lambda st: {k: v.float().cpu().numpy() for k, v in st.items()}  # noqa: E731
        self.o_t = OracleModel(_dims(tcfg), host(tst))
        self.o_d = OracleModel(_dims(dcfg), host(dst))
        del tst, dst
        B = len(ctx)
        blocks = sum(-(-(c + 4 * (gamma + 1)) // 16) + 1 for c in ctx) + 16
        ccfg = CacheConfig(16, blocks, "bfloat16")
        self.cache = PagedKVCache(tcfg, ccfg, DEV)
        self.dec = SpeculativeDecoder(self.target, self.draft, ccfg, gamma=gamma, device=DEV)
        self.dec.lookahead = False  # the checks read this round's logits out of its buffers
        rng = np.random.default_rng(seed)
        self.reqs, self.gens, self.oreqs = [], {}, []
        for i, c in enumerate(ctx):
            prompt = rng.integers(0, tcfg.vocab_size, int(c)).tolist()
            r = Request(i, prompt, sampling)
            r.num_computed = c - 1
            self.reqs.append(r)
            self.gens[i] = torch.Generator().manual_seed(9000 + i)
        # interleaved allocation, 16 tokens at a time: non-contiguous tables
        remaining = np.asarray(ctx) - 1
        while remaining.max() > 0:
            stp = np.minimum(remaining, 16)
            live = [i for i in range(B) if stp[i] > 0]
            self.cache.append_many(live, stp[live])
            self.dec.draft_cache.append_many(live, stp[live])
            remaining -= stp
        g = torch.Generator(device=DEV).manual_seed(seed + 5)
        for pool in (self.cache.pool, self.dec.draft_cache.pool):
            pool.normal_(generator=g)
        for i, c in enumerate(ctx):
            o = OracleRequest(i, list(self.reqs[i].prompt_ids), sampling.temperature,
                              sampling.top_k, sampling.top_p, seed=9000 + i)
            o.target_kv = pool_history(self.cache, i, c - 1)
            o.draft_kv = pool_history(self.dec.draft_cache, i, c - 1)
            self.oreqs.append(o)

    def round(self, gamma: int) -> dict[str, object]:
        """One device round, checked against the oracle; returns statistics."""
        dec, B = self.dec, len(self.reqs)
        steps = [r.rng_step for r in self.reqs]
        emitted = dec.step(self.reqs, self.cache, self.gens)
        torch.cuda.synchronize()
        V = self.target.cfg.vocab_size
        dlog = dec._buf.dlogits.cpu().numpy()  # (G, B, V)
        vlog = dec._buf.vlogits.cpu().numpy().reshape(B, gamma + 1, V)
        props = dec._buf.proposals.cpu().numpy()  # (G, B)
        # logits: the oracle's draft passes fed the device's proposals, then its verify pass
        pending = [o.all_ids[o.draft_kv.length:] for o in self.oreqs]
        for j in range(gamma):
            lg = self.o_d.forward(pending, [o.draft_kv for o in self.oreqs],
                                  logit_rows=[[len(p) - 1] for p in pending])
            assert_bf16_close(dlog[j], np.stack([x[0] for x in lg]))
            pending = [[int(props[j, b])] for b in range(B)]
        lists = [o.all_ids[o.target_kv.length:] + props[:, b].tolist()
                 for b, o in enumerate(self.oreqs)]
        wins = [[len(t) - (gamma + 1) + i for i in range(gamma + 1)] for t in lists]
        tl = self.o_t.forward(lists, [o.target_kv for o in self.oreqs], logit_rows=wins)
        assert_bf16_close(vlog, np.stack(tl))
        # decisions on the device's own logits
        sc = self.reqs[0].sampling
        odd = {}
        entropy = []
        for b, o in enumerate(self.oreqs):
            seed = int(self.gens[b].initial_seed())
            mine = decide(seed, steps[b], dlog[:, b], vlog[b], sc.temperature, sc.top_k, sc.top_p)
            rr = decide(seed, steps[b], dlog[:, b], vlog[b], sc.temperature, sc.top_k, sc.top_p,
                        proposals=props[:, b].tolist())
            for j in range(gamma):
                if props[j, b] != mine.proposals[j]:
                    u = float(philox.uniform(seed, steps[b], j))
                    assert near_boundary(mine.q_rows[j], u, 1e-5), (b, j)
                    odd[b] = f"draft draw {j}"
            if emitted[b] != rr.emitted:
                why = explain(rr, props[:, b].tolist(), emitted[b], tol=1e-5)
                assert why is not None, (b, emitted[b], rr.emitted)
                odd[b] = why
            if sc.temperature > 0:
                pr = rr.p_rows[0].probs
                entropy.append(float(-(pr[pr > 0] * np.log(pr[pr > 0])).sum()))
            # roll both oracle histories back as the device did
            keep = len(o.all_ids) + len(emitted[b]) - 1
            o.target_kv.truncate(keep)
            o.draft_kv.truncate(min(o.draft_kv.length, keep))
            o.output_ids.extend(emitted[b])
            self.reqs[b].output_ids.extend(emitted[b])
            assert self.cache.num_tokens(b) == self.reqs[b].num_tokens - 1
        assert len(odd) <= 1, odd
        assert self.dec.draft_cache.allocator.num_free >= 0
        from microserve_b200 import _lib

        assert _lib.device_error() == 0
        return {"accepted": sum(len(e) - 1 for e in emitted), "entropy": entropy}


LLAMA_1B = dict(vocab_size=32000, n_layers=2, d_model=2048, n_heads=32, n_kv_heads=4, d_ff=5632,
                rope_theta=10000.0, max_seq_len=4096)
LLAMA_8B = dict(vocab_size=128256, n_layers=2, d_model=4096, n_heads=32, n_kv_heads=8,
                d_ff=14336, rope_theta=500000.0, max_seq_len=8192)
DRAFT_8B = dict(vocab_size=128256, n_layers=2, d_model=2048, n_heads=32, n_kv_heads=8, d_ff=8192,
                rope_theta=500000.0, max_seq_len=8192)


@pytest.mark.parametrize("mode", ["sampled", "greedy"])
def test_config3_shape_rounds_match_oracle(mode: str) -> None:
    """Llama-1.1B widths (d 2048, 32/4 heads of 64, SwiGLU 5632, vocab 32000,
    RoPE 1e4), 2 target layers and the 2-layer draft, 16 requests with
    contexts uniform in [512, 2048], block 16, gamma 4, temperature 0.8 and
    top-p 0.9 (or greedy): two rounds, logits and decisions against the oracle."""
    from microserve_b200.config import SamplingConfig

    sc = (SamplingConfig(temperature=0.8, top_p=0.9, max_new_tokens=1 << 20) if mode == "sampled"
          else SamplingConfig(temperature=0.0, max_new_tokens=1 << 20))
    ctx = np.random.default_rng(31).integers(512, 2049, 16).tolist()
    s = _Setup(LLAMA_1B, dict(LLAMA_1B, n_layers=2), 4, ctx, 20.0, sc, 31)
    stats = [s.round(4) for _ in range(2)]
    if mode == "sampled":
        ent = np.concatenate([st["entropy"] for st in stats])
        assert ent.mean() > 0.5, "target rows are near one-hot: the sampled check is vacuous"


@pytest.mark.parametrize("mode", ["sampled", "greedy"])
def test_config4_shape_rounds_match_oracle(mode: str) -> None:
    """Llama-3-8B widths (d 4096, 32/8 heads of 128, SwiGLU 14336, vocab 128256,
    RoPE 5e5; 2 layers) with a 1B-class draft at its widths (d 2048, 32/8
    heads of 64, SwiGLU 8192; 2 layers), 8 requests with contexts up to 2048,
    gamma 5, temperature 0.8 and top-p 0.9 (thread-block-cluster samplers at
    this vocabulary) or greedy: two rounds against the oracle."""
    from microserve_b200.config import SamplingConfig

    sc = (SamplingConfig(temperature=0.8, top_p=0.9, max_new_tokens=1 << 20) if mode == "sampled"
          else SamplingConfig(temperature=0.0, max_new_tokens=1 << 20))
    ctx = [2048, 1500, 64, 700, 1999, 9, 1024, 333]
    s = _Setup(LLAMA_8B, DRAFT_8B, 5, ctx, 20.0, sc, 47)
    stats = [s.round(5) for _ in range(2)]
    if mode == "sampled":
        ent = np.concatenate([st["entropy"] for st in stats])
        assert ent.mean() > 0.5, "target rows are near one-hot: the sampled check is vacuous"


def test_sampling_filters_at_128256_are_not_degenerate() -> None:
    """Guard for the check above: the oracle's top-p filter keeps many tokens
    on logits with the spread the 8B-shape rounds produce."""
    rng = np.random.default_rng(0)
    row = filter_row((rng.standard_normal(128256) * 2).astype(np.float32), 0.8, None, 0.9)
    assert (row.e > 0).sum() > 100


@pytest.mark.parametrize("temperature", [0.0, 0.8])
def test_chunked_prefill_keeps_the_streams(temperature: float) -> None:
    """Config-0 models and workload with SchedulerConfig.prefill_chunk = 24:
    prompts of 8-256 tokens are prefilled over several engine steps, mixed
    with other requests' decode steps.  Greedy: every request's tokens equal
    those of the unchunked engine.  Sampled: the first token (drawn when the
    prompt is complete, on the request's first round counter) is the same;
    later draws depend on which steps were speculative rounds, which the
    different schedules change."""
    from microserve_b200.config import (CacheConfig, EngineConfig, SamplingConfig,
                                        SchedulerConfig, SpeculativeConfig)
    from microserve_b200.engine import LLMEngine

    target, draft, _, _ = _char_models(20.0)
    w = _wl().config0()
    outs = []
    for chunk in (None, 24):
        cfg = EngineConfig(model=target.cfg, cache=CacheConfig(block_size=16, num_blocks=256),
                           scheduler=SchedulerConfig(max_batch_size=8, max_batched_tokens=96,
                                                     prefill_chunk=chunk),
                           speculative=SpeculativeConfig(enabled=True, gamma=3))
        eng = LLMEngine(target, cfg, draft_model=draft)
        sc = SamplingConfig(temperature=temperature, max_new_tokens=20)
        reqs = [eng.add_request(p, sc) for p in w.prompts]
        done = {o.request_id: o.output_ids for o in eng.run()}
        outs.append([done[r.request_id] for r in reqs])
        if chunk is not None:
            assert eng.stats.num_steps > 8  # the prompts really took several steps
    if temperature == 0.0:
        assert outs[0] == outs[1]
    else:
        assert [o[0] for o in outs[0]] == [o[0] for o in outs[1]]
