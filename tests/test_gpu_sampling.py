"""Device sampling kernels (ms_sample, ms_spec_accept, ms_verify_probs) against the oracle."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import philox
from oracle.sampling import Row, draw, filter_row, near_boundary, sample_row, verify

from .spec_check import RequestRound, explain

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _lib():
    from microserve_b200 import _lib

    return _lib


def _params(cfgs: list[tuple[float, int | None, float | None]], seeds, steps) -> torch.Tensor:
    from microserve_b200.config import SamplingConfig
    from microserve_b200.sampling import make_params, params_to_device

    sc = [SamplingConfig(temperature=t, top_k=k, top_p=p) for t, k, p in cfgs]
    return params_to_device(make_params(sc, seeds, steps), torch.device(DEV))


def test_philox_device_matches_oracle() -> None:
    from microserve_b200.speculative import _u64_tensor

    L = _lib()
    n = 4096
    seeds = np.arange(n, dtype=np.uint64) * np.uint64(0x9E3779B97F4A7C15)
    steps = np.arange(n, dtype=np.uint64) * np.uint64(7) + np.uint64(1 << 40)
    ds, dst = _u64_tensor(seeds.tolist(), torch.device(DEV)), _u64_tensor(steps.tolist(), torch.device(DEV))
    for lane in (0, 3, 64, 128):
        out = torch.empty(n, dtype=torch.float32, device=DEV)
        L.call("ms_philox_uniforms", ds.data_ptr(), dst.data_ptr(), n, lane, out.data_ptr(),
               L.stream_ptr())
        want = philox.uniform(seeds, steps, lane)
        assert np.array_equal(out.cpu().numpy(), want)


SETTINGS = [(1.0, None, None), (0.8, None, None), (1.0, 5, None), (1.0, None, 0.9),
            (0.7, 5, 0.9), (1.3, None, 0.5), (1.0, 50, 0.9), (0.0, None, None)]


@pytest.mark.parametrize("vocab", [65, 1000, 32000, 50000, 128256])
def test_sample_distribution_and_draws_match_oracle(vocab: int) -> None:
    L = _lib()
    rng = np.random.default_rng(vocab)
    rows = 24
    logits = (rng.standard_normal((rows, vocab)) * 2.0).astype(np.float32)
    dl = torch.from_numpy(logits).to(DEV)
    mismatches = 0
    for si, (t, k, p) in enumerate(SETTINGS):
        seeds = [1000 + r for r in range(rows)]
        steps = [si] * rows
        params = _params([(t, k, p)] * rows, seeds, steps)
        toks = torch.empty(rows, dtype=torch.int32, device=DEV)
        probs = torch.empty((rows, vocab), dtype=torch.float32, device=DEV)
        L.call("ms_sample", dl.data_ptr(), vocab, rows, vocab, params.data_ptr(), None, 3,
               toks.data_ptr(), probs.data_ptr(), None, None, None, L.stream_ptr())
        got_p = probs.cpu().numpy()
        got_t = toks.cpu().numpy()
        for r in range(rows):
            u = float(philox.uniform(seeds[r], steps[r], 3))
            tok, row = sample_row(logits[r], t, k, p, u)
            np.testing.assert_allclose(got_p[r], row.probs, rtol=2e-5, atol=1e-7)
            if got_t[r] != tok:
                assert near_boundary(row, u), (vocab, si, r, got_t[r], tok)
                mismatches += 1
    assert mismatches <= 1


def _ties_kept(logits: np.ndarray, t: float, p, u: float):
    """The oracle row with every value equal to its top-p cut kept: the kernels
    keep x >= cut, where the reference's sort keeps a prefix of the ties."""
    tok, row = sample_row(logits, t, None, p, u)
    if row.onehot is not None or p is None or p >= 1.0:
        return tok, row
    x = logits if t == 1.0 else (logits / np.float32(t)).astype(np.float32)
    cut = x[row.e > 0].min()
    e = np.where(x >= cut, np.exp((x - x.max()).astype(np.float32)), np.float32(0)).astype(np.float32)
    kept = Row(e, float(e.sum(dtype=np.float64)))
    return draw(e, u), kept


@pytest.mark.parametrize("vocab", [50000, 128256])
def test_sample_flat_and_tied_rows_match_oracle(vocab: int) -> None:
    """Rows whose top-p crossing bin is crowded: a narrow spread (second-level
    bins), all-equal and two-valued rows (more tied candidates than one
    cluster ranks: the single-CTA path), a spike over a flat floor.  Ties at
    the cut are all kept."""
    L = _lib()
    rng = np.random.default_rng(vocab + 1)
    rows = [rng.standard_normal(vocab) * 0.02, rng.standard_normal(vocab) * 0.002,
            np.zeros(vocab), np.where(rng.random(vocab) < 0.5, 1.0, 0.0),
            np.concatenate([[12.0], np.full(vocab - 1, -1.0)]),
            rng.standard_normal(vocab) * 0.3]
    logits = np.stack(rows).astype(np.float32)
    n = logits.shape[0]
    dl = torch.from_numpy(logits).to(DEV)
    mismatches = 0
    for si, (t, k, p) in enumerate([(1.0, None, 0.9), (0.7, None, 0.5), (1.0, None, 0.999),
                                    (1.0, None, None), (0.0, None, None)]):
        seeds = [77 + r for r in range(n)]
        steps = [si] * n
        params = _params([(t, k, p)] * n, seeds, steps)
        toks = torch.empty(n, dtype=torch.int32, device=DEV)
        probs = torch.empty((n, vocab), dtype=torch.float32, device=DEV)
        L.call("ms_sample", dl.data_ptr(), vocab, n, vocab, params.data_ptr(), None, 1,
               toks.data_ptr(), probs.data_ptr(), None, None, None, L.stream_ptr())
        got_p = probs.cpu().numpy()
        got_t = toks.cpu().numpy()
        for r in range(n):
            u = float(philox.uniform(seeds[r], steps[r], 1))
            tok, row = _ties_kept(logits[r], t, p, u)
            np.testing.assert_allclose(got_p[r], row.probs, rtol=2e-5, atol=1e-7)
            if got_t[r] != tok:
                assert near_boundary(row, u), (vocab, si, r, got_t[r], tok)
                mismatches += 1
    assert mismatches <= 1
    assert L.device_error() == 0


def test_greedy_ties_pick_first_index() -> None:
    L = _lib()
    logits = torch.tensor([[1.0, 3.0, 3.0, 0.0], [5.0, 5.0, 5.0, 5.0]], device=DEV)
    params = _params([(0.0, None, None)] * 2, [0, 0], [0, 0])
    toks = torch.empty(2, dtype=torch.int32, device=DEV)
    L.call("ms_sample", logits.data_ptr(), 4, 2, 4, params.data_ptr(), None, 0, toks.data_ptr(),
           None, None, None, None, L.stream_ptr())
    assert toks.tolist() == [1, 0]


def test_top_k_ties_keep_more_and_top_p_keeps_crossing_token() -> None:
    from microserve_b200.sampling import apply_top_k, apply_top_p

    x = torch.tensor([[1.0, 1.0, 1.0, 0.0]], device=DEV)
    assert int(torch.isfinite(apply_top_k(x, 2)).sum()) == 3
    logits = torch.tensor([[0.5, 0.3, 0.2]], device=DEV).log()
    out = apply_top_p(logits, 0.6)
    assert torch.isfinite(out[0, :2]).all() and out[0, 2] == float("-inf")
    one = apply_top_p(torch.tensor([[0.0, -100.0, -100.0]], device=DEV), 0.01)
    assert int(torch.isfinite(one).sum()) >= 1


def _accept_case(B: int, G: int, V: int, t: float, k, p, seed: int):
    rng = np.random.default_rng(seed)
    tl = (rng.standard_normal((B, G + 1, V)) * 2.0).astype(np.float32)
    dl = (tl[:, :G] + rng.standard_normal((B, G, V)) * 0.5).astype(np.float32)
    seeds = np.arange(B) + 1234
    steps = np.full(B, 7)
    # draft tokens sampled from q with the draft lanes, as the spec round does
    qrows = [[filter_row(dl[b, i], t, k, p) for i in range(G)] for b in range(B)]
    props = np.zeros((G, B), np.int32)
    for b in range(B):
        for i in range(G):
            u = float(philox.uniform(seeds[b], steps[b], i))
            props[i, b] = qrows[b][i].onehot if qrows[b][i].onehot is not None else draw(qrows[b][i].e, u)
    return tl, dl, seeds, steps, qrows, props


@pytest.mark.parametrize("setting,draft_mode,V", [
    *[(s, m, 4000) for s in [(1.0, None, None), (1.0, 50, None), (1.0, None, 0.9),
                             (0.8, 20, 0.95), (0.0, None, None)]
      for m in ("logits", "stats", "probs")],
    *[(s, "stats", 32000) for s in [(1.0, 50, None), (1.0, None, 0.9), (0.8, 50, 0.9),
                                    (0.8, None, 0.9), (0.0, None, None), (1.3, None, None)]],
    *[(s, "stats", 100000) for s in [(0.8, None, 0.9), (0.0, None, None), (1.0, 50, None)]],
])
def test_spec_accept_matches_oracle(setting, draft_mode: str, V: int) -> None:
    """config-1-shaped (rows x gamma=5 x vocab) at a reduced row count."""
    L = _lib()
    t, k, p = setting
    B, G = (48, 5) if V <= 32000 else (24, 5)
    tl, dl, seeds, steps, qrows, props = _accept_case(B, G, V, t, k, p, 99)
    params = _params([(t, k, p)] * B, seeds.tolist(), steps.tolist())
    d_tl = torch.from_numpy(tl.reshape(B * (G + 1), V)).to(DEV)
    d_dl = torch.from_numpy(np.ascontiguousarray(dl.transpose(1, 0, 2)).reshape(G * B, V)).to(DEV)
    d_props = torch.from_numpy(props).to(DEV)
    stats = None
    draft_rows, mode = d_dl, 0
    if draft_mode == "stats":
        stats = torch.empty((G * B, 4), dtype=torch.int32, device=DEV)
        tok = torch.empty(G * B, dtype=torch.int32, device=DEV)
        pidx = torch.arange(G * B, device=DEV, dtype=torch.int32) % B
        L.call("ms_sample", d_dl.data_ptr(), V, G * B, V, params.data_ptr(), pidx.data_ptr(), 0,
               tok.data_ptr(), None, stats.data_ptr(), None, None, L.stream_ptr())
    elif draft_mode == "probs":
        qp = np.stack([[qrows[b][i].probs for b in range(B)] for i in range(G)]).reshape(G * B, V)
        draft_rows, mode = torch.from_numpy(qp.astype(np.float32)).to(DEV), 1
    out = torch.empty(B * (G + 1), dtype=torch.int32, device=DEV)
    nacc = torch.empty(B, dtype=torch.int32, device=DEV)
    L.call("ms_spec_accept", d_tl.data_ptr(), V, draft_rows.data_ptr(), V, L.ptr(stats), mode,
           d_props.data_ptr(), params.data_ptr(), B, G, V, out.data_ptr(), nacc.data_ptr(),
           L.stream_ptr())
    got_tok = out.cpu().numpy().reshape(B, G + 1)
    got_n = nacc.cpu().numpy()
    odd = {}
    for b in range(B):
        prow = [filter_row(tl[b, i], t, k, p) for i in range(G + 1)]
        ua = philox.uniform(seeds[b], steps[b], 64 + np.arange(G))
        ud = float(philox.uniform(seeds[b], steps[b], 128))
        toks, n = verify(prow, qrows[b], props[:, b].tolist(), ua, ud)
        got = got_tok[b, : got_n[b] + 1].tolist()
        if got != toks:
            # allowed only at a decision boundary: |u - p/q| < 1e-5 or a draw
            # within float rounding of a CDF step (same logits on both sides)
            rr = RequestRound(int(seeds[b]), int(steps[b]), qrows[b], prow,
                              props[:, b].tolist(), toks, n)
            why = explain(rr, props[:, b].tolist(), got, tol=1e-5)
            assert why is not None, (b, got, toks)
            odd[b] = why
    assert len(odd) <= 1, odd


def test_verify_proposals_api_cases() -> None:
    from microserve_b200.speculative import verify_proposals

    r = verify_proposals(torch.tensor([[0.5, 0.5]]), torch.tensor([[1.0, 0.0], [1.0, 0.0]]), [0],
                         torch.Generator().manual_seed(0))
    assert r.num_accepted == 1 and r.tokens[0] == 0
    r = verify_proposals(torch.tensor([[0.0, 1.0]]), torch.tensor([[1.0, 0.0], [1.0, 0.0]]), [1],
                         torch.Generator().manual_seed(0))
    assert r.num_accepted == 0 and r.tokens == [0]
    with pytest.raises(ValueError, match="do not match"):
        verify_proposals(torch.ones(2, 4) / 4, torch.ones(2, 4) / 4, [0, 1])
    gen = torch.Generator().manual_seed(0)
    probs = torch.rand(8, generator=gen) + 1e-3
    probs /= probs.sum()
    for _ in range(10):
        r = verify_proposals(probs.repeat(3, 1), probs.repeat(4, 1), [0, 1, 2], gen)
        assert r.num_accepted == 3 and len(r.tokens) == 4


def test_emitted_token_follows_the_target_chi_square() -> None:
    """gamma=1 over many requests: the emitted token is distributed as p_target
    (reference test_speculative.py:88-114, on the device kernel)."""
    from scipy.stats import chisquare

    L = _lib()
    V, B = 8, 30000
    rng = np.random.default_rng(5)
    q = rng.random(V) + 1e-3
    q /= q.sum()
    pt = rng.random(V) + 1e-3
    pt /= pt.sum()
    tl = np.log(np.tile(pt, (B, 2, 1))).astype(np.float32).reshape(B * 2, V)
    dl = np.log(np.tile(q, (B, 1))).astype(np.float32)
    seeds = np.arange(B) + 77
    params = _params([(1.0, None, None)] * B, seeds.tolist(), [0] * B)
    d_dl = torch.from_numpy(dl).to(DEV)
    props = torch.empty(B, dtype=torch.int32, device=DEV)
    stats = torch.empty((B, 4), dtype=torch.int32, device=DEV)
    L.call("ms_sample", d_dl.data_ptr(), V, B, V, params.data_ptr(), None, 0, props.data_ptr(),
           None, stats.data_ptr(), None, None, L.stream_ptr())
    out = torch.empty(B * 2, dtype=torch.int32, device=DEV)
    nacc = torch.empty(B, dtype=torch.int32, device=DEV)
    d_tl = torch.from_numpy(tl).to(DEV)
    L.call("ms_spec_accept", d_tl.data_ptr(), V, d_dl.data_ptr(), V, stats.data_ptr(), 0,
           props.data_ptr(), params.data_ptr(), B, 1, V, out.data_ptr(), nacc.data_ptr(),
           L.stream_ptr())
    first = out.cpu().numpy().reshape(B, 2)[:, 0]
    counts = np.bincount(first, minlength=V)
    expected = pt / pt.sum() * B
    assert chisquare(counts, expected).pvalue > 0.01
    # negative control: the draft's own proposals are visibly biased
    biased = np.bincount(props.cpu().numpy(), minlength=V)
    assert chisquare(biased, expected).pvalue < 0.01
