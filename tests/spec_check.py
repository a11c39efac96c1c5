"""Checks of device speculative rounds against the oracle (test helpers).

A sampled decision of the device may legitimately differ from the oracle's
only where the shared uniform sits at a decision boundary, within float
rounding of the two computations:

* a draw (draft proposal, residual resample, bonus token) whose ``u * total``
  lies within ``tol`` (relative) of a step of the row's CDF;
* an accept roll with ``|u - min(1, p(x)/q(x))| < tol``
  (reference speculative.py:62-85).

``explain`` finds, for a request whose emitted tokens differ, a boundary
case at or before the first differing position, and the tests assert that
every differing request has one.  ``tol`` is 1e-5 where the device and the
oracle sample from the same logits, and the logit tolerance of the
comparison (1e-4 in float32) where each side computes its own logits.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from oracle import philox
from oracle.model import SeqKV
from oracle.sampling import Row, draw, filter_row, near_boundary, verify
from oracle.spec import LANE_ACCEPT, LANE_RESAMPLE

F32 = np.float32


def pool_history(cache, seq_id: int, n: int) -> SeqKV:
    """The first ``n`` tokens' K/V of ``seq_id``, read out of the device pool
    with plain torch indexing through the host block table (no library call)."""
    pool = cache.pool
    _, L, _, hkv, bs, dh = pool.shape
    nb = -(-n // bs)
    blocks = torch.tensor(cache.tables[seq_id].blocks[:nb], device=pool.device, dtype=torch.long)
    sel = pool.index_select(2, blocks)  # (2, L, nb, hkv, bs, dh)
    sel = sel.permute(0, 1, 2, 4, 3, 5).reshape(2, L, nb * bs, hkv, dh)[:, :, :n]
    arr = sel.float().cpu().numpy()
    return SeqKV(k=[np.ascontiguousarray(arr[0, i]) for i in range(L)],
                 v=[np.ascontiguousarray(arr[1, i]) for i in range(L)])


@dataclass
class RequestRound:
    """One request's side of a round, as the oracle decides it."""

    seed: int
    step: int
    q_rows: list[Row]
    p_rows: list[Row]
    proposals: list[int]
    emitted: list[int]
    num_accepted: int


def _residual(p: Row, q: Row) -> Row:
    r = np.maximum(p.probs - q.probs, F32(0)).astype(F32)
    if float(r.sum(dtype=np.float64)) <= 1e-9:
        return p
    return Row(r, float(r.sum(dtype=np.float64)))


def explain(rr: RequestRound, got_proposals: list[int] | None, got_emitted: list[int],
            tol: float) -> str | None:
    """A boundary case that lets the device's decisions differ from ``rr``, or None."""
    G = len(rr.proposals)
    lim = G
    if got_proposals is not None:
        for j in range(G):
            if got_proposals[j] != rr.proposals[j]:
                lim = j
                break
    for i, (a, b) in enumerate(zip(got_emitted, rr.emitted)):
        if a != b:
            lim = min(lim, i)
            break
    else:
        lim = min(lim, min(len(got_emitted), len(rr.emitted)))
    lim = min(lim, G)
    u_draw = float(philox.uniform(rr.seed, rr.step, LANE_RESAMPLE))
    for j in range(lim + 1):
        if j < G:
            u = float(philox.uniform(rr.seed, rr.step, j))
            if near_boundary(rr.q_rows[j], u, tol):
                return f"draft draw {j} at a CDF step"
            x = rr.proposals[j]
            p, q = rr.p_rows[j].probs, rr.q_rows[j].probs
            ratio = min(float(p[x]) / max(float(q[x]), 1e-10), 1.0)
            ua = float(philox.uniform(rr.seed, rr.step, LANE_ACCEPT + j))
            if abs(ua - ratio) < tol * max(1.0, ratio):
                return f"accept roll {j}: |u - p/q| = {abs(ua - ratio):.2e}"
            if near_boundary(_residual(rr.p_rows[j], rr.q_rows[j]), u_draw, tol):
                return f"residual draw at {j} at a CDF step"
        elif near_boundary(rr.p_rows[G], u_draw, tol):
            return "bonus draw at a CDF step"
    return None


def decide(seed: int, step: int, draft_logits: np.ndarray, target_logits: np.ndarray,
           temperature: float, top_k: int | None, top_p: float | None,
           proposals: list[int] | None = None) -> RequestRound:
    """The oracle's decisions for one request given its logits: proposals drawn
    from the draft rows (or taken as given), then verify_proposals."""
    G = draft_logits.shape[0]
    q_rows = [filter_row(draft_logits[j], temperature, top_k, top_p) for j in range(G)]
    if proposals is None:
        proposals = []
        for j in range(G):
            u = float(philox.uniform(seed, step, j))
            r = q_rows[j]
            proposals.append(r.onehot if r.onehot is not None else draw(r.e, u))
    p_rows = [filter_row(target_logits[i], temperature, top_k, top_p) for i in range(G + 1)]
    ua = philox.uniform(seed, step, LANE_ACCEPT + np.arange(G))
    ud = float(philox.uniform(seed, step, LANE_RESAMPLE))
    toks, n = verify(p_rows, q_rows, list(proposals), ua, ud)
    return RequestRound(seed, step, q_rows, p_rows, list(proposals), toks, n)
