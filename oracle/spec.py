"""The speculative round restated on the CPU -- test infrastructure (checker only).

Follows reference src/microserve/speculative.py:115-226: the draft catches
up on the tokens it has not seen, proposes gamma tokens (probs_from_logits +
a draw per request per pass), the target scores
``all_ids[cached:] + proposals``, verify_proposals runs on the last gamma+1
rows, and both caches roll back to ``num_tokens + num_accepted`` (the draft
to at most that).  Draws use the Philox lanes of the device path: draft draw
j on lane j, accept roll i on lane 64+i, residual/bonus draw on lane 128, all
at the request's draw step, which advances by one per round.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

from . import philox
from .model import OracleModel, SeqKV
from .sampling import Row, filter_row, sample_row, verify

LANE_ACCEPT = 64
LANE_RESAMPLE = 128


@dataclass
class OracleRequest:
    request_id: int
    prompt_ids: list[int]
    temperature: float
    top_k: int | None
    top_p: float | None
    seed: int
    output_ids: list[int] = field(default_factory=list)
    step: int = 0
    target_kv: SeqKV = field(default_factory=SeqKV)
    draft_kv: SeqKV = field(default_factory=SeqKV)
    num_proposed: int = 0
    num_accepted: int = 0

    @property
    def all_ids(self) -> list[int]:
        return self.prompt_ids + self.output_ids


@dataclass
class RoundTrace:
    """What one round decided, for comparison with the device."""

    proposals: list[list[int]]
    num_accepted: list[int]
    emitted: list[list[int]]
    draft_rows: list[list[Row]]
    target_rows: list[list[Row]]


def spec_round(target: OracleModel, draft: OracleModel, gamma: int,
               reqs: list[OracleRequest]) -> RoundTrace:
    """One SpeculativeDecoder.step over ``reqs`` (emitted tokens are NOT appended)."""
    B = len(reqs)
    pending = [r.all_ids[r.draft_kv.length:] for r in reqs]
    proposals: list[list[int]] = [[] for _ in range(B)]
    qrows: list[list[Row]] = [[] for _ in range(B)]
    for j in range(gamma):
        last = [[len(p) - 1] for p in pending]
        logits = draft.forward(pending, [r.draft_kv for r in reqs], logit_rows=last)
        for b, r in enumerate(reqs):
            u = float(philox.uniform(r.seed, r.step, j))
            tok, row = sample_row(logits[b][0], r.temperature, r.top_k, r.top_p, u)
            proposals[b].append(tok)
            qrows[b].append(row)
        pending = [[p[-1]] for p in proposals]

    token_lists = [r.all_ids[r.target_kv.length:] + proposals[b] for b, r in enumerate(reqs)]
    windows = [[len(t) - (gamma + 1) + i for i in range(gamma + 1)] for t in token_lists]
    tlogits = target.forward(token_lists, [r.target_kv for r in reqs], logit_rows=windows)
    nacc: list[int] = []
    emitted: list[list[int]] = []
    prows: list[list[Row]] = []
    for b, r in enumerate(reqs):
        p = [filter_row(tlogits[b][i], r.temperature, r.top_k, r.top_p) for i in range(gamma + 1)]
        ua = philox.uniform(r.seed, r.step, LANE_ACCEPT + np.arange(gamma))
        ud = float(philox.uniform(r.seed, r.step, LANE_RESAMPLE))
        toks, n = verify(p, qrows[b], proposals[b], ua, ud)
        keep = len(r.all_ids) + n
        r.target_kv.truncate(keep)
        r.draft_kv.truncate(min(r.draft_kv.length, keep))
        r.step += 1
        r.num_proposed += gamma
        r.num_accepted += n
        nacc.append(n)
        emitted.append(toks)
        prows.append(p)
    return RoundTrace(proposals, nacc, emitted, qrows, prows)


def prefill(target: OracleModel, reqs: list[OracleRequest]) -> list[int]:
    """The engine's ordinary step for prompts (reference engine.py:204-220):
    prefill the target and sample one token per request on lane 0."""
    lists = [r.all_ids[r.target_kv.length:] for r in reqs]
    logits = target.forward(lists, [r.target_kv for r in reqs],
                            logit_rows=[[len(t) - 1] for t in lists])
    out = []
    for b, r in enumerate(reqs):
        u = float(philox.uniform(r.seed, r.step, 0))
        tok, _ = sample_row(logits[b][0], r.temperature, r.top_k, r.top_p, u)
        r.step += 1
        out.append(tok)
    return out
