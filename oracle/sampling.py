"""Sampling and accept/reject restated in numpy -- test infrastructure (checker only).

Follows reference src/microserve/sampling.py and speculative.py line by line,
except that draws are inverse-CDF lookups on explicit uniforms:

* ``filter_row``    -- apply_temperature / apply_top_k / apply_top_p
                       (sampling.py:17-51), then softmax (sampling.py:74);
* ``draw``          -- replaces torch.multinomial (sampling.py:77-81): the
                       first index whose float64 running sum of the weights
                       exceeds u * total;
* ``verify``        -- verify_proposals (speculative.py:44-86) with the roll
                       ``torch.rand`` replaced by ``u_accept[i]``.

Greedy (temperature 0) is the one-hot distribution at the first argmax
(sampling.py:64-71).
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

F32 = np.float32


@dataclass
class Row:
    """A processed row: unnormalised weights ``e`` (0 where filtered) and their sum."""

    e: np.ndarray  # float32 (V,)
    z: float
    onehot: int | None = None

    @property
    def probs(self) -> np.ndarray:
        if self.onehot is not None:
            p = np.zeros_like(self.e)
            p[self.onehot] = 1.0
            return p
        return (self.e / F32(self.z)).astype(F32)


def filter_row(logits: np.ndarray, temperature: float, top_k: int | None, top_p: float | None) -> Row:
    """probs_from_logits for one row (reference sampling.py:17-74)."""
    logits = np.asarray(logits, dtype=F32)
    V = logits.shape[-1]
    if temperature == 0.0:
        am = int(np.argmax(logits))  # first maximum, as torch.argmax
        e = np.zeros(V, F32)
        e[am] = 1.0
        return Row(e, 1.0, onehot=am)
    # apply_temperature: identity at 1.0, else a float32 divide (sampling.py:17-22)
    x = logits if temperature == 1.0 else (logits / F32(temperature)).astype(F32)
    keep = np.ones(V, dtype=bool)
    # apply_top_k: threshold at the k-th largest, keep >= (ties keep more) (sampling.py:25-31)
    if top_k is not None and top_k < V:
        kth = np.partition(x, V - top_k)[V - top_k]
        keep &= x >= kth
    m = F32(x[keep].max())
    e = np.where(keep, np.exp((x - m).astype(F32)), F32(0)).astype(F32)
    # apply_top_p on the top-k-masked row (sampling.py:34-51): sort descending,
    # softmax, cumsum, drop where the preceding mass already reached top_p,
    # always keep the first.
    if top_p is not None and top_p < 1.0:
        z = np.float64(e.sum(dtype=np.float64))
        p = (e / F32(z)).astype(F32)
        idx = np.nonzero(keep)[0]
        order = idx[np.argsort(-x[idx], kind="stable")]
        ps = p[order]
        cum = np.cumsum(ps, dtype=np.float64)
        prev = cum - ps.astype(np.float64)
        remove = prev >= top_p
        remove[0] = False
        keep = np.zeros(V, dtype=bool)
        keep[order[~remove]] = True
        e = np.where(keep, e, F32(0)).astype(F32)
    return Row(e, float(e.sum(dtype=np.float64)))


def draw(weights: np.ndarray, u: float) -> int:
    """Inverse CDF in vocabulary order (stands in for torch.multinomial)."""
    w = np.asarray(weights, dtype=F32)
    c = np.cumsum(w, dtype=np.float64)
    t = np.float64(F32(u)) * c[-1]
    i = int(np.searchsorted(c, t, side="right"))
    if i >= len(w):
        pos = np.nonzero(w > 0)[0]
        i = int(pos[-1]) if pos.size else 0
    return i


def sample_row(logits: np.ndarray, temperature: float, top_k: int | None, top_p: float | None,
               u: float) -> tuple[int, Row]:
    """sample() for one row (reference sampling.py:84-92): greedy -> argmax."""
    row = filter_row(logits, temperature, top_k, top_p)
    if row.onehot is not None:
        return row.onehot, row
    return draw(row.e, u), row


def verify(
    p_rows: list[Row],
    q_rows: list[Row],
    proposals: list[int],
    u_accept: np.ndarray,
    u_draw: float,
) -> tuple[list[int], int]:
    """verify_proposals (reference speculative.py:44-86) with explicit uniforms.

    Returns (emitted tokens, number accepted).
    """
    gamma = len(proposals)
    if len(q_rows) != gamma or len(p_rows) != gamma + 1:
        raise ValueError("probability tensors do not match the proposal length")
    accepted: list[int] = []
    for i, x in enumerate(proposals):
        p = p_rows[i].probs
        q = q_rows[i].probs
        ratio = min(F32(p[x]) / max(F32(q[x]), F32(1e-10)), F32(1.0))
        if F32(u_accept[i]) < ratio:
            accepted.append(int(x))
            continue
        r = np.maximum(p - q, F32(0)).astype(F32)
        if float(r.sum(dtype=np.float64)) <= 1e-9:
            r = p
        return [*accepted, draw(r, u_draw)], len(accepted)
    last = p_rows[gamma]
    bonus = last.onehot if last.onehot is not None else draw(last.e, u_draw)
    return [*accepted, bonus], gamma


def verify_probs(p: np.ndarray, q: np.ndarray, proposals: list[int], u_accept: np.ndarray,
                 u_draw: float) -> tuple[list[int], int]:
    """verify() on raw probability rows (the verify_proposals API)."""
    prow = [Row(np.asarray(r, F32), float(np.sum(r, dtype=np.float64))) for r in p]
    qrow = [Row(np.asarray(r, F32), float(np.sum(r, dtype=np.float64))) for r in q]
    # probabilities are used as given (no renormalisation), as the reference does
    for r in prow + qrow:
        r.z = 1.0
    return verify(prow, qrow, proposals, u_accept, u_draw)


def near_boundary(row: Row, u: float, tol: float = 1e-5) -> bool:
    """True when u*total lies within tol (relative) of a CDF step of the row:
    such draws may legitimately differ between float orders of summation."""
    if row.onehot is not None:
        return False
    c = np.cumsum(row.e, dtype=np.float64)
    t = np.float64(u) * c[-1]
    return bool(np.min(np.abs(c - t)) <= tol * max(c[-1], 1e-30))
