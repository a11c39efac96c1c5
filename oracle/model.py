"""The transformer forward restated in numpy float32 -- test infrastructure (checker only).

Follows reference src/microserve/model.py: pre-norm RMSNorm (:69-79),
half-split RoPE with float32 cos/sin tables (:82-113), SwiGLU (:116-127),
causal attention where a query at absolute position p sees keys 0..p
(:185-222), tied lm_head (:277-278, :353).  Grouped-query attention (absent
from the reference) maps query head h to kv head h // (n_heads / n_kv_heads);
with the kv weights repeated per group this is exactly the reference's
multi-head layer.

The paged structure is not restated: each sequence's cache is its logical
K/V history (what ``PagedKVCache.gather`` materialises, cache.py:255-272),
so a batch forward equals the reference's ``forward_paged``.  GEMMs run on
the flattened rows of the whole batch, attention per sequence.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

F32 = np.float32


@dataclass
class Dims:
    vocab_size: int
    d_model: int
    n_layers: int
    n_heads: int
    n_kv_heads: int
    d_ff: int
    max_seq_len: int = 1024
    rope_theta: float = 10_000.0
    norm_eps: float = 1e-5

    @property
    def d_head(self) -> int:
        return self.d_model // self.n_heads


@dataclass
class SeqKV:
    """One sequence's logical K/V history: per layer (n, n_kv_heads, d_head)."""

    k: list[np.ndarray] = field(default_factory=list)
    v: list[np.ndarray] = field(default_factory=list)

    @property
    def length(self) -> int:
        return 0 if not self.k else int(self.k[0].shape[0])

    def truncate(self, n: int) -> None:
        self.k = [a[:n] for a in self.k]
        self.v = [a[:n] for a in self.v]


def rope_tables(d_head: int, max_seq_len: int, theta: float) -> tuple[np.ndarray, np.ndarray]:
    """cos/sin of outer(pos, 1/theta^(2i/d_head)) in float32 (reference model.py:92-98)."""
    inv_freq = (F32(1.0) / (F32(theta) ** (np.arange(0, d_head, 2, dtype=F32) / F32(d_head)))).astype(F32)
    pos = np.arange(max_seq_len, dtype=F32)
    ang = np.outer(pos, inv_freq).astype(F32)
    return np.cos(ang).astype(F32), np.sin(ang).astype(F32)


def rmsnorm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    ms = np.mean(x * x, axis=-1, keepdims=True, dtype=F32)
    return (x * (F32(1.0) / np.sqrt(ms + F32(eps))) * w).astype(F32)


def apply_rope(x: np.ndarray, cos: np.ndarray, sin: np.ndarray) -> np.ndarray:
    """x: (n, heads, d_head); cos/sin: (n, d_head/2)."""
    half = x.shape[-1] // 2
    x1, x2 = x[..., :half], x[..., half:]
    c, s = cos[:, None, :], sin[:, None, :]
    return np.concatenate([x1 * c - x2 * s, x2 * c + x1 * s], axis=-1).astype(F32)


class OracleModel:
    """float32 numpy model from a reference-format state dict."""

    def __init__(self, dims: Dims, state: dict[str, np.ndarray]) -> None:
        self.dims = dims
        g = lambda k: np.ascontiguousarray(np.asarray(state[k], dtype=F32))  # noqa: E731
        self.embed = g("embed.weight")
        self.norm = g("norm.weight")
        self.layers = []
        for i in range(dims.n_layers):
            p = f"blocks.{i}."
            self.layers.append({
                "attn_norm": g(p + "attn_norm.weight"),
                "wq": g(p + "attn.q_proj.weight"),
                "wk": g(p + "attn.k_proj.weight"),
                "wv": g(p + "attn.v_proj.weight"),
                "wo": g(p + "attn.o_proj.weight"),
                "ffn_norm": g(p + "ffn_norm.weight"),
                "wg": g(p + "ffn.gate_proj.weight"),
                "wu": g(p + "ffn.up_proj.weight"),
                "wd": g(p + "ffn.down_proj.weight"),
            })
        self.cos, self.sin = rope_tables(dims.d_head, dims.max_seq_len, dims.rope_theta)

    def forward(
        self,
        token_lists: list[list[int]],
        caches: list[SeqKV],
        logit_rows: list[list[int]] | None = None,
    ) -> list[np.ndarray]:
        """One flattened pass over several sequences; appends to their caches.

        Returns per sequence the float32 logits of the requested local rows
        (default: every new token).
        """
        d = self.dims
        hq, hkv, dh = d.n_heads, d.n_kv_heads, d.d_head
        group = hq // hkv
        lens = [len(t) for t in token_lists]
        starts = [c.length for c in caches]
        ids = np.asarray([t for ts in token_lists for t in ts], dtype=np.int64)
        pos = np.concatenate([np.arange(s, s + n) for s, n in zip(starts, lens, strict=True)])
        cos, sin = self.cos[pos], self.sin[pos]
        x = self.embed[ids].astype(F32)
        offs = np.concatenate([[0], np.cumsum(lens)])
        for li, L in enumerate(self.layers):
            h = rmsnorm(x, L["attn_norm"], d.norm_eps)
            q = (h @ L["wq"].T).reshape(-1, hq, dh)
            k = (h @ L["wk"].T).reshape(-1, hkv, dh)
            v = (h @ L["wv"].T).reshape(-1, hkv, dh)
            q = apply_rope(q, cos, sin)
            k = apply_rope(k, cos, sin)
            att = np.empty((len(ids), hq, dh), dtype=F32)
            for b, c in enumerate(caches):
                a, e = offs[b], offs[b + 1]
                if li == len(c.k):
                    c.k.append(np.zeros((0, hkv, dh), F32))
                    c.v.append(np.zeros((0, hkv, dh), F32))
                K = np.concatenate([c.k[li], k[a:e]], axis=0)
                Vv = np.concatenate([c.v[li], v[a:e]], axis=0)
                c.k[li], c.v[li] = K, Vv
                qb = q[a:e]  # (n, hq, dh)
                Kg = np.repeat(K, group, axis=1)  # (ctx, hq, dh)
                Vg = np.repeat(Vv, group, axis=1)
                scores = np.einsum("nhd,chd->hnc", qb, Kg).astype(F32) * F32(1.0 / np.sqrt(dh))
                qpos = pos[a:e]
                mask = np.arange(K.shape[0])[None, :] <= qpos[:, None]
                scores = np.where(mask[None], scores, -np.inf).astype(F32)
                scores -= scores.max(axis=-1, keepdims=True)
                pr = np.exp(scores).astype(F32)
                pr /= pr.sum(axis=-1, keepdims=True)
                att[a:e] = np.einsum("hnc,chd->nhd", pr, Vg).astype(F32)
            x = (x + att.reshape(len(ids), hq * dh) @ L["wo"].T).astype(F32)
            h2 = rmsnorm(x, L["ffn_norm"], d.norm_eps)
            gate = h2 @ L["wg"].T
            up = h2 @ L["wu"].T
            act = (gate / (F32(1.0) + np.exp(-gate))).astype(F32) * up
            x = (x + act @ L["wd"].T).astype(F32)
        out = []
        for b in range(len(caches)):
            a, e = offs[b], offs[b + 1]
            rows = list(range(e - a)) if logit_rows is None else logit_rows[b]
            xr = rmsnorm(x[a + np.asarray(rows, dtype=np.int64)], self.norm, d.norm_eps)
            out.append((xr @ self.embed.T).astype(F32))
        return out
