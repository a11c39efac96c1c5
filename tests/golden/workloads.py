"""Seeded synthetic workloads and random-init weights shared by the fixture
generator (``make_golden.py``, which runs them through the reference) and the
tests (which regenerate the same inputs on the GPU box and compare).

Everything is drawn with numpy's ``default_rng`` (PCG64), whose streams are
the same on every platform, so nothing but the reference's outputs has to be
stored.  Shapes follow the benchmark configurations:

* config 0: a character-level target (vocab 65, d_model 128, 4 layers, 4
  heads, SwiGLU 352) and draft (d_model 64, 2 layers, 2 heads, SwiGLU 176);
  8 requests, prompt ids uniform over the vocabulary, prompt lengths
  lognormal with mean 100 (std 50) clipped to [8, 256], 50 new tokens;
* config 2: the same models; prompt lengths lognormal mean 100 std 50
  clipped to [8, 512], output budgets uniform over 1..50.

The weight recipe is the reference's initialisation (model.py:279-299):
N(0, 0.02) for embeddings and projections, N(0, 0.02/sqrt(2L)) for o_proj
and down_proj, ones for the norms.  ``amplify`` scales o_proj and down_proj
as the reference's test fixture does (tests/conftest.py:41-56): fresh
models all predict "repeat the last token", which makes greedy agreement
vacuous.  Prompt lengths use the reference benchmark's lognormal
parameterisation (scripts/benchmark.py:81-85): linear mean and std given,
clipped, then truncated to int.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np

VOCAB_CHAR = 65


@dataclass(frozen=True)
class Shape:
    vocab_size: int
    n_layers: int
    d_model: int
    n_heads: int
    n_kv_heads: int
    d_ff: int
    max_seq_len: int = 1024
    rope_theta: float = 10_000.0

    @property
    def d_head(self) -> int:
        return self.d_model // self.n_heads


CHAR_TARGET = Shape(VOCAB_CHAR, 4, 128, 4, 4, 352, max_seq_len=1024)
CHAR_DRAFT = Shape(VOCAB_CHAR, 2, 64, 2, 2, 176, max_seq_len=1024)


def init_state(shape: Shape, seed: int, amplify: float = 1.0,
               std: float = 0.02) -> dict[str, np.ndarray]:
    """A reference-format float32 state dict with the reference's init rule."""
    rng = np.random.default_rng(seed)
    d, hq, hkv, dh, ff, L = (shape.d_model, shape.n_heads, shape.n_kv_heads, shape.d_head,
                             shape.d_ff, shape.n_layers)
    res = std / math.sqrt(2 * L)

    def normal(rows: int, cols: int, s: float) -> np.ndarray:
        return (rng.standard_normal((rows, cols), dtype=np.float32) * np.float32(s))

    st: dict[str, np.ndarray] = {"embed.weight": normal(shape.vocab_size, d, std)}
    for i in range(L):
        p = f"blocks.{i}."
        st[p + "attn.q_proj.weight"] = normal(hq * dh, d, std)
        st[p + "attn.k_proj.weight"] = normal(hkv * dh, d, std)
        st[p + "attn.v_proj.weight"] = normal(hkv * dh, d, std)
        st[p + "attn.o_proj.weight"] = normal(d, hq * dh, res) * np.float32(amplify)
        st[p + "ffn.gate_proj.weight"] = normal(ff, d, std)
        st[p + "ffn.up_proj.weight"] = normal(ff, d, std)
        st[p + "ffn.down_proj.weight"] = normal(d, ff, res) * np.float32(amplify)
        st[p + "attn_norm.weight"] = np.ones(d, np.float32)
        st[p + "ffn_norm.weight"] = np.ones(d, np.float32)
    st["norm.weight"] = np.ones(d, np.float32)
    st["lm_head.weight"] = st["embed.weight"]
    return st


def lognormal_lengths(rng: np.random.Generator, n: int, mean: float, std: float, lo: int,
                      hi: int) -> np.ndarray:
    """Lengths whose linear mean and std are ``mean``/``std``, clipped to
    [lo, hi] and truncated to int."""
    var = math.log(1.0 + (std / mean) ** 2)
    mu = math.log(mean) - var / 2.0
    raw = np.exp(rng.standard_normal(n) * math.sqrt(var) + mu)
    return np.clip(raw, lo, hi).astype(np.int64)


@dataclass
class Workload:
    prompts: list[list[int]]
    max_new_tokens: list[int]


def config0(seed: int = 0) -> Workload:
    """8 requests, prompt lengths lognormal(100, 50) in [8, 256], 50 new tokens."""
    rng = np.random.default_rng(seed + 1000)
    lens = lognormal_lengths(rng, 8, 100.0, 50.0, 8, 256)
    prompts = [rng.integers(0, VOCAB_CHAR, int(n)).tolist() for n in lens]
    return Workload(prompts, [50] * 8)


def config2(n: int, seed: int = 0) -> Workload:
    """``n`` requests, prompt lengths lognormal(100, 50) in [8, 512], outputs U{1..50}."""
    rng = np.random.default_rng(seed + 2000)
    lens = lognormal_lengths(rng, n, 100.0, 50.0, 8, 512)
    outs = rng.integers(1, 51, n)
    prompts = [rng.integers(0, VOCAB_CHAR, int(k)).tolist() for k in lens]
    return Workload(prompts, [int(o) for o in outs])


SCHEDULER_CASES = [  # (policy, batching, tokens_per_step, num_blocks, max_batch, max_tokens)
    ("fcfs", "continuous", 1, 40, 8, 96),
    ("sjf", "continuous", 1, 40, 8, 96),
    ("lifo", "continuous", 4, 40, 6, 64),
    ("fcfs", "static", 1, 60, 5, 200),
    ("fcfs", "continuous", 6, 24, 8, 2048),
]


def scheduler_trace(Request, Scheduler, SamplingConfig, SchedulerConfig, cache, case,
                    seed: int = 0, steps: int = 120) -> list[list[int]]:
    """Drive a scheduler through a synthetic serving run under memory
    pressure and record its decisions.

    Works with any implementation of the reference's scheduler API (the
    same calls are made on both sides).  Each step: ``schedule``; every
    scheduled request has its uncomputed tokens appended to the cache (block
    size 4) and then gains 1..tokens_per_step generated tokens; requests that
    reach their budget finish; new requests arrive now and then.  Returns one
    record per step: ``[n_scheduled, *scheduled ids, n_preempted, *preempted
    ids, total_preemptions]``.
    """
    policy, batching, tps, _, max_batch, max_tokens = case
    sched = Scheduler(SchedulerConfig(policy=policy, batching=batching, max_batch_size=max_batch,
                                      max_batched_tokens=max_tokens), cache)
    sched.tokens_per_step = tps
    rng = np.random.default_rng(seed)
    next_id = 0
    records: list[list[int]] = []

    def arrive(now: float) -> None:
        nonlocal next_id
        n = int(rng.integers(1, 30))
        sc = SamplingConfig(max_new_tokens=int(rng.integers(1, 25)))
        sched.add(Request(next_id, [int(t) for t in rng.integers(0, 50, n)], sc,
                          arrival_time=now + float(rng.random())))
        next_id += 1

    for _ in range(6):
        arrive(0.0)
    for step in range(steps):
        now = float(step)
        if rng.random() < 0.35:
            arrive(now)
        plan = sched.schedule(now)
        records.append([len(plan.scheduled), *[r.request_id for r in plan.scheduled],
                        len(plan.preempted), *[r.request_id for r in plan.preempted],
                        sched.total_preemptions])
        for r in plan.scheduled:
            n = r.num_uncomputed
            if n > 0 and cache.blocks_needed(r.request_id, n) <= cache.num_free_blocks:
                cache.append(r.request_id, n)
                r.num_computed += n
            gained = int(rng.integers(1, tps + 1))
            for _ in range(gained):
                if r.should_stop():
                    break
                r.output_ids.append(int(rng.integers(0, 50)))
            if r.should_stop():
                sched.finish(r, now)
        if not sched.waiting and not sched.running:
            break
    return records
