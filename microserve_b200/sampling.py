"""Logit post-processing and token sampling on the device.

Same functions as reference src/microserve/sampling.py (temperature ->
top-k -> top-p -> softmax; greedy as a one-hot distribution), computed by
``ms_sample`` in libmicroserve_b200 without sorting the vocabulary.

Randomness.  The reference draws with ``torch.multinomial`` from a CPU
``torch.Generator`` (mt19937), a stream no GPU kernel can reproduce.  Here
every draw is an inverse-CDF lookup with a Philox4x32-10 uniform keyed by
``(seed, step, lane)``: ``seed`` is the generator's ``initial_seed()``,
``step`` a counter and ``lane`` the draw's role.  The distribution drawn from
is identical; the individual draws differ from the reference's, which is
why sampled parity is checked against a restatement that takes the same
uniforms, plus a chi-square test against the reference itself.
"""

from __future__ import annotations

import numpy as np
import torch

from . import _lib
from .config import SamplingConfig

NEG_INF = float("-inf")


def make_params(
    cfgs: list[SamplingConfig], seeds: list[int] | np.ndarray, steps: list[int] | np.ndarray
) -> np.ndarray:
    """Host array of ``ms_sampling_params`` (one entry per request)."""
    p = np.zeros(len(cfgs), dtype=_lib.SAMPLING_PARAMS_DTYPE)
    p["temperature"] = [c.temperature for c in cfgs]
    p["top_p"] = [1.0 if c.top_p is None else c.top_p for c in cfgs]
    p["top_k"] = [0 if c.top_k is None else c.top_k for c in cfgs]
    p["seed"] = np.asarray(seeds, dtype=np.uint64)
    p["step"] = np.asarray(steps, dtype=np.uint64)
    return p


def validate(cfg: SamplingConfig) -> None:
    if cfg.temperature < 0.0:
        raise ValueError("temperature must be > 0; use greedy sampling instead")
    if cfg.top_k is not None and cfg.top_k <= 0:
        raise ValueError("top_k must be positive")
    if cfg.top_p is not None and not 0.0 < cfg.top_p <= 1.0:
        raise ValueError("top_p must be in (0, 1]")


def params_to_device(params: np.ndarray, device: torch.device) -> torch.Tensor:
    raw = torch.from_numpy(params.view(np.uint8).copy())
    return raw.to(device)


def generator_seed_and_step(generator: torch.Generator | None) -> tuple[int, int]:
    """Philox key and a fresh counter drawn from ``generator`` (advancing it)."""
    if generator is None:
        generator = torch.default_generator
    seed = int(generator.initial_seed()) & 0xFFFFFFFFFFFFFFFF
    dev = generator.device
    step = int(torch.randint(0, 2**62, (1,), generator=generator, device=dev).item())
    return seed, step


def _run_sample(
    logits: torch.Tensor,
    cfg: SamplingConfig,
    seed: int,
    step: int,
    want_probs: bool,
    want_stats: bool = False,
) -> tuple[torch.Tensor, torch.Tensor | None, np.ndarray | None]:
    validate(cfg)
    dev = _lib.require_cuda(logits.device)
    x = logits.to(torch.float32)
    squeeze = x.dim() == 1
    x = x.reshape(1, -1) if squeeze else x.reshape(-1, x.shape[-1])
    x = x.contiguous()
    rows, vocab = x.shape
    params = make_params([cfg] * rows, [seed] * rows, [step] * rows)
    dparams = params_to_device(params, dev)
    tokens = torch.empty(rows, dtype=torch.int32, device=dev)
    probs = torch.empty((rows, vocab), dtype=torch.float32, device=dev) if want_probs else None
    stats = torch.empty((rows, 4), dtype=torch.int32, device=dev) if want_stats else None
    _lib.call("ms_sample", x.data_ptr(), vocab, rows, vocab, dparams.data_ptr(), None,
              _lib.LANE_SAMPLE, tokens.data_ptr(), _lib.ptr(probs), _lib.ptr(stats), None, None,
              _lib.stream_ptr(dev))
    st = None
    if stats is not None:
        st = stats.cpu().numpy().view(_lib.ROW_STATS_DTYPE).reshape(-1)
    return tokens, probs, st


def apply_temperature(logits: torch.Tensor, temperature: float) -> torch.Tensor:
    if temperature <= 0.0:
        raise ValueError("temperature must be > 0; use greedy sampling instead")
    if temperature == 1.0:
        return logits
    return logits / temperature


def _mask_from_stats(x: torch.Tensor, stats: np.ndarray) -> torch.Tensor:
    thresh = torch.from_numpy(stats["thresh"].astype(np.float32)).to(x.device)
    keep = x >= thresh.view(-1, *([1] * (x.dim() - 1)))
    return x.masked_fill(~keep, NEG_INF)


def apply_top_k(logits: torch.Tensor, top_k: int) -> torch.Tensor:
    """Keep the ``top_k`` highest logits per row (ties keep more), mask the rest."""
    if top_k <= 0:
        raise ValueError("top_k must be positive")
    cfg = SamplingConfig(temperature=1.0, top_k=top_k)
    _, _, st = _run_sample(logits, cfg, 0, 0, want_probs=False, want_stats=True)
    assert st is not None
    x = logits.reshape(-1, logits.shape[-1]).float()
    return _mask_from_stats(x, st).reshape(logits.shape).to(logits.dtype)


def apply_top_p(logits: torch.Tensor, top_p: float) -> torch.Tensor:
    """Nucleus filter: the smallest descending prefix whose mass reaches ``top_p``
    (the crossing token is kept, so at least one token survives)."""
    if not 0.0 < top_p <= 1.0:
        raise ValueError("top_p must be in (0, 1]")
    if top_p == 1.0:
        return logits
    cfg = SamplingConfig(temperature=1.0, top_p=top_p)
    _, _, st = _run_sample(logits, cfg, 0, 0, want_probs=False, want_stats=True)
    assert st is not None
    x = logits.reshape(-1, logits.shape[-1]).float()
    return _mask_from_stats(x, st).reshape(logits.shape).to(logits.dtype)


def process_logits(logits: torch.Tensor, cfg: SamplingConfig) -> torch.Tensor:
    """Temperature, then top-k, then top-p (reference sampling.py:54-61)."""
    x = apply_temperature(logits, cfg.temperature)
    if cfg.top_k is None and cfg.top_p is None:
        return x
    c = SamplingConfig(temperature=1.0, top_k=cfg.top_k, top_p=cfg.top_p)
    _, _, st = _run_sample(x, c, 0, 0, want_probs=False, want_stats=True)
    assert st is not None
    xf = x.reshape(-1, x.shape[-1]).float()
    return _mask_from_stats(xf, st).reshape(x.shape).to(logits.dtype)


def probs_from_logits(logits: torch.Tensor, cfg: SamplingConfig) -> torch.Tensor:
    """The exact distribution a draw uses; greedy is one-hot (reference sampling.py:64-74)."""
    _, probs, _ = _run_sample(logits, cfg, 0, 0, want_probs=True)
    assert probs is not None
    return probs.reshape(logits.shape)


def sample_from_probs(probs: torch.Tensor, generator: torch.Generator | None = None) -> torch.Tensor:
    """Inverse-CDF draw per row of a probability tensor, returning ``(rows,)`` int64 ids.

    Implemented as a draw from ``log(probs)`` at temperature 1: the kernel's
    softmax of log-probabilities is the normalised ``probs``.
    """
    seed, step = generator_seed_and_step(generator)
    logp = torch.log(probs.float())
    tokens, _, _ = _run_sample(logp, SamplingConfig(temperature=1.0), seed, step, want_probs=False)
    return tokens.long()


def sample(
    logits: torch.Tensor, cfg: SamplingConfig, generator: torch.Generator | None = None
) -> torch.Tensor:
    """One token id per row of ``logits`` (reference sampling.py:84-92)."""
    if cfg.greedy:
        tokens, _, _ = _run_sample(logits, cfg, 0, 0, want_probs=False)
        return tokens.long().reshape(logits.shape[:-1])
    seed, step = generator_seed_and_step(generator)
    tokens, _, _ = _run_sample(logits, cfg, seed, step, want_probs=False)
    return tokens.long().reshape(logits.shape[:-1])
