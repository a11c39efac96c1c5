#!/usr/bin/env python
"""Throughput of the speculative-decoding step on B200.

Workload (the configuration the headline metric -- accepted tok/s per B200
at gamma=4 -- is quoted on): a Llama-style 1.1B bf16 target (d_model 2048,
22 layers, 32 query / 4 KV heads, SwiGLU 5632, vocab 32000, RoPE 1e4) with
a 2-layer draft of the same width, random-init weights (std 0.02); 256
requests per GPU with contexts uniform in [512, 2048] (token ids uniform
over the vocabulary, K/V pools filled with synthetic values), paged block
16, gamma = 4, temperature 0.8, top-p 0.9.  One step = one speculative
round over all requests (4 draft passes, one 5-token verify pass, fused
accept/resample, rollback).  The K timed rounds run as several timed regions
(``--repeats``, each after a fresh admission of the same contexts and a
warm-up), so that at least 200 rounds are measured by default.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

For N > 1 run under torchrun (one process per GPU); each rank serves its own
256 requests (weak scaling), there is no collective in the decode loop, and
the end-of-run counters are reduced over NCCL (SUM of tokens, MAX of time).

Reported: ``value`` = emitted tokens of all ranks / max over ranks of the
summed device time of the rounds' kernels (metadata already on the device);
``e2e`` = the same tokens / the time of the public ``SpeculativeDecoder.step``
calls including host bookkeeping, the pinned host->device metadata copies and
the device->host copy of the accepted tokens.  The GEMM roofline, the verify
step time and the attention rate come from further rounds of the same
workload after the timed ones, where CUDA events bracket every launch of the
kernel class (inside the timed rounds those events would cost ~1.1 ms a round).
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "accepted tok/s per B200 (spec γ=4)"
WORKLOAD = "llama-1.1b-bf16 target + 2-layer draft, 256 req/GPU, ctx U[512,2048], gamma 4, T 0.8, top-p 0.9"

TARGET = dict(vocab_size=32000, n_layers=22, d_model=2048, n_heads=32, n_kv_heads=4, d_ff=5632,
              rope_theta=10000.0)
DRAFT = dict(TARGET, n_layers=2)
GAMMA = 4
BLOCK = 16
MAX_SEQ = 4096
CTX_LOGNORMAL: tuple[float, float] | None = None  # (mean, std) of the context lengths

# --model 8b: the 8B-class workload (a Llama-3-8B-shape target with a 1B-class
# draft, 2048 requests over 8 GPUs = 256 per GPU, contexts lognormal with mean
# 2048 and std 1024 clipped to [8, 8192], gamma 5).  Not the headline metric.
TARGET_8B = dict(vocab_size=128256, n_layers=32, d_model=4096, n_heads=32, n_kv_heads=8,
                 d_ff=14336, rope_theta=500000.0)
DRAFT_8B = dict(vocab_size=128256, n_layers=16, d_model=2048, n_heads=32, n_kv_heads=8,
                d_ff=8192, rope_theta=500000.0)


def parse() -> argparse.Namespace:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--repeats", type=int, default=0,
                    help="timed regions of --steps rounds per wave, each after a fresh "
                         "admission and warm-up (0: enough for at least 200 timed rounds, at "
                         "most 20; 1 with --total-requests)")
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--requests", type=int, default=256, help="requests per GPU (weak scaling)")
    ap.add_argument("--total-requests", type=int, default=0,
                    help="strong scaling: one set of this many requests split over the GPUs, "
                         "served in waves of what fits in HBM")
    ap.add_argument("--ctx-min", type=int, default=512)
    ap.add_argument("--ctx-max", type=int, default=2048)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--cpu-requests", type=int, default=4,
                    help="cpu_baseline of the GPU arm: requests in the reference's sample")
    ap.add_argument("--cpu-requests-ref", type=int, default=0,
                    help="--impl reference: fix the sample size (default: sized by time and memory)")
    ap.add_argument("--ref-seconds", type=float, default=120.0,
                    help="--impl reference: target seconds for the warm-up and timed steps")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--small", action="store_true", help="tiny model (for profiling captures)")
    ap.add_argument("--model", choices=["1b", "8b"], default="1b",
                    help="8b: the 8B-target workload instead of the headline 1.1B one")
    ap.add_argument("--micro", choices=["gemm8b", "gemm1b", "attention", "accept", "engine",
                                        "sample"],
                    default=None,
                    help="time one kernel family alone (1 GPU) instead of the speculative round")
    ap.add_argument("--only", default=None, help="--micro gemm8b: one shape (qkv, o_proj, ...)")
    ap.add_argument("--qlen", type=int, default=5, help="--micro attention: query tokens per sequence")
    ap.add_argument("--dh", type=int, default=64, choices=[64, 128], help="--micro attention: head size")
    ap.add_argument("--iters", type=int, default=20, help="--micro: timed launches")
    ap.add_argument("--timeline", action="store_true",
                    help="1 GPU: record every kernel of the run with torch.profiler (CUPTI) and "
                         "print each timed round's live time per kernel as a second JSON line")
    ap.add_argument("--gemm-policy", type=int, default=0, choices=[0, 1, 2],
                    help="tensor-core GEMM kernel: 0 by shape, 1 one CTA per tile, 2 CTA pairs")
    return ap.parse_args()


def model_cfgs(small: bool):
    from microserve_b200.config import ModelConfig

    t, d = dict(TARGET), dict(DRAFT)
    if small:
        t.update(n_layers=2)
        d.update(n_layers=1)
    msl = MAX_SEQ
    return (ModelConfig(**t, max_seq_len=msl, dtype="bfloat16"),
            ModelConfig(**d, max_seq_len=msl, dtype="bfloat16"))


def contexts(n: int, lo: int, hi: int, seed: int) -> np.ndarray:
    rng = np.random.default_rng(seed)
    if CTX_LOGNORMAL is not None:  # lognormal with the given mean and std, clipped
        mean, std = CTX_LOGNORMAL
        sig2 = np.log(1.0 + (std / mean) ** 2)
        x = rng.lognormal(np.log(mean) - sig2 / 2, np.sqrt(sig2), n)
        return np.clip(x, lo, hi).astype(np.int64)
    return rng.integers(lo, hi + 1, n)


# -- clocks during the timed region ------------------------------------------------
class ClockSampler:
    """SM clock and clock-event reasons of one GPU, polled through NVML every
    ``period_s`` on a host thread while the timed region runs (a region of
    ~0.1 s would fall between two samples of a 200 ms ``nvidia-smi`` loop).
    Read-only: it queries clocks and reasons and sets nothing."""

    REASONS = {"hw_slowdown": "nvmlClocksEventReasonHwSlowdown",
               "hw_thermal_slowdown": "nvmlClocksEventReasonHwThermalSlowdown",
               "sw_thermal_slowdown": "nvmlClocksEventReasonSwThermalSlowdown",
               "sw_power_cap": "nvmlClocksEventReasonSwPowerCap"}

    def __init__(self, device, period_s: float = 0.005) -> None:
        self.device = device
        self.period = period_s
        self.samples: list[tuple[float, float, int]] = []
        self._stop = None
        self._thread = None
        self._nvml = None
        self._handle = None

    def _open(self) -> bool:
        try:
            import pynvml
            import torch

            pynvml.nvmlInit()
            self._nvml = pynvml
            want = str(torch.cuda.get_device_properties(self.device).uuid)
            for i in range(pynvml.nvmlDeviceGetCount()):
                h = pynvml.nvmlDeviceGetHandleByIndex(i)
                uid = pynvml.nvmlDeviceGetUUID(h)
                uid = uid.decode() if isinstance(uid, bytes) else uid
                if uid.replace("GPU-", "") == want.replace("GPU-", ""):
                    self._handle = h
                    return True
            return False
        except Exception:
            return False

    def start(self) -> None:
        """Starts (or resumes) polling; samples accumulate over every
        start/pause interval."""
        import threading

        if self._handle is None and not self._open():
            return
        if self._thread is not None and self._thread.is_alive():
            return
        nv, h = self._nvml, self._handle
        self._stop = threading.Event()

        def poll() -> None:
            while not self._stop.is_set():
                try:
                    sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
                    mx = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
                    rs = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                    self.samples.append((float(sm), float(mx), int(rs)))
                except Exception:
                    return
                self._stop.wait(self.period)

        self._thread = threading.Thread(target=poll, daemon=True)
        self._thread.start()

    def pause(self) -> None:
        if self._thread is not None:
            self._stop.set()
            self._thread.join(timeout=5)

    def stop(self) -> dict[str, object] | None:
        if self._thread is None:
            return None
        self.pause()
        if not self.samples:
            return None
        nv = self._nvml
        reasons = sorted({name for name, const in self.REASONS.items()
                          for *_, bits in self.samples if bits & getattr(nv, const)})
        sm = [a for a, _, _ in self.samples]
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": max(b for _, b, _ in self.samples),
                "sm_mhz_min": min(sm), "samples": len(sm), "source": "nvml, 5 ms polling",
                "reasons": reasons}


# -- GPU arm -----------------------------------------------------------------------
def gemm_flops_per_round(shape: dict[str, int], tcfg, dcfg) -> float:
    """2*M*N*K over every GEMM launch of one round (the algorithmic FLOPs)."""

    def per_pass(cfg, m: int, rows: int) -> float:
        d, hq, hkv, dh, ff = cfg.d_model, cfg.n_heads, cfg.kv_heads, cfg.d_head, cfg.ffn_hidden
        # qkv, o_proj, gate+up, down
        layer = 2 * m * (d * (hq + 2 * hkv) * dh + hq * dh * d + d * 2 * ff + ff * d)
        return cfg.n_layers * layer + 2 * rows * d * cfg.vocab_size

    B, G = shape["B"], shape["gamma"]
    draft = per_pass(dcfg, shape["T0"], B) + (G - 1) * per_pass(dcfg, B, B)
    return draft + per_pass(tcfg, shape["Tv"], B * (G + 1))


class RequestSet:
    """The requests one rank serves, with their global ids.

    Weak scaling (default): every rank has its own ``--requests`` requests
    (contexts and token ids from a per-rank seed).  Strong scaling
    (``--total-requests T``): one set of T requests, the same on every rank,
    partitioned by ``distributed.shard_requests`` (longest-processing-time on
    context plus the tokens the timed rounds can add); a request's token ids
    and its generator seed depend only on its global id, so its stream is
    the same for any number of GPUs."""

    def __init__(self, args: argparse.Namespace, rank: int, world: int, vocab: int) -> None:
        from microserve_b200 import distributed

        self.strong = bool(args.total_requests)
        if self.strong:
            total = args.total_requests
            ctx_all = contexts(total, args.ctx_min, args.ctx_max, args.seed * 1000)
            cost = (ctx_all + args.steps * (GAMMA + 1)).astype(float).tolist()
            self.ids = np.asarray(distributed.shard_requests(cost, world, rank), dtype=np.int64)
            self.ctx = ctx_all[self.ids]
            self.total = total
        else:
            rng_seed = args.seed * 1000 + rank
            self.ctx = contexts(args.requests, args.ctx_min, args.ctx_max, rng_seed)
            self.ids = rank * args.requests + np.arange(args.requests, dtype=np.int64)
            self.total = args.requests * world
            tok_rng = np.random.default_rng(rng_seed + 7)
            self._prompts = [tok_rng.integers(0, vocab, int(c)).tolist() for c in self.ctx]
            self._seeds = [rng_seed * 100003 + i for i in range(args.requests)]
        self.args = args
        self.vocab = vocab

    def __len__(self) -> int:
        return len(self.ids)

    def prompt(self, k: int) -> list[int]:
        if not self.strong:
            return self._prompts[k]
        rng = np.random.default_rng([self.args.seed, int(self.ids[k])])
        return rng.integers(0, self.vocab, int(self.ctx[k])).tolist()

    def seed(self, k: int) -> int:
        if not self.strong:
            return self._seeds[k]
        return self.args.seed * 100003 + int(self.ids[k])


def plan_waves(ctx: np.ndarray, per_req_blocks: np.ndarray, cap_blocks: int, max_batch: int
               ) -> list[np.ndarray]:
    """Consecutive groups of the rank's requests that fit the cache together:
    admission with a waiting queue, a wave entering when the previous one
    has finished its rounds."""
    waves, cur, used = [], [], 0
    for k in range(len(ctx)):
        b = int(per_req_blocks[k])
        if cur and (used + b > cap_blocks or len(cur) >= max_batch):
            waves.append(np.asarray(cur))
            cur, used = [], 0
        cur.append(k)
        used += b
    if cur:
        waves.append(np.asarray(cur))
    return waves


# DRAM bytes per round of the GEMM class on the default 1.1B workload (256
# requests, gamma 4, chained rounds): the per-launch traffic of an ncu capture
# (dram__bytes_read.sum + dram__bytes_write.sum of every GEMM shape,
# profiles/gemm_tc_kernel_dram_traffic_llama1.1b.md) times each shape's
# launches per round.
GEMM_DRAM_BYTES_PER_ROUND_1B = 4.66e9


def run_gpu(args: argparse.Namespace) -> None:
    import torch

    from microserve_b200 import _lib, distributed
    from microserve_b200.cache import PagedKVCache
    from microserve_b200.config import CacheConfig, SamplingConfig
    from microserve_b200.model import Transformer
    from microserve_b200.scheduler import Request
    from microserve_b200.speculative import SpeculativeDecoder

    info = distributed.init("nccl", timeout_s=300.0) if args.gpus > 1 else distributed.rank_info()
    dev = torch.device("cuda", info.local_rank)
    torch.cuda.set_device(dev)
    _lib.load()
    tcfg, dcfg = model_cfgs(args.small)
    target = Transformer(tcfg, dev, seed=args.seed)
    draft = Transformer(dcfg, dev, seed=args.seed + 1)
    reqset = RequestSet(args, info.rank, info.world_size, tcfg.vocab_size)

    # Cache blocks per request: its context plus every round this run makes
    # (warm-up, timed, GEMM-profile and attention-rate rounds).
    rounds_total = args.warmup + 2 * args.steps + 2
    per_req_blocks = (reqset.ctx + rounds_total * (GAMMA + 1) + 2 * BLOCK) // BLOCK + 1
    # Resident requests: as many as the free HBM holds (K/V of both models,
    # logits rows of a round), the rest wait for the next wave.
    kv_block_bytes = BLOCK * 2 * 2 * (tcfg.n_layers * tcfg.kv_heads * tcfg.d_head
                                      + dcfg.n_layers * dcfg.kv_heads * dcfg.d_head)
    logit_bytes = (2 * GAMMA + 1) * tcfg.vocab_size * 4
    free_b, _ = torch.cuda.mem_get_info(dev)
    budget = 0.85 * free_b - 4e9  # workspace, sampler scratch, allocator slack
    mean_blocks = float(per_req_blocks.mean()) if len(reqset) else 1.0
    max_batch = max(1, int(budget / (mean_blocks * kv_block_bytes + logit_bytes)))
    cap_blocks = max(int(per_req_blocks.max()) if len(reqset) else 1,
                     int((budget - max_batch * logit_bytes) / kv_block_bytes))
    # the partial wave first, so the profiling rounds after the timed ones
    # run on a full one (the caches hold the last wave)
    waves = plan_waves(reqset.ctx, per_req_blocks, cap_blocks, max_batch)[::-1]
    nblocks = max(int(per_req_blocks[w].sum()) for w in waves) + 64
    ccfg = CacheConfig(BLOCK, nblocks, "bfloat16")
    tcache = PagedKVCache(tcfg, ccfg, dev)
    dec = SpeculativeDecoder(target, draft, ccfg, gamma=GAMMA, device=dev)
    g = torch.Generator(device=dev).manual_seed(args.seed * 1000 + info.rank)
    for pool in (tcache.pool, dec.draft_cache.pool):  # synthetic K/V for every context
        for lyr in range(pool.shape[1]):
            pool[:, lyr].normal_(generator=g)
    sc = SamplingConfig(temperature=0.8, top_p=0.9, max_new_tokens=1 << 30)

    def admit(wave: np.ndarray) -> tuple[list, dict]:
        """Take a wave into the caches: its contexts' slots are reserved
        (interleaved, 16 tokens at a time: non-contiguous tables) and hold
        the synthetic K/V already in the pools."""
        tcache.reset()
        dec.reset()
        reqs, gens = [], {}
        for k in wave.tolist():
            prompt = reqset.prompt(k)
            r = Request(int(reqset.ids[k]), prompt, sc)
            r.num_computed = len(prompt) - 1
            reqs.append(r)
            gens[r.request_id] = torch.Generator().manual_seed(reqset.seed(k))
        ids = np.asarray([r.request_id for r in reqs])
        remaining = reqset.ctx[wave] - 1
        while remaining.max() > 0:
            step = np.minimum(remaining, BLOCK)
            live = step > 0
            tcache.append_many(ids[live].tolist(), step[live])
            dec.draft_cache.append_many(ids[live].tolist(), step[live])
            remaining -= step
        torch.cuda.synchronize(dev)
        return reqs, gens

    def one_round(reqs: list, gens: dict) -> int:
        out = dec.step(reqs, tcache, gens)
        n = 0
        for r, toks in zip(reqs, out, strict=True):
            r.output_ids.extend(toks)
            n += len(toks)
        return n

    clocks = ClockSampler(dev) if info.rank == 0 else None
    emitted = accepted = proposed = 0
    h2d = d2h = launches = 0
    dev_ms = e2e_ms = 0.0
    # Several timed regions per wave (each after a fresh admission of the
    # same contexts and its own warm-up), so the clock record covers a long
    # stretch of rounds without the contexts growing past the workload's.
    # The count depends on the arguments only, so every rank runs the same.
    # Strong scaling already times every wave of its request set: once.
    repeats = args.repeats or (1 if reqset.strong else
                               max(1, min(20, -(-200 // max(1, args.steps)))))
    distributed.barrier()
    torch.cuda.synchronize(dev)
    for wave in [w for w in waves for _ in range(repeats)]:
        reqs, gens = admit(wave)
        for i in range(args.warmup):
            # A round's draft passes may be launched ahead by the round before
            # it (round chaining), so the events of the first timed round
            # start during the last warm-up round.
            if i == args.warmup - 1:
                dec.round_events = []
            one_round(reqs, gens)
        acc0, prop0 = dec.num_accepted, dec.num_proposed
        dec.round_events = []
        if dec._pending is not None and dec._pending.events is None and args.warmup:
            raise RuntimeError("the first timed round has no start event")
        launches0 = _lib.launch_count()
        torch.cuda.synchronize(dev)
        if clocks:
            clocks.start()
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(args.steps):
            emitted += one_round(reqs, gens)
            h2d += dec.last_h2d_bytes
            d2h += dec.last_d2h_bytes
        end.record()
        torch.cuda.synchronize(dev)
        if clocks:
            clocks.pause()
        launches += _lib.launch_count() - launches0
        e2e_ms += start.elapsed_time(end)
        dev_ms += sum(a.elapsed_time(b) for a, b in dec.round_events)
        dec.round_events = None
        accepted += dec.num_accepted - acc0
        proposed += dec.num_proposed - prop0
    distributed.barrier()
    torch.cuda.synchronize(dev)
    clk = clocks.stop() if clocks else None
    # GEMM roofline and verify-step time: as many further rounds of the last
    # wave with a CUDA-event pair around every GEMM launch (and around the
    # verify pass).  They stay out of the timed rounds: ~250 event records a
    # round there added ~1.1 ms per round (and broke the programmatic
    # dependent launches between kernels).
    dec.verify_events = []
    flops = 0.0
    _lib.call("ms_profile_start", 1)
    for _ in range(args.steps):
        one_round(reqs, gens)
        flops += gemm_flops_per_round(dec.last_round_shape, tcfg, dcfg)
    torch.cuda.synchronize(dev)
    gemm_ms = _c_double()
    gemm_n = _c_int64()
    _lib.call("ms_profile_stop", _byref(gemm_ms), _byref(gemm_n))
    verify_us = 1e3 * sum(a.elapsed_time(b) for a, b in dec.verify_events) / max(
        1, len(dec.verify_events))
    dec.verify_events = None
    # Paged-attention HBM rate, from extra rounds outside the timed region:
    # attention-class kernel time (CUDA events on the stream) against the K/V
    # bytes the round's passes read (real context lengths).
    attn_rounds = max(1, min(2, args.steps))
    kv_bytes = 0.0
    _lib.call("ms_profile_start", 2)
    for _ in range(attn_rounds):
        one_round(reqs, gens)
        sh = dec.last_round_shape
        kv_bytes += sh["kv_tokens_verify"] * tcfg.n_layers * 2 * tcfg.kv_heads * tcfg.d_head * 2
        kv_bytes += sh["kv_tokens_draft"] * dcfg.n_layers * 2 * dcfg.kv_heads * dcfg.d_head * 2
    torch.cuda.synchronize(dev)
    attn_ms = _c_double()
    attn_n = _c_int64()
    _lib.call("ms_profile_stop", _byref(attn_ms), _byref(attn_n))
    counters = {"emitted": emitted, "accepted": accepted, "proposed": proposed,
                "requests": len(reqset), "waves": len(waves)}
    tot, dev_ms_max = distributed.reduce_stats(counters, dev_ms / 1e3)
    _, e2e_s_max = distributed.reduce_stats({}, e2e_ms / 1e3)
    if info.rank != 0:
        distributed.shutdown()
        return

    peaks = _peaks()
    achieved = flops / (gemm_ms.value / 1e3) / 1e12 if gemm_ms.value > 0 else 0.0
    default_workload = (not args.small and not reqset.strong and args.model == "1b"
                        and args.requests == 256)
    weight_bytes_round = target.weight_bytes() + GAMMA * draft.weight_bytes()
    rounds_timed = args.steps * len(waves) * repeats
    workload = WORKLOAD if not args.small else WORKLOAD + " [small: 2+1 layers]"
    if reqset.strong:
        workload = workload.replace(f"{args.requests} req/GPU",
                                    f"{reqset.total} requests split over the GPUs")
    line = {
        "metric": METRIC,
        "value": tot["emitted"] / dev_ms_max,
        "unit": "tok/s",
        "n_gpus": info.world_size,
        "steps": args.steps,
        "warmup": args.warmup,
        "repeats": repeats,
        "rounds_timed": rounds_timed,
        "ms_per_step": dev_ms_max * 1e3 / rounds_timed,
        "higher_is_better": True,
        "scaling": "strong" if reqset.strong else "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (random-init weights, uniform token ids, synthetic K/V contexts)",
        "config": {
            "workload": workload,
            "requests_total": reqset.total,
            "requests_rank0": len(reqset), "waves_rank0": len(waves),
            "resident_max": int(max(len(w) for w in waves)),
            "gamma": GAMMA, "block_size": BLOCK,
            "ctx_range": [args.ctx_min, args.ctx_max],
            "target": TARGET if not args.small else dict(TARGET, n_layers=2),
            "draft_layers": dcfg.n_layers, "temperature": 0.8, "top_p": 0.9,
            "l2": f"inputs larger than L2 ({target.weight_bytes() / 1e9:.1f} GB target weights + "
                  f"{kv_bytes / attn_rounds / 1e9:.1f} GB of K/V read per round)",
            "parallelism": f"request-sharded x{info.world_size}, no decode-loop collective",
        },
        "acceptance_rate": tot["accepted"] / max(1, tot["proposed"]),
        "emitted_tokens": tot["emitted"],
        "verify_step_us": verify_us,
        "attention": {
            "kernel": "paged attention (verify and draft passes)",
            "bound": "hbm",
            "achieved": kv_bytes / (attn_ms.value / 1e3) / 1e9 if attn_ms.value > 0 else 0.0,
            "peak": peaks["hbm_gbs"],
            "unit": "GB/s",
            "frac": (kv_bytes / (attn_ms.value / 1e3) / 1e9 / peaks["hbm_gbs"]
                     if attn_ms.value > 0 else 0.0),
            "kv_bytes_per_round": kv_bytes / attn_rounds,
            "launches": int(attn_n.value),
            "device_ms": attn_ms.value,
            "rounds": attn_rounds,
        },
        "e2e": {
            "value": tot["emitted"] / e2e_s_max,
            "unit": "tok/s",
            "h2d_bytes_per_step": h2d // rounds_timed,
            "d2h_bytes_per_step": d2h // rounds_timed,
            "ms_per_step": e2e_s_max * 1e3 / rounds_timed,
        },
        "gpu_launches": int(launches),
        "roofline": {
            "kernel": "GEMM (all projection and lm_head launches)",
            "bound": "tensor",
            "achieved": achieved,
            "peak": peaks["bf16_sustained"],
            "unit": "TFLOP/s",
            "frac": achieved / peaks["bf16_sustained"],
            "peak_source": peaks["source"],
            "traffic": (GEMM_DRAM_BYTES_PER_ROUND_1B if default_workload else None),
            "traffic_unit": "bytes per round (all GEMM launches of a round, ncu capture)",
            "weight_bytes_per_round": weight_bytes_round,
            "launches": int(gemm_n.value),
            "device_ms": gemm_ms.value,
            "measured_over": f"{args.steps} rounds of the same workload after the timed rounds, "
                             "a CUDA-event pair around each GEMM launch on its stream",
        },
        "clocks": clk,
    }
    if not args.no_cpu_baseline and info.world_size == 1:
        line["cpu_baseline"] = cpu_baseline(args)
    print(json.dumps(line), flush=True)
    distributed.shutdown()


def _c_double():
    import ctypes

    return ctypes.c_double(0.0)


def _c_int64():
    import ctypes

    return ctypes.c_int64(0)


def _byref(x):
    import ctypes

    return ctypes.byref(x)


def _peaks() -> dict[str, object]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16": d["bf16_tflops"],
                "bf16_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]),
                "source": "measured (MEASURED_PEAKS.json)"}
    return {"hbm_gbs": 6650.0, "bf16": 1590.0, "bf16_sustained": 1400.0, "source": "fallback"}


# -- CPU side: the reference's own implementation of the path -------------------------------
REF_DIR = ROOT / "baseline" / "_ref"


def reference_installed() -> bool:
    return (REF_DIR / "microserve" / "speculative.py").exists()


class ReferenceRun:
    """The unmodified reference (``baseline/_ref``: its ``SpeculativeDecoder``,
    ``Transformer``, ``PagedKVCache`` and samplers, float32 on the CPU) on a
    sample of the benchmark workload: the first ``n`` requests of rank 0's
    request set (the same contexts and token ids as the GPU arm), the same
    model shapes with the same initialisation recipe (the reference's own
    init, weights rounded to bf16 values), grouped-query attention expressed
    as the reference's multi-head attention with each K/V head's projection
    rows repeated over its query group, and synthetic K/V histories written
    into its cache pools.  One step = one ``SpeculativeDecoder.step`` over the
    sample; emitted tokens are appended as the engine does."""

    def __init__(self, args: argparse.Namespace, n_req: int, threads: int) -> None:
        import torch

        if str(REF_DIR) not in sys.path:
            sys.path.insert(0, str(REF_DIR))
        from microserve.cache import PagedKVCache
        from microserve.config import CacheConfig, ModelConfig, SamplingConfig
        from microserve.model import Transformer
        from microserve.scheduler import Request
        from microserve.speculative import SpeculativeDecoder

        torch.set_num_threads(threads)
        self.threads = torch.get_num_threads()
        torch.manual_seed(args.seed)
        t, d = dict(TARGET), dict(DRAFT)
        if args.small:
            t.update(n_layers=2)
            d.update(n_layers=1)

        def build(c: dict) -> object:
            cfg = ModelConfig(vocab_size=c["vocab_size"], n_layers=c["n_layers"],
                              d_model=c["d_model"], n_heads=c["n_heads"], d_ff=c["d_ff"],
                              max_seq_len=MAX_SEQ, rope_theta=c["rope_theta"])
            m = Transformer(cfg).eval()
            dh, group = c["d_model"] // c["n_heads"], c["n_heads"] // c["n_kv_heads"]
            with torch.no_grad():
                for blk in m.blocks:
                    for lin in (blk.attn.k_proj, blk.attn.v_proj):
                        w = lin.weight
                        kv = w[: c["n_kv_heads"] * dh].view(c["n_kv_heads"], dh, -1)
                        w.copy_(kv.repeat_interleave(group, 0).reshape(w.shape))
                for prm in m.parameters():
                    prm.copy_(prm.bfloat16().float())
            return m

        self.target, self.draft = build(t), build(d)
        ctx = contexts(args.requests, args.ctx_min, args.ctx_max, args.seed * 1000)[:n_req]
        rounds = args.warmup + args.steps + 2
        blocks = int(((ctx + rounds * (GAMMA + 1) + 2 * BLOCK) // BLOCK + 1).sum()) + 16
        ccfg = CacheConfig(block_size=BLOCK, num_blocks=blocks)
        self.cache = PagedKVCache(self.target.cfg, ccfg)
        self.dec = SpeculativeDecoder(self.target, self.draft, ccfg, gamma=GAMMA)
        tok_rng = np.random.default_rng(args.seed * 1000 + 7)
        sc = SamplingConfig(temperature=0.8, top_p=0.9, max_new_tokens=1 << 30)
        self.reqs, self.gens = [], {}
        for i in range(n_req):
            prompt = tok_rng.integers(0, t["vocab_size"], int(ctx[i])).tolist()
            r = Request(request_id=i, prompt_ids=prompt, sampling=sc)
            r.num_computed = len(prompt) - 1
            self.cache.append(i, len(prompt) - 1)
            self.dec.draft_cache.append(i, len(prompt) - 1)
            self.reqs.append(r)
            self.gens[i] = torch.Generator().manual_seed(args.seed * 100003 + i)
        bank = torch.randn(1 << 20, generator=torch.Generator().manual_seed(args.seed))
        for c in (self.cache, self.dec.draft_cache):
            for pool in (*c.k_cache, *c.v_cache):
                flat = pool.view(-1)
                reps = flat.numel() // bank.numel()
                flat[: reps * bank.numel()].view(reps, -1).copy_(bank.expand(reps, -1))
                flat[reps * bank.numel():].copy_(bank[: flat.numel() - reps * bank.numel()])
        self.n = n_req
        self.accepted = 0
        self.proposed = 0

    @staticmethod
    def bytes_per_request(args: argparse.Namespace) -> float:
        """Host memory one request takes: its share of both float32 caches
        (multi-head layout) and of the padded gather of a pass."""
        t = TARGET
        per_tok = 2 * t["d_model"] * 4 * (t["n_layers"] + DRAFT["n_layers"])
        return per_tok * (args.ctx_max + 64) * 1.5

    def rounds(self, k: int) -> tuple[int, float]:
        """``k`` steps; returns (emitted tokens, seconds)."""
        emitted = 0
        acc0, prop0 = self.dec.num_accepted, self.dec.num_proposed
        t0 = time.perf_counter()
        for _ in range(k):
            out = self.dec.step(self.reqs, self.cache, self.gens)
            for r, toks in zip(self.reqs, out, strict=True):
                r.output_ids.extend(toks)
                emitted += len(toks)
        secs = time.perf_counter() - t0
        self.accepted += self.dec.num_accepted - acc0
        self.proposed += self.dec.num_proposed - prop0
        return emitted, secs


def _available_ram() -> float:
    try:
        import psutil

        return float(psutil.virtual_memory().available)
    except ImportError:
        return float(os.sysconf("SC_AVPHYS_PAGES") * os.sysconf("SC_PAGE_SIZE"))


def cpu_baseline(args: argparse.Namespace) -> dict[str, object]:
    """The reference's CPU path on a bounded sample (a few requests x 2 steps,
    all host cores), reported beside the GPU number; the numpy restatement
    when the reference is not installed."""
    n = max(1, args.cpu_requests)
    if not reference_installed():
        return cpu_baseline_port(args, n)
    run = ReferenceRun(args, n, os.cpu_count() or 1)
    run.rounds(1)
    emitted, secs = run.rounds(2)
    return {"value": emitted / secs, "unit": "tok/s", "cores": run.threads, "kind": "reference",
            "sample": f"{n} of the workload's requests x 2 steps of the unmodified reference "
                      f"SpeculativeDecoder (float32, CPU), {secs:.1f} s"}


def run_reference(args: argparse.Namespace) -> None:
    """``--impl reference``: the reference's own CPU implementation of the
    speculative step, on this host's cores, for the same metric and workload.

    The sample is the first n requests of the workload, n the largest that
    fits half of the free host memory and keeps the warm-up and timed steps
    near two minutes (from a timed probe step of a few requests), at most the
    workload's request count.  Rank 0 runs it; other ranks exit."""
    if int(os.environ.get("RANK", "0")) != 0:
        return
    cores = os.cpu_count() or 1
    if not reference_installed():
        print(json.dumps({"impl": "reference", "metric": METRIC,
                          "unavailable": "baseline/_ref is not installed"}), flush=True)
        return
    probe_n = min(4, args.requests)
    probe = ReferenceRun(args, probe_n, cores)
    probe.rounds(1)
    _, secs = probe.rounds(1)
    per_req_s = secs / probe_n
    budget_s = float(args.ref_seconds)
    by_time = int(budget_s / max(1e-6, per_req_s * (args.warmup + args.steps)))
    by_ram = int(0.5 * _available_ram() / ReferenceRun.bytes_per_request(args))
    n = max(1, min(args.requests, by_time, by_ram))
    del probe
    if args.cpu_requests_ref:
        n = min(args.requests, args.cpu_requests_ref)
    run = ReferenceRun(args, n, cores)
    run.rounds(args.warmup)
    emitted, secs = run.rounds(args.steps)
    value = emitted / secs
    # the reference's published setting: one thread, one step of a small sample
    one = ReferenceRun(args, min(n, 4), 1)
    e1, s1 = one.rounds(1)
    line = {
        "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": secs * 1e3 / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (random-init weights, uniform token ids, synthetic K/V contexts)",
        "impl": "reference",
        "config": {"workload": WORKLOAD, "requests_sampled": n, "requests_in_workload": args.requests,
                   "same_config": n == args.requests, "gamma": GAMMA, "block_size": BLOCK,
                   "ctx_range": [args.ctx_min, args.ctx_max], "temperature": 0.8, "top_p": 0.9},
        "acceptance_rate": run.accepted / max(1, run.proposed),
        "per_request_tok_s": value / n,
        "cpu_baseline": {"value": value, "unit": "tok/s", "cores": run.threads, "kind": "reference",
                         "sample": f"first {n} of {args.requests} requests of the workload, "
                                   f"{args.steps} steps of the unmodified reference "
                                   "SpeculativeDecoder.step (float32 on the CPU, GQA as "
                                   "repeated K/V heads)",
                         "single_thread": {"value": e1 / s1, "unit": "tok/s", "threads": 1,
                                           "sample": f"{min(n, 4)} requests x 1 step"}},
        "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# -- the numpy restatement, when the reference is not installed ----------------------------
def cpu_baseline_port(args: argparse.Namespace, n_req: int) -> dict[str, object]:
    """The oracle restatement of the same round on a few requests (kind "port")."""
    from oracle.model import Dims, OracleModel
    from oracle.spec import OracleRequest, spec_round

    seed = args.seed + 99
    rng = np.random.default_rng(seed)

    def state(cfg: dict) -> dict[str, np.ndarray]:
        d, hq, hkv, ff, L = cfg["d_model"], cfg["n_heads"], cfg["n_kv_heads"], cfg["d_ff"], cfg["n_layers"]
        dh = d // hq
        res = 0.02 / np.sqrt(2 * L)
        n = lambda *s, std=0.02: rng.standard_normal(s, dtype=np.float32) * np.float32(std)  # noqa: E731
        st = {"embed.weight": n(cfg["vocab_size"], d), "norm.weight": np.ones(d, np.float32)}
        for i in range(L):
            p = f"blocks.{i}."
            st[p + "attn.q_proj.weight"] = n(hq * dh, d)
            st[p + "attn.k_proj.weight"] = n(hkv * dh, d)
            st[p + "attn.v_proj.weight"] = n(hkv * dh, d)
            st[p + "attn.o_proj.weight"] = n(d, hq * dh, std=res)
            st[p + "ffn.gate_proj.weight"] = n(ff, d)
            st[p + "ffn.up_proj.weight"] = n(ff, d)
            st[p + "ffn.down_proj.weight"] = n(d, ff, std=res)
            st[p + "attn_norm.weight"] = np.ones(d, np.float32)
            st[p + "ffn_norm.weight"] = np.ones(d, np.float32)
        return st

    t, dr = dict(TARGET), dict(DRAFT)
    if args.small:
        t.update(n_layers=2)
        dr.update(n_layers=1)
    dims = lambda c: Dims(c["vocab_size"], c["d_model"], c["n_layers"], c["n_heads"],  # noqa: E731
                          c["n_kv_heads"], c["d_ff"], MAX_SEQ, c["rope_theta"])
    target, draft = OracleModel(dims(t), state(t)), OracleModel(dims(dr), state(dr))
    ctx = contexts(n_req, args.ctx_min, args.ctx_max, seed + 1)
    reqs = []
    for i in range(n_req):
        r = OracleRequest(i, rng.integers(0, t["vocab_size"], int(ctx[i])).tolist(), 0.8, None,
                          0.9, seed=seed * 7 + i)
        dh = t["d_model"] // t["n_heads"]
        for kv, cfg in ((r.target_kv, t), (r.draft_kv, dr)):
            shape = (int(ctx[i]) - 1, cfg["n_kv_heads"], dh)
            kv.k = [rng.standard_normal(shape, dtype=np.float32) for _ in range(cfg["n_layers"])]
            kv.v = [rng.standard_normal(shape, dtype=np.float32) for _ in range(cfg["n_layers"])]
        reqs.append(r)
    emitted = 0
    t0 = time.perf_counter()
    for _ in range(2):
        tr = spec_round(target, draft, GAMMA, reqs)
        for r, toks in zip(reqs, tr.emitted, strict=True):
            r.output_ids.extend(toks)
            emitted += len(toks)
    secs = time.perf_counter() - t0
    return {"value": emitted / secs, "unit": "tok/s", "cores": os.cpu_count(), "kind": "port",
            "sample": f"{n_req} requests x 2 steps, numpy float32 restatement of the reference "
                      f"path (the reference is not installed), {secs:.1f} s"}


# -- kernel micro-benchmarks (one GPU; not the headline metric) --------------------------
GEMM8B = [  # (name, N, K, epilogue, output dtype) at M = 256 requests x 6 tokens
    ("qkv", 6144, 4096, 0, "bf16"), ("o_proj", 4096, 4096, 1, "f32"),
    ("gate_up", 28672, 4096, 2, "bf16"), ("down", 4096, 14336, 1, "f32"),
    ("lm_head", 128256, 4096, 0, "f32"),
]


# The 1.1B target's verify GEMMs (M = 256 requests x 5 tokens) and the draft's (M = 256):
# (name, M, N, K, epilogue, output dtype); weights cycle over the 22 layers' copies.
GEMM1B = [
    ("qkv", 1280, 2560, 2048, 0, "bf16"), ("o_proj", 1280, 2048, 2048, 1, "f32"),
    ("gate_up", 1280, 11264, 2048, 2, "bf16"), ("down", 1280, 2048, 5632, 1, "f32"),
    ("lm_head", 1280, 32000, 2048, 0, "f32"),
    ("draft_qkv", 256, 2560, 2048, 0, "bf16"), ("draft_o_proj", 256, 2048, 2048, 1, "f32"),
    ("draft_gate_up", 256, 11264, 2048, 2, "bf16"), ("draft_down", 256, 2048, 5632, 1, "f32"),
    ("draft_lm_head", 256, 32000, 2048, 0, "f32"),
]


def _time_launches(call, iters: int) -> float:
    """Mean microseconds per launch over `iters` back-to-back launches (CUDA events)."""
    import torch

    for _ in range(3):
        call()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        call()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / iters * 1e3


def run_micro_accept(args: argparse.Namespace, peaks: dict[str, float]) -> None:
    """The acceptance microbenchmark: 4096 requests, gamma 5, vocab 32000, fp32 logits.

    Target logits N(0, 2^2); draft logits = the target's first gamma rows plus
    N(0, 0.5^2) noise (seed 1234).  Proposals are drawn from the draft rows
    (ms_sample, untimed); the timed call is ms_spec_accept over all requests.
    Algorithmic bytes: every target and draft row read once,
    4096 * (2*gamma + 1) * V * 4 B = 5.77 GB per call.
    """
    import torch

    from microserve_b200 import _lib
    from microserve_b200.sampling import params_to_device

    B, G, V = 4096, 5, 32000
    gen = torch.Generator(device="cuda").manual_seed(1234)
    target = torch.randn(B, G + 1, V, device="cuda", generator=gen) * 2.0
    noise = torch.randn(G, B, V, device="cuda", generator=gen) * 0.5
    draft = target[:, :G, :].permute(1, 0, 2) + noise  # position-major: row i*B + b
    del noise
    target = target.reshape(B * (G + 1), V)
    draft = draft.contiguous().reshape(G * B, V)
    proposals = torch.empty(G * B, dtype=torch.int32, device="cuda")
    stats = torch.empty(G * B * 16, dtype=torch.uint8, device="cuda")
    out = torch.empty(B * (G + 1), dtype=torch.int32, device="cuda")
    nacc = torch.empty(B, dtype=torch.int32, device="cuda")
    kv_bytes = float(B) * (2 * G + 1) * V * 4
    stream = _lib.stream_ptr()
    for label, top_k, top_p in (("plain", 0, 1.0), ("top-k 50", 50, 1.0), ("top-p 0.9", 0, 0.9)):
        p = np.zeros(B, dtype=_lib.SAMPLING_PARAMS_DTYPE)
        p["temperature"] = 1.0
        p["top_k"] = top_k
        p["top_p"] = top_p
        p["seed"] = 1234
        p["step"] = np.arange(B, dtype=np.uint64)
        params = params_to_device(p, torch.device("cuda"))
        for i in range(G):
            _lib.call("ms_sample", draft[i * B:].data_ptr(), V, B, V, params.data_ptr(), None,
                      _lib.LANE_DRAFT + i, proposals[i * B:].data_ptr(), None,
                      stats[i * B * 16:].data_ptr(), None, None, stream)

        def call() -> None:
            _lib.call("ms_spec_accept", target.data_ptr(), V, draft.data_ptr(), V,
                      stats.data_ptr(), 0, proposals.data_ptr(), params.data_ptr(), B, G, V,
                      out.data_ptr(), nacc.data_ptr(), stream)

        us = _time_launches(call, args.iters)
        rate = float(nacc.float().mean()) / G
        print(json.dumps({"micro": "accept", "variant": label, "requests": B, "gamma": G,
                          "vocab": V, "us": us, "algorithmic_bytes": kv_bytes,
                          "gbs": kv_bytes / us / 1e3, "frac_hbm": kv_bytes / us / 1e3 / peaks["hbm_gbs"],
                          "acceptance_rate": rate, "device_error": _lib.device_error()}),
              flush=True)


def run_micro_engine(args: argparse.Namespace) -> None:
    """Continuous batching with speculative decoding through the public LLMEngine.

    The character-level fp32 models (target d128 L4 H4 ff352 V65, draft d64
    L2 H2 ff176), random-init weights; 1024 concurrent requests, prompts
    lognormal (mean 100, std 50, clipped to [8, 512]) of uniform token ids,
    output budgets uniform in [1, 50]; block 16 with interleaved allocation
    (the scheduler admits requests in arrival order).  One line per (gamma,
    greedy | T 0.8): generated tokens / wall time of ``LLMEngine.run`` from
    the first prefill to the last request finishing, and the K/V bytes the
    speculative rounds' attention read (target 4 KB and draft 1 KB per cached
    token per pass).
    """
    import torch

    from microserve_b200.config import (CacheConfig, EngineConfig, ModelConfig, SamplingConfig,
                                        SchedulerConfig, SpeculativeConfig)
    from microserve_b200.engine import LLMEngine
    from microserve_b200.model import Transformer

    n_req = 1024
    rng = np.random.default_rng(args.seed)
    mean, std = 100.0, 50.0
    sig2 = np.log(1.0 + (std / mean) ** 2)
    lens = np.clip(rng.lognormal(np.log(mean) - sig2 / 2, np.sqrt(sig2), n_req), 8, 512).astype(int)
    outs = rng.integers(1, 51, n_req)
    prompts = [rng.integers(0, 65, int(n)).tolist() for n in lens]
    msl = 512 + 64
    tcfg = ModelConfig(vocab_size=65, d_model=128, n_layers=4, n_heads=4, d_ff=352, max_seq_len=msl)
    dcfg = ModelConfig(vocab_size=65, d_model=64, n_layers=2, n_heads=2, d_ff=176, max_seq_len=msl)
    target = Transformer(tcfg, "cuda", seed=0)
    draft = Transformer(dcfg, "cuda", seed=1)
    blocks = int(((lens + outs + 16) // 16 + 2).sum()) + 64
    for gamma in (1, 2, 3, 5):
        for temp in (0.0, 0.8):
            cfg = EngineConfig(
                model=tcfg, cache=CacheConfig(16, blocks, "float32"),
                scheduler=SchedulerConfig(max_batch_size=n_req, max_batched_tokens=1 << 18),
                speculative=SpeculativeConfig(enabled=True, gamma=gamma), seed=args.seed)
            eng = LLMEngine(target, cfg, draft_model=draft)
            for pr, o in zip(prompts, outs.tolist()):
                eng.add_request(pr, SamplingConfig(temperature=temp, max_new_tokens=o))
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            results = eng.run()
            torch.cuda.synchronize()
            secs = time.perf_counter() - t0
            toks = sum(len(r.output_ids) for r in results)
            st = eng.stats
            print(json.dumps({"micro": "engine", "gamma": gamma, "temperature": temp,
                              "requests": n_req, "generated_tokens": toks, "seconds": secs,
                              "tok_s": toks / secs, "steps": st.num_steps,
                              "spec_rounds": st.num_spec_rounds,
                              "acceptance_rate": st.acceptance_rate,
                              "mean_batch": st.mean_batch_size}), flush=True)
            del eng


def run_micro_sample(args: argparse.Namespace) -> None:
    """One ms_sample launch over 256 rows (a draft pass's draws) at vocab
    32000 (the 1.1B model) and 128256 (the 8B one): logits N(0, 1.3^2),
    temperature 0.8, top-p 0.9 and no filter."""
    import torch

    from microserve_b200 import _lib
    from microserve_b200.sampling import params_to_device

    B = args.requests
    gen = torch.Generator(device="cuda").manual_seed(args.seed)
    for V in (32000, 128256):
        logits = torch.randn(B, V, device="cuda", generator=gen) * 1.3
        tokens = torch.empty(B, dtype=torch.int32, device="cuda")
        for top_p in (0.9, 1.0):
            p = np.zeros(B, dtype=_lib.SAMPLING_PARAMS_DTYPE)
            p["temperature"] = 0.8
            p["top_p"] = top_p
            p["seed"] = 7
            p["step"] = np.arange(B, dtype=np.uint64)
            params = params_to_device(p, torch.device("cuda"))

            def call() -> None:
                _lib.call("ms_sample", logits.data_ptr(), V, B, V, params.data_ptr(), None, 0,
                          tokens.data_ptr(), None, None, None, None, _lib.stream_ptr())

            us = _time_launches(call, args.iters)
            print(json.dumps({"micro": "sample", "rows": B, "vocab": V, "temperature": 0.8,
                              "top_p": top_p, "us": us, "gbs": B * V * 4 / us / 1e3,
                              "device_error": _lib.device_error()}), flush=True)
        del logits


def run_micro(args: argparse.Namespace) -> None:
    import ctypes

    import torch

    from microserve_b200 import _lib

    _lib.load()
    peaks = _peaks()
    g = torch.Generator(device="cuda").manual_seed(args.seed)
    if args.micro == "gemm8b":
        M = 1536
        for name, N, K, epi, cd in GEMM8B:
            if args.only and name != args.only:
                continue
            A = (torch.randn(M, K, device="cuda", generator=g) * 0.5).bfloat16()
            B = (torch.randn(N, K, device="cuda", generator=g) * 0.02).bfloat16()
            C = torch.zeros(M, N // 2 if epi == 2 else N, device="cuda",
                            dtype=torch.float32 if cd == "f32" else torch.bfloat16)
            R = C if epi == 1 else None
            cdt = _lib.DTYPE_F32 if cd == "f32" else _lib.DTYPE_BF16

            def call() -> None:
                _lib.call("ms_gemm", A.data_ptr(), B.data_ptr(), C.data_ptr(), _lib.ptr(R), M, N,
                          K, 0, _lib.DTYPE_BF16, cdt, epi, _lib.stream_ptr())

            us = _time_launches(call, args.iters)
            tf = 2.0 * M * N * K / us / 1e6
            print(json.dumps({"micro": "gemm8b", "gemm": name, "M": M, "N": N, "K": K, "us": us,
                              "tflops": tf, "frac_sustained": tf / peaks["bf16_sustained"],
                              "device_error": _lib.device_error()}), flush=True)
        return
    if args.micro == "gemm1b":
        for name, M, N, K, epi, cd in GEMM1B:
            if args.only and name != args.only:
                continue
            copies = 1 if name.endswith("lm_head") else TARGET["n_layers"]
            A = (torch.randn(M, K, device="cuda", generator=g) * 0.5).bfloat16()
            Bs = [(torch.randn(N, K, device="cuda", generator=g) * 0.02).bfloat16()
                  for _ in range(copies)]
            C = torch.zeros(M, N // 2 if epi == 2 else N, device="cuda",
                            dtype=torch.float32 if cd == "f32" else torch.bfloat16)
            R = C if epi == 1 else None
            cdt = _lib.DTYPE_F32 if cd == "f32" else _lib.DTYPE_BF16
            it = [0]

            def call() -> None:
                B = Bs[it[0] % copies]
                it[0] += 1
                _lib.call("ms_gemm", A.data_ptr(), B.data_ptr(), C.data_ptr(), _lib.ptr(R), M, N,
                          K, 0, _lib.DTYPE_BF16, cdt, epi, _lib.stream_ptr())

            us = _time_launches(call, max(args.iters, copies))
            tf = 2.0 * M * N * K / us / 1e6
            wbytes = N * K * 2
            print(json.dumps({"micro": "gemm1b", "gemm": name, "M": M, "N": N, "K": K, "us": us,
                              "tflops": tf, "frac_sustained": tf / peaks["bf16_sustained"],
                              "weight_gbs": wbytes / us / 1e3, "weight_copies": copies,
                              "device_error": _lib.device_error()}), flush=True)
            del Bs
        return
    if args.micro == "accept":
        run_micro_accept(args, peaks)
        return
    if args.micro == "engine":
        run_micro_engine(args)
        return
    if args.micro == "sample":
        run_micro_sample(args)
        return
    # attention: the config-3 verify (qlen 5) or draft (qlen 1) pass of one layer
    from microserve_b200.batching import build_paged_batch
    from microserve_b200.cache import PagedKVCache
    from microserve_b200.config import CacheConfig, ModelConfig

    # dh 64: the 1.1B target (4 kv heads); dh 128: the 8B target's heads (8 kv heads)
    hq, bs, nseq = TARGET["n_heads"], BLOCK, args.requests
    dh = args.dh
    hkv = TARGET["n_kv_heads"] if dh == 64 else 8
    # longest context first: the order ms_forward schedules a batch's sequences in
    ctx = np.sort(contexts(nseq, args.ctx_min, args.ctx_max, args.seed))[::-1].copy()
    cfg = ModelConfig(vocab_size=16, n_layers=1, d_model=hq * dh, n_heads=hq, n_kv_heads=hkv,
                      max_seq_len=max(4096, args.ctx_max + 64), dtype="bfloat16")
    cache = PagedKVCache(cfg, CacheConfig(bs, int(sum(-(-int(c) // bs) for c in ctx)) + 16,
                                          "bfloat16"), "cuda")
    cache.pool.normal_(generator=g)
    pre = ctx - args.qlen
    done = np.zeros(nseq, np.int64)
    ids = list(range(nseq))
    while (done < pre).any():  # interleaved block allocation
        step = np.minimum(bs, pre - done)
        live = [i for i in ids if step[i] > 0]
        cache.append_many(live, step[live])
        done += step
    batch = build_paged_batch(cache, ids, [[1] * args.qlen for _ in ids], pre.tolist())
    q = torch.randn(batch.n_tokens, hq * dh, device="cuda", generator=g).bfloat16()
    out = torch.empty_like(q)
    cb, cs = batch.c_struct(), cache.c_struct()

    def call() -> None:
        _lib.call("ms_paged_attention", q.data_ptr(), ctypes.byref(cs), 0, ctypes.byref(cb), hq,
                  out.data_ptr(), _lib.stream_ptr())

    us = _time_launches(call, args.iters)
    kv = float(ctx.sum()) * hkv * dh * 2 * 2
    print(json.dumps({"micro": "attention", "qlen": args.qlen, "dh": dh, "kv_heads": hkv,
                      "seqs": nseq, "ctx_range": [args.ctx_min, args.ctx_max], "order": "longest first",
                      "us": us,
                      "kv_bytes": kv, "gbs": kv / us / 1e3, "frac_hbm": kv / us / 1e3 / peaks["hbm_gbs"],
                      "device_error": _lib.device_error()}), flush=True)


def use_8b(args: argparse.Namespace) -> None:
    """Switch the module's workload constants to the 8B-class configuration."""
    global TARGET, DRAFT, GAMMA, MAX_SEQ, CTX_LOGNORMAL, METRIC, WORKLOAD
    TARGET, DRAFT, GAMMA, MAX_SEQ = dict(TARGET_8B), dict(DRAFT_8B), 5, 8192 + 512
    CTX_LOGNORMAL = (2048.0, 1024.0)
    args.ctx_min, args.ctx_max = 8, 8192
    METRIC = "accepted tok/s per B200 (spec γ=5, 8B target)"
    WORKLOAD = ("llama-3-8b-shape bf16 target + 1b-class 16-layer draft, 256 req/GPU, "
                "ctx lognormal(2048, 1024) in [8, 8192], gamma 5, T 0.8, top-p 0.9")
    args.no_cpu_baseline = True  # the CPU restatement of an 8B model is out of reach


def main() -> None:
    args = parse()
    if args.gemm_policy:
        from microserve_b200 import _lib

        _lib.call("ms_gemm_set_policy", args.gemm_policy)
    if args.model == "8b":
        if args.impl == "reference" or args.micro:
            raise SystemExit("--model 8b runs the speculative rounds on the GPU only")
        use_8b(args)
    if args.micro:
        run_micro(args)
    elif args.impl == "reference":
        run_reference(args)
    elif args.timeline:
        run_timeline(args)
    else:
        run_gpu(args)


def run_timeline(args: argparse.Namespace) -> None:
    """The GPU arm under torch.profiler's CUDA activity records: each timed
    round's span, idle time and per-kernel live time.  With programmatic
    dependent launch a kernel starts while its predecessor still runs, so a
    kernel's live time is counted from the later of its start and the end
    of every kernel before it (the sum over a round is its busy time).  A
    round ends with its accept kernel.  The first timed round is left out:
    it also holds the host synchronisation between the warm-up and the timed
    rounds.  Timing under the profiler is not a bench value; the breakdown
    is what this is for."""
    import torch
    from torch.profiler import ProfilerActivity, profile

    if int(os.environ.get("WORLD_SIZE", "1")) > 1:
        raise SystemExit("--timeline runs on one GPU")
    args.repeats = 1
    with profile(activities=[ProfilerActivity.CUDA], acc_events=True) as prof:
        run_gpu(args)
        torch.cuda.synchronize()
    ev = [(e.time_range.start, e.time_range.end, e.name) for e in prof.events()
          if e.device_type.name == "CUDA" and e.name
          and "Memcpy" not in e.name and "Memset" not in e.name]
    print(json.dumps(timeline_summary(ev, args.warmup + 1, args.warmup + args.steps)),
          flush=True)


def _short_kernel_name(n: str) -> str:
    n = n.replace("(anonymous namespace)::", "").replace("void ", "").replace("ms::", "")
    return n.split("(")[0][:60]


def timeline_summary(events: list[tuple[float, float, str]], first: int, stop: int) -> dict:
    """Rounds ``first`` .. ``stop - 1`` (0-based, a round ending with its
    accept kernel) of a kernel list ``(start, end, name)`` in microseconds:
    each round's span and idle time, and each kernel's live time, counted
    from the later of its own start and the end of every kernel before it
    (kernels that start early and wait for their predecessor overlap it)."""
    ev = sorted(events)
    ends = [i for i, (_, _, n) in enumerate(ev) if "spec_accept" in n]
    per: dict[str, list[float]] = {}
    spans, idles = [], []
    for r in range(first, min(stop, len(ends))):
        seg = ev[ends[r - 1] + 1 : ends[r] + 1] if r else ev[: ends[0] + 1]
        prev_end, idle = seg[0][0], 0.0
        for s_, e_, n in seg:
            idle += max(0.0, s_ - prev_end)
            slot = per.setdefault(_short_kernel_name(n), [0, 0.0])
            slot[0] += 1
            slot[1] += max(0.0, e_ - max(prev_end, s_))
            prev_end = max(prev_end, e_)
        spans.append(seg[-1][1] - seg[0][0])
        idles.append(idle)
    n = max(1, len(spans))
    return {
        "timeline": "live time per kernel and timed round (torch.profiler CUDA activities)",
        "rounds": len(spans), "round_us": sum(spans) / n, "idle_us": sum(idles) / n,
        "round_us_each": [round(x, 1) for x in spans], "idle_us_each": [round(x, 1) for x in idles],
        "kernels": {k: {"launches": c / n, "us": t / n, "share": t / max(1e-9, sum(spans))}
                    for k, (c, t) in sorted(per.items(), key=lambda x: -x[1][1])},
    }


if __name__ == "__main__":
    main()
