"""ms_paged_attention against a float32 torch reference of the same bf16 K/V.

bf16 caches with d_head 64/128 take the tensor-core kernels (TMA-fed for
power-of-two block sizes 8..64, cp.async-fed otherwise); float32 and other
head sizes the CUDA-core kernel.  The reference runs on the CPU: it reads
each sequence's keys out of a host copy of the pool by plain indexing
through the host block table (no library call) and applies the reference's
causal rule (key j is visible to a query at absolute position p iff j <= p).

Tolerance (bf16): per sequence, ``|got - ref| <= 2e-3 * max|ref_seq| +
8e-3 * |ref|``.  The output is rounded to bf16 (2^-9 relative) and P enters
the PV product in bf16; the scale of the absolute term follows each
sequence, so at a context of 2048 (outputs ~0.02) one wrong key -- a
probability of ~1/2048 times a value difference of ~1 -- exceeds it, which
the negative control checks."""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _case(dtype: str, hq: int, hkv: int, dh: int, bs: int, ctx: list[int], qlen: list[int], seed: int):
    from microserve_b200 import _lib
    from microserve_b200.batching import build_paged_batch
    from microserve_b200.cache import PagedKVCache
    from microserve_b200.config import CacheConfig, ModelConfig

    cfg = ModelConfig(vocab_size=16, n_layers=1, d_model=hq * dh, n_heads=hq, n_kv_heads=hkv,
                      max_seq_len=4096, dtype=dtype)
    nblocks = sum(-(-c // bs) for c in ctx) + 8
    cache = PagedKVCache(cfg, CacheConfig(bs, nblocks, dtype), DEV)
    g = torch.Generator(device=DEV).manual_seed(seed)
    cache.pool.copy_(torch.randn(cache.pool.shape, generator=g, device=DEV))
    rng = np.random.default_rng(seed)
    # prefix already cached, then a pass of qlen tokens; interleave allocation
    pre = [c - q for c, q in zip(ctx, qlen)]
    done = [0] * len(ctx)
    while any(d < p for d, p in zip(done, pre)):
        for i in range(len(ctx)):
            n = min(bs, pre[i] - done[i])
            if n > 0:
                cache.append(i, n)
                done[i] += n
    toks = [rng.integers(0, 16, q).tolist() for q in qlen]
    batch = build_paged_batch(cache, list(range(len(ctx))), toks, pre)
    T = batch.n_tokens
    q = torch.randn(T, hq * dh, generator=g, device=DEV).to(cache.dtype)
    out = torch.empty_like(q)
    cb = batch.c_struct()
    _lib.call("ms_paged_attention", q.data_ptr(), ctypes.byref(cache.c_struct()), 0,
              ctypes.byref(cb), hq, out.data_ptr(), _lib.stream_ptr())
    torch.cuda.synchronize()
    ref = _reference(cache, q.float().cpu().view(T, hq, dh), ctx, qlen, hq, hkv)
    return out.float().cpu().view(T, hq, dh), ref, cache, q


def _reference(cache, qf: torch.Tensor, ctx: list[int], qlen: list[int], hq: int, hkv: int,
               plant: tuple[int, int] | None = None) -> torch.Tensor:
    """float32 attention on the CPU from a host copy of the pool.  ``plant``
    = (sequence, key) replaces that key and value with the next key's (a
    deliberate one-key error for the negative control)."""
    pool = cache.pool.float().cpu()  # (2, 1, num_blocks, hkv, bs, dh)
    _, _, _, _, bs, dh = pool.shape
    T = qf.shape[0]
    ref = torch.empty(T, hq, dh)
    o = 0
    for b, (c, ql) in enumerate(zip(ctx, qlen)):
        blocks = torch.tensor(cache.tables[b].blocks[: -(-c // bs)], dtype=torch.long)
        kb = pool[0, 0, blocks].permute(0, 2, 1, 3).reshape(-1, hkv, dh)[:c].clone()
        vb = pool[1, 0, blocks].permute(0, 2, 1, 3).reshape(-1, hkv, dh)[:c].clone()
        if plant is not None and plant[0] == b:
            j = plant[1]
            kb[j], vb[j] = kb[j + 1].clone(), vb[j + 1].clone()
        kb = kb.repeat_interleave(hq // hkv, dim=1)  # (c, hq, dh)
        vb = vb.repeat_interleave(hq // hkv, dim=1)
        qb = qf[o : o + ql]  # (ql, hq, dh)
        s = torch.einsum("qhd,khd->hqk", qb, kb) / dh ** 0.5
        pos = torch.arange(c - ql, c)
        mask = torch.arange(c)[None, :] <= pos[:, None]
        s = s.masked_fill(~mask[None], float("-inf"))
        ref[o : o + ql] = torch.einsum("hqk,khd->qhd", torch.softmax(s, -1), vb)
        o += ql
    return ref


def _bf16_ok(got: torch.Tensor, ref: torch.Tensor, qlen: list[int]) -> bool:
    o = 0
    for ql in qlen:
        g, r = got[o : o + ql], ref[o : o + ql]
        tol = 2e-3 * float(r.abs().max()) + 8e-3 * r.abs()
        if not bool(((g - r).abs() <= tol).all()):
            return False
        o += ql
    return True


def _assert_bf16(got, ref, qlen) -> None:
    assert _bf16_ok(got, ref, qlen), float((got - ref).abs().max())


@pytest.mark.parametrize("hq,hkv,dh", [(32, 4, 64), (32, 8, 128), (8, 8, 64), (4, 1, 128)])
@pytest.mark.parametrize("bs", [16, 8, 32, 4])
def test_tensor_core_attention_decode_and_verify(hq, hkv, dh, bs) -> None:
    ctx = [17, 600, 1290, 64, 5, 333]
    qlen = [1, 5, 5, 6, 5, 2]
    got, ref, _, _ = _case("bfloat16", hq, hkv, dh, bs, ctx, qlen, seed=hq + dh + bs)
    _assert_bf16(got, ref, qlen)


@pytest.mark.parametrize("dh", [64, 128])
@pytest.mark.parametrize("qlen", [1, 2, 4, 5])
def test_tensor_core_attention_key_slices(dh: int, qlen: int) -> None:
    """Uniform decode (8 rows: every consumer warp takes a key slice of each
    chunk), two-token (16 rows) and verify (40 rows) batches, with contexts
    that end mid-chunk, mid-slice and on a chunk boundary."""
    ctx = [1, 16, 127, 128, 129, 700, 2049, 40]
    got, ref, _, _ = _case("bfloat16", 32, 4, dh, 16, [max(c, qlen) for c in ctx],
                           [qlen] * len(ctx), seed=dh + qlen)
    _assert_bf16(got, ref, [qlen] * len(ctx))


@pytest.mark.parametrize("hq,hkv,dh", [(16, 4, 64), (8, 2, 128)])
def test_tensor_core_attention_prefill_tiles(hq, hkv, dh) -> None:
    """Long query runs span several 64-row tiles with a causal staircase."""
    ctx = [300, 77, 130]
    qlen = [300, 40, 90]
    got, ref, _, _ = _case("bfloat16", hq, hkv, dh, 16, ctx, qlen, seed=5)
    _assert_bf16(got, ref, qlen)


@pytest.mark.parametrize("dh", [32, 64])
def test_cuda_core_attention_float32(dh: int) -> None:
    got, ref, _, _ = _case("float32", 4, 2, dh, 16, [40, 200], [4, 3], seed=9)
    torch.testing.assert_close(got, ref, rtol=1e-4, atol=1e-5)


@pytest.mark.parametrize("dh", [64, 128])
def test_one_wrong_key_at_long_context_is_detected(dh: int) -> None:
    """Negative control for the bf16 tolerance: the device output passes
    against the true reference, and fails against a reference in which one
    key (and its value) of a 2048-token context was swapped for its
    neighbour's -- the size of a single mask or page error."""
    ctx, qlen = [2048, 900], [5, 5]
    got, ref, cache, q = _case("bfloat16", 32, 4, dh, 16, ctx, qlen, seed=dh)
    assert _bf16_ok(got, ref, qlen)
    qf = q.float().cpu().view(-1, 32, dh)
    for key in (0, 777, 2040):
        bad = _reference(cache, qf, ctx, qlen, 32, 4, plant=(0, key))
        assert not _bf16_ok(got, bad, qlen), key
