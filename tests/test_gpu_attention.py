"""ms_paged_attention against a float32 torch reference of the same bf16 K/V.

bf16 caches with d_head 64/128 take the tensor-core kernels (TMA-fed for
power-of-two block sizes 8..64, cp.async-fed otherwise); float32 and other
head sizes the CUDA-core kernel.  The reference gathers each sequence's keys
through its block table and applies the reference's causal rule (key j is
visible to a query at absolute position p iff j <= p)."""

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
    # reference
    tables, _ = cache.build_block_tables(list(range(len(ctx))))
    K, V = cache.gather(0, tables, max(ctx))
    ref = torch.empty(T, hq, dh, device=DEV)
    qf = q.float().view(T, hq, dh)
    o = 0
    for b, (c, ql) in enumerate(zip(ctx, qlen)):
        kb = K[b, :c].repeat_interleave(hq // hkv, dim=1)  # (c, hq, dh)
        vb = V[b, :c].repeat_interleave(hq // hkv, dim=1)
        qb = qf[o : o + ql]  # (ql, hq, dh)
        s = torch.einsum("qhd,khd->hqk", qb, kb) / dh ** 0.5
        pos = torch.arange(c - ql, c, device=DEV)
        mask = torch.arange(c, device=DEV)[None, :] <= pos[:, None]
        s = s.masked_fill(~mask[None], float("-inf"))
        ref[o : o + ql] = torch.einsum("hqk,khd->qhd", torch.softmax(s, -1), vb)
        o += ql
    return out.float().view(T, hq, dh), ref


@pytest.mark.parametrize("hq,hkv,dh", [(32, 4, 64), (32, 8, 128), (8, 8, 64), (4, 1, 128)])
@pytest.mark.parametrize("bs", [16, 8, 32, 4])
def test_tensor_core_attention_decode_and_verify(hq, hkv, dh, bs) -> None:
    ctx = [17, 600, 1290, 64, 5, 333]
    qlen = [1, 5, 5, 6, 5, 2]
    got, ref = _case("bfloat16", hq, hkv, dh, bs, ctx, qlen, seed=hq + dh + bs)
    torch.testing.assert_close(got, ref, rtol=2e-2, atol=2e-2)


@pytest.mark.parametrize("dh", [64, 128])
@pytest.mark.parametrize("qlen", [1, 2, 4, 5])
def test_tensor_core_attention_key_slices(dh: int, qlen: int) -> None:
    """Uniform decode (8 rows: every consumer warp takes a key slice of each
    chunk), two-token (16 rows) and verify (40 rows) batches, with contexts
    that end mid-chunk, mid-slice and on a chunk boundary."""
    ctx = [1, 16, 127, 128, 129, 700, 2049, 40]
    got, ref = _case("bfloat16", 32, 4, dh, 16, [max(c, qlen) for c in ctx], [qlen] * len(ctx),
                     seed=dh + qlen)
    torch.testing.assert_close(got, ref, rtol=2e-2, atol=2e-2)


@pytest.mark.parametrize("hq,hkv,dh", [(16, 4, 64), (8, 2, 128)])
def test_tensor_core_attention_prefill_tiles(hq, hkv, dh) -> None:
    """Long query runs span several 64-row tiles with a causal staircase."""
    ctx = [300, 77, 130]
    qlen = [300, 40, 90]
    got, ref = _case("bfloat16", hq, hkv, dh, 16, ctx, qlen, seed=5)
    torch.testing.assert_close(got, ref, rtol=2e-2, atol=2e-2)


@pytest.mark.parametrize("dh", [32, 64])
def test_cuda_core_attention_float32(dh: int) -> None:
    got, ref = _case("float32", 4, 2, dh, 16, [40, 200], [4, 3], seed=9)
    torch.testing.assert_close(got, ref, rtol=1e-4, atol=1e-5)
