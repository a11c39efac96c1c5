"""ms_forward_static_scratch: the paged forward for callers that cannot allocate.

Some hosts reach this library only through its C ABI (an FFI binding with no
CUDA allocator of its own), and some serving loops must not call cudaMalloc
once they run.  For them the forward keeps its scratch in a 16 MiB array
compiled into the library.  These tests call that entry point through the C
ABI and check it against ms_forward with a caller-provided workspace, on two
calls in a row (the array keeps the previous call's contents), and that an
oversized batch is refused before anything runs.  This file is collected
last on purpose and needs no state from other test files.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"
FP32_TOL = dict(rtol=1e-4, atol=1e-5)
BF16_TOL = dict(rtol=2e-2, atol=2e-2)


def _setup(dtype: str, d_model: int, n_heads: int, n_kv: int, lens: list[int]):
    from microserve_b200.batching import build_paged_batch
    from microserve_b200.cache import PagedKVCache
    from microserve_b200.config import CacheConfig, ModelConfig
    from microserve_b200.model import Transformer

    cfg = ModelConfig(vocab_size=500, n_layers=3, d_model=d_model, n_heads=n_heads,
                      n_kv_heads=n_kv, d_ff=4 * d_model, max_seq_len=512, dtype=dtype)
    model = Transformer(cfg, DEV, seed=3)
    cache = PagedKVCache(cfg, CacheConfig(16, 256, dtype), DEV)
    rng = np.random.default_rng(0)
    seqs = [rng.integers(0, 500, n).tolist() for n in lens]
    batch = build_paged_batch(cache, list(range(len(seqs))), seqs, [0] * len(seqs))
    return model, cache, batch


def _static_forward(model, cache, batch, rows: torch.Tensor | None) -> tuple[int, torch.Tensor]:
    from microserve_b200 import _lib

    n = batch.n_tokens if rows is None else int(rows.numel())
    out = torch.full((n, model.cfg.vocab_size), float("nan"), dtype=torch.float32, device=DEV)
    cb = batch.c_struct()
    rc = _lib.load().ms_forward_static_scratch(
        ctypes.byref(model._c_model), ctypes.byref(cache.c_struct()), ctypes.byref(cb),
        _lib.ptr(rows), n, out.data_ptr(), 0, _lib.stream_ptr())
    torch.cuda.synchronize()
    return rc, out


@pytest.mark.parametrize("dtype,d_model,n_heads,n_kv,tol", [
    ("float32", 128, 4, 4, FP32_TOL),
    ("bfloat16", 512, 8, 2, BF16_TOL),
])
def test_static_scratch_forward_matches_ms_forward(dtype, d_model, n_heads, n_kv, tol) -> None:
    model, cache, batch = _setup(dtype, d_model, n_heads, n_kv, [37, 5, 120])
    want = model.forward_paged(batch, cache).cpu().numpy()
    rows = torch.tensor([36, 41, 161], dtype=torch.int32, device=DEV)
    want_rows = model.forward_paged(batch, cache, logit_rows=rows).cpu().numpy()
    for _ in range(2):  # the second call starts from the first call's scratch contents
        rc, got = _static_forward(model, cache, batch, None)
        assert rc == 0
        np.testing.assert_allclose(got.cpu().numpy(), want, **tol)
        rc, got_rows = _static_forward(model, cache, batch, rows)
        assert rc == 0
        np.testing.assert_allclose(got_rows.cpu().numpy(), want_rows, **tol)


def test_static_scratch_refuses_batches_beyond_its_size() -> None:
    from microserve_b200 import _lib

    model, cache, batch = _setup("float32", 128, 4, 4, [200, 200, 200])
    need = _lib.load().ms_forward_workspace_size(ctypes.byref(model._c_model), 4000, 4000)
    assert need > 16 << 20
    big = type(batch)(batch.input_ids, batch.positions, batch.slot_mapping, batch.block_tables,
                      batch.context_lens, batch.q_lens, batch.q_start, batch.max_q, 4000)
    rc, out = _static_forward(model, cache, big, None)
    assert rc == _lib.MS_ERR_TOO_LARGE
    assert b"16 MiB" in _lib.load().ms_last_error()
    assert torch.isnan(out).all()  # nothing ran
