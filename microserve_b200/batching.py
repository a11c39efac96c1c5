"""Turn (sequence, new tokens) pairs into a device :class:`PagedBatch`.

Same contract as reference src/microserve/batching.py:19-68: reserve cache
slots for each sequence's new tokens (``start_positions[i]`` must equal the
tokens already cached) and flatten them into one batch.  The per-token work
is vectorised in numpy and the batch's int32 arrays reach the device in one
pinned host-to-device copy.
"""

from __future__ import annotations

from collections.abc import Sequence

import numpy as np
import torch

from .cache import PagedKVCache
from .model import PagedBatch


class HostStaging:
    """A growable pinned host buffer plus its device twin, for one-copy uploads."""

    def __init__(self, device: torch.device) -> None:
        self.device = device
        self._host: torch.Tensor | None = None
        self._dev: torch.Tensor | None = None
        self._copied: torch.cuda.Event | None = None

    def upload(self, blob: np.ndarray) -> torch.Tensor:
        """Copy an int32 array to the device (stream-ordered) and return the view.

        The device buffer is reused: a caller must not upload again while
        kernels that read the previous upload are still to be launched on
        another stream.
        """
        n = int(blob.size)
        if self._host is None or self._host.numel() < n:
            cap = max(n, 1024, 2 * (0 if self._host is None else self._host.numel()))
            if self._copied is not None:
                self._copied.synchronize()
            self._host = torch.empty(cap, dtype=torch.int32, pin_memory=True)
            self._dev = torch.empty(cap, dtype=torch.int32, device=self.device)
        assert self._dev is not None
        if self._copied is not None:
            self._copied.synchronize()  # the previous copy out of the pinned buffer is done
        self._host[:n].numpy()[:] = blob.reshape(-1)
        self._dev[:n].copy_(self._host[:n], non_blocking=True)
        self._copied = torch.cuda.Event()
        self._copied.record(torch.cuda.current_stream(self.device))
        return self._dev[:n]


    def upload_on(self, blob: np.ndarray, side: torch.cuda.Stream,
                  after: torch.cuda.Event | None) -> torch.Tensor:
        """Like :meth:`upload`, but the copy runs on ``side`` as soon as the
        consuming (current) stream has passed ``after`` -- the point after
        which nothing enqueued there reads the previous upload -- instead of
        in the consuming stream's order.  The consuming stream waits for the
        copy before its next work, so the copy overlaps the kernels enqueued
        between ``after`` and now.  ``after=None``: the copy waits for
        everything enqueued on the consuming stream so far."""
        n = int(blob.size)
        main = torch.cuda.current_stream(self.device)
        if self._host is None or self._host.numel() < n:
            # the buffers are replaced: nothing queued may still read the old ones
            main.synchronize()
            if self._copied is not None:
                self._copied.synchronize()
            cap = max(n, 1024, 2 * (0 if self._host is None else self._host.numel()))
            self._host = torch.empty(cap, dtype=torch.int32, pin_memory=True)
            self._dev = torch.empty(cap, dtype=torch.int32, device=self.device)
        assert self._dev is not None
        if self._copied is not None:
            self._copied.synchronize()  # the previous copy out of the pinned buffer is done
        self._host[:n].numpy()[:] = blob.reshape(-1)
        if after is not None:
            side.wait_event(after)
        else:
            side.wait_stream(main)
        with torch.cuda.stream(side):
            self._dev[:n].copy_(self._host[:n], non_blocking=True)
        done = torch.cuda.Event()
        done.record(side)
        main.wait_event(done)
        self._copied = done
        return self._dev[:n]


def pack_int32(parts: list[np.ndarray]) -> tuple[np.ndarray, list[tuple[int, int]]]:
    """Concatenate int32 arrays; return the blob and (offset, size) per part."""
    spans = []
    off = 0
    for p in parts:
        spans.append((off, int(p.size)))
        off += int(p.size)
    blob = np.empty(off, dtype=np.int32)
    for (o, n), p in zip(spans, parts, strict=True):
        blob[o : o + n] = p.reshape(-1)
    return blob, spans


def batch_from_host(
    dev_blob: torch.Tensor,
    spans: list[tuple[int, int]],
    n_seqs: int,
    width: int,
    max_q: int,
    n_tokens: int,
    max_context: int = 0,
) -> PagedBatch:
    """Device views of a packed [ids, positions, slots, q_start, ctx, q_lens, tables] blob."""
    v = [dev_blob[o : o + n] for o, n in spans]
    return PagedBatch(
        input_ids=v[0],
        positions=v[1],
        slot_mapping=v[2],
        q_start=v[3],
        context_lens=v[4],
        q_lens=v[5],
        block_tables=v[6].view(n_seqs, width),
        max_q=max_q,
        n_tokens=n_tokens,
        max_context=max_context,
    )


def host_batch_arrays(
    cache: PagedKVCache,
    seq_ids: Sequence[int],
    token_lists: Sequence[Sequence[int]],
    start_positions: Sequence[int],
) -> tuple[list[np.ndarray], int, int, int]:
    """Reserve slots and build the host int32 arrays of a batch."""
    if not (len(seq_ids) == len(token_lists) == len(start_positions)):
        raise ValueError("seq_ids, token_lists and start_positions must align")
    q_lens = np.fromiter((len(t) for t in token_lists), dtype=np.int64, count=len(token_lists))
    for seq_id, n in zip(seq_ids, q_lens, strict=True):
        if n == 0:
            raise ValueError(f"sequence {seq_id} contributes no tokens")
    cached = np.fromiter((cache.num_tokens(s) for s in seq_ids), dtype=np.int64, count=len(seq_ids))
    starts = np.asarray(start_positions, dtype=np.int64)
    bad = np.nonzero(cached != starts)[0]
    if bad.size:
        i = int(bad[0])
        raise ValueError(
            f"sequence {seq_ids[i]}: cache holds {cached[i]} tokens but the batch "
            f"claims to start at position {starts[i]}"
        )
    slots = cache.append_many(seq_ids, q_lens)
    n_tokens = int(q_lens.sum())
    ids = np.fromiter((t for toks in token_lists for t in toks), dtype=np.int32, count=n_tokens)
    seq_idx = np.repeat(np.arange(len(seq_ids)), q_lens)
    q_start = np.zeros(len(seq_ids) + 1, dtype=np.int64)
    np.cumsum(q_lens, out=q_start[1:])
    positions = starts[seq_idx] + np.arange(n_tokens) - q_start[:-1][seq_idx]
    tables, lens, width = cache.table_rows(seq_ids)
    parts = [ids, positions.astype(np.int32), slots.astype(np.int32), q_start.astype(np.int32),
             lens.astype(np.int32), q_lens.astype(np.int32), tables]
    max_q = int(q_lens.max()) if len(q_lens) else 0
    return parts, width, max_q, n_tokens


def build_paged_batch(
    cache: PagedKVCache,
    seq_ids: Sequence[int],
    token_lists: Sequence[Sequence[int]],
    start_positions: Sequence[int],
    device: str | torch.device | None = None,
    staging: HostStaging | None = None,
) -> PagedBatch:
    """Allocate slots for ``token_lists`` and flatten them into one device batch."""
    parts, width, max_q, n_tokens = host_batch_arrays(cache, seq_ids, token_lists, start_positions)
    blob, spans = pack_int32(parts)
    dev = torch.device(device) if device is not None else cache.device
    if staging is not None:
        dev_blob = staging.upload(blob)
    else:
        dev_blob = torch.from_numpy(blob).to(dev)
    return batch_from_host(dev_blob, spans, len(seq_ids), width, max_q, n_tokens,
                           int(parts[4].max()) if len(seq_ids) else 0)


def last_token_rows(q_lens: torch.Tensor) -> torch.Tensor:
    """Row indices of each sequence's final query token in the flat output."""
    return torch.cumsum(q_lens.long(), 0) - 1
