"""Paged KV cache: host block allocator and tables, device K/V pools.

Same interface and semantics as MicroServe's ``PagedKVCache`` (reference
src/microserve/cache.py): a refcounted free list of ``num_blocks`` blocks,
per-sequence block tables, logical position ``p`` of a sequence at slot
``table[p // block_size] * block_size + p % block_size``, ``truncate`` for
speculative rollback, ``write``/``gather`` tensor plumbing.

B200 layout.  The device pools are one tensor per cache,
``(n_layers, num_blocks, n_kv_heads, block_size, d_head)``: a (block, kv
head) tile is contiguous, so the attention kernel streams whole tiles.  The
host keeps the tables as a dense ``int32`` array (one row per live
sequence) so a whole batch's slots and tables come out of a few numpy
operations instead of per-token Python loops; ``tables[seq]`` still returns a
:class:`BlockTable` view as in the reference.

A cache built with a non-CUDA device keeps only the host bookkeeping; its
tensor methods raise (there is no CPU compute path).
"""

from __future__ import annotations

import ctypes
from collections.abc import Iterator, Sequence

import numpy as np
import torch

from . import _lib
from .config import CacheConfig, ModelConfig


def _addr(a: np.ndarray) -> int:
    """Address of a contiguous numpy array's data (for the host helpers)."""
    return a.__array_interface__["data"][0]


class OutOfCacheMemory(RuntimeError):
    """Raised when the block pool cannot satisfy an allocation."""


class BlockAllocator:
    """Reference-counted free list over ``num_blocks`` blocks (reference cache.py:32-93).

    Allocation pops from the end of the free list, so block ids come out in
    the same order as the reference's.
    """

    def __init__(self, num_blocks: int) -> None:
        if num_blocks <= 0:
            raise ValueError("num_blocks must be positive")
        self.num_blocks = num_blocks
        self._free: list[int] = list(range(num_blocks))
        self._refcount = np.zeros(num_blocks, dtype=np.int32)

    @property
    def num_free(self) -> int:
        return len(self._free)

    @property
    def num_used(self) -> int:
        return self.num_blocks - len(self._free)

    @property
    def utilization(self) -> float:
        return self.num_used / self.num_blocks

    def refcount(self, block: int) -> int:
        return int(self._refcount[block])

    def allocate(self) -> int:
        if not self._free:
            raise OutOfCacheMemory("block pool exhausted")
        block = self._free.pop()
        self._refcount[block] = 1
        return block

    def allocate_many(self, n: int) -> list[int]:
        if n > len(self._free):
            raise OutOfCacheMemory(f"need {n} blocks, {len(self._free)} free")
        if n <= 0:
            return []
        blocks = self._free[-n:][::-1]
        del self._free[-n:]
        self._refcount[blocks] = 1
        return blocks

    def incref(self, block: int) -> None:
        if self._refcount[block] == 0:
            raise ValueError(f"cannot incref free block {block}")
        self._refcount[block] += 1

    def free(self, block: int) -> None:
        """Drop one reference; the block returns to the pool at zero refs."""
        if self._refcount[block] == 0:
            raise ValueError(f"double free of block {block}")
        self._refcount[block] -= 1
        if self._refcount[block] == 0:
            self._free.append(block)

    def free_many(self, blocks: Sequence[int] | np.ndarray) -> None:
        """``free`` each block in order (blocks reaching zero refs rejoin the
        free list in that order)."""
        arr = np.asarray(blocks, dtype=np.int64).reshape(-1)
        if arr.size == 0:
            return
        if np.unique(arr).size != arr.size:
            for b in arr.tolist():
                self.free(b)
            return
        if np.any(self._refcount[arr] == 0):
            bad = int(arr[self._refcount[arr] == 0][0])
            raise ValueError(f"double free of block {bad}")
        self._refcount[arr] -= 1
        self._free.extend(arr[self._refcount[arr] == 0].tolist())

    def check_invariants(self) -> None:
        """Assert internal consistency; used by tests."""
        if len(set(self._free)) != len(self._free):
            raise AssertionError("duplicate block in free list")
        free = np.asarray(self._free, dtype=np.int64)
        if free.size and np.any(self._refcount[free] != 0):
            raise AssertionError("free block has references")
        held = int(np.count_nonzero(self._refcount > 0))
        if held + len(self._free) != self.num_blocks:
            raise AssertionError("blocks leaked: neither free nor referenced")


class BlockTable:
    """Read-only view of one sequence's row of the dense table."""

    __slots__ = ("_cache", "_row")

    def __init__(self, cache: PagedKVCache, row: int) -> None:
        self._cache = cache
        self._row = row

    @property
    def blocks(self) -> list[int]:
        c = self._cache
        return c._table[self._row, : c._nblk[self._row]].tolist()

    @property
    def num_tokens(self) -> int:
        return int(self._cache._ntok[self._row])

    def capacity(self, block_size: int) -> int:
        return int(self._cache._nblk[self._row]) * block_size

    def slot(self, position: int, block_size: int) -> int:
        return self.blocks[position // block_size] * block_size + position % block_size


class _TableView:
    """``cache.tables``: mapping seq_id -> BlockTable, like the reference's dict."""

    def __init__(self, cache: PagedKVCache) -> None:
        self._cache = cache

    def __getitem__(self, seq_id: int) -> BlockTable:
        return BlockTable(self._cache, self._cache._rows[seq_id])

    def get(self, seq_id: int, default: object = None) -> object:
        row = self._cache._rows.get(seq_id)
        return default if row is None else BlockTable(self._cache, row)

    def __contains__(self, seq_id: object) -> bool:
        return seq_id in self._cache._rows

    def __iter__(self) -> Iterator[int]:
        return iter(list(self._cache._rows))

    def __len__(self) -> int:
        return len(self._cache._rows)

    def keys(self) -> list[int]:
        return list(self._cache._rows)

    def __eq__(self, other: object) -> bool:
        if isinstance(other, _TableView):
            other = {k: (other[k].blocks, other[k].num_tokens) for k in other}
        if not isinstance(other, dict):
            return NotImplemented
        mine = {k: (self[k].blocks, self[k].num_tokens) for k in self}
        theirs = {
            k: (v.blocks, v.num_tokens) if isinstance(v, BlockTable) else v
            for k, v in other.items()
        }
        return mine == theirs


class PagedKVCache:
    """Device K/V storage plus host tables (reference cache.py:110-277)."""

    def __init__(
        self,
        model: ModelConfig,
        cache: CacheConfig,
        device: str | torch.device = "cuda",
    ) -> None:
        if cache.dtype not in _lib.DTYPE_CODES:
            raise ValueError(f"cache dtype {cache.dtype!r} is not supported on the device path")
        if cache.dtype != model.dtype:
            raise ValueError(
                f"cache dtype {cache.dtype!r} must equal the model dtype {model.dtype!r}"
            )
        self.model_cfg = model
        self.cfg = cache
        self.block_size = cache.block_size
        self.dtype = _lib.TORCH_DTYPES[_lib.DTYPE_CODES[cache.dtype]]
        self.device = torch.device(device)
        self.allocator = BlockAllocator(cache.num_blocks)
        self.tables = _TableView(self)

        self._max_blocks = max(1, min(cache.num_blocks, -(-model.max_seq_len // self.block_size)))
        self._rows: dict[int, int] = {}
        self._free_rows: list[int] = []
        # Bumped whenever a sequence gains or loses its table row, so callers
        # may keep ``rows_of`` results while it is unchanged.
        self.generation = 0
        self._table = np.zeros((8, self._max_blocks), dtype=np.int32)
        self._freed = np.empty(cache.num_blocks, dtype=np.int32)  # truncate_many's output
        self._nblk = np.zeros(8, dtype=np.int32)
        self._ntok = np.zeros(8, dtype=np.int64)

        self.pool: torch.Tensor | None = None
        self._c_cache: _lib.MsKVCache | None = None
        if self.device.type == "cuda":
            _lib.require_cuda(self.device)
            shape = (2, model.n_layers, cache.num_blocks, model.kv_heads, self.block_size,
                     model.d_head)
            self.pool = torch.zeros(shape, dtype=self.dtype, device=self.device)
            self._k = [self.pool[0, i] for i in range(model.n_layers)]
            self._v = [self.pool[1, i] for i in range(model.n_layers)]
            self._kptrs = _lib.pointer_array(self._k)
            self._vptrs = _lib.pointer_array(self._v)
            self._c_cache = _lib.MsKVCache(
                model.n_layers, cache.num_blocks, self.block_size, model.kv_heads, model.d_head,
                _lib.DTYPE_CODES[cache.dtype],
                ctypes.cast(self._kptrs, ctypes.POINTER(ctypes.c_void_p)),
                ctypes.cast(self._vptrs, ctypes.POINTER(ctypes.c_void_p)),
            )

    # -- device views ------------------------------------------------------
    @property
    def k_cache(self) -> list[torch.Tensor]:
        """Per-layer key pools, ``(num_blocks, n_kv_heads, block_size, d_head)``."""
        self._need_device()
        return self._k

    @property
    def v_cache(self) -> list[torch.Tensor]:
        self._need_device()
        return self._v

    def c_struct(self) -> _lib.MsKVCache:
        self._need_device()
        assert self._c_cache is not None
        return self._c_cache

    def _need_device(self) -> None:
        if self.pool is None:
            raise RuntimeError(
                "this PagedKVCache was built without a CUDA device; it keeps host tables only"
            )

    # -- capacity accounting ---------------------------------------------
    @property
    def num_free_blocks(self) -> int:
        return self.allocator.num_free

    @property
    def utilization(self) -> float:
        return self.allocator.utilization

    def blocks_needed(self, seq_id: int, num_new_tokens: int) -> int:
        """Extra blocks required to append ``num_new_tokens`` to ``seq_id``."""
        row = self._rows.get(seq_id)
        ntok = 0 if row is None else int(self._ntok[row])
        nblk = 0 if row is None else int(self._nblk[row])
        needed = (ntok + num_new_tokens + self.block_size - 1) // self.block_size
        return max(0, needed - nblk)

    def blocks_needed_many(self, seq_ids: Sequence[int], counts: Sequence[int] | np.ndarray,
                           rows: np.ndarray | None = None) -> int:
        """Total extra blocks ``append_many(seq_ids, counts)`` would take (no change).
        ``rows``: the sequences' ``rows_of`` result, when the caller has it."""
        counts = np.ascontiguousarray(counts, dtype=np.int64)
        if rows is not None:
            rows = np.ascontiguousarray(rows, dtype=np.int64)
            if counts.shape != rows.shape:
                raise ValueError("blocks_needed_many: one count per sequence")
            return int(_lib.load().ms_host_blocks_needed(
                _addr(rows), _addr(counts), len(rows), _addr(self._ntok), _addr(self._nblk),
                self.block_size, None))
        return int(self.blocks_needed_each(seq_ids, counts).sum())

    def blocks_needed_each(self, seq_ids: Sequence[int],
                           counts: Sequence[int] | np.ndarray) -> np.ndarray:
        """``blocks_needed`` of every sequence (int64 array; unknown ids hold 0 tokens)."""
        counts = np.ascontiguousarray(counts, dtype=np.int64)
        get = self._rows.get
        rows = np.fromiter((get(s, -1) for s in seq_ids), dtype=np.int64, count=len(seq_ids))
        known = rows >= 0
        ntok = np.zeros(len(rows), np.int64)
        nblk = np.zeros(len(rows), np.int64)
        ntok[known] = self._ntok[rows[known]]
        nblk[known] = self._nblk[rows[known]]
        need = (ntok + counts + self.block_size - 1) // self.block_size - nblk
        return np.maximum(need, 0)

    def can_append(self, seq_id: int, num_new_tokens: int) -> bool:
        return self.blocks_needed(seq_id, num_new_tokens) <= self.allocator.num_free

    def num_tokens(self, seq_id: int) -> int:
        row = self._rows.get(seq_id)
        return 0 if row is None else int(self._ntok[row])

    # -- rows of the dense table -------------------------------------------
    def _row_of(self, seq_id: int) -> int:
        row = self._rows.get(seq_id)
        if row is not None:
            return row
        if self._free_rows:
            row = self._free_rows.pop()
        else:
            row = len(self._rows)
            if row >= self._table.shape[0]:
                grow = self._table.shape[0]
                self._table = np.concatenate(
                    [self._table, np.zeros((grow, self._table.shape[1]), np.int32)]
                )
                self._nblk = np.concatenate([self._nblk, np.zeros(grow, np.int32)])
                self._ntok = np.concatenate([self._ntok, np.zeros(grow, np.int64)])
        self._rows[seq_id] = row
        self._nblk[row] = 0
        self._ntok[row] = 0
        self.generation += 1
        return row

    def rows_of(self, seq_ids: Sequence[int]) -> np.ndarray:
        """Dense-table rows of ``seq_ids`` (new sequences get a row)."""
        try:
            return np.fromiter(map(self._rows.__getitem__, seq_ids), dtype=np.int64,
                               count=len(seq_ids))
        except KeyError:
            return np.fromiter((self._row_of(s) for s in seq_ids), dtype=np.int64,
                               count=len(seq_ids))

    def rows_if_all_present(self, seq_ids: Sequence[int]) -> np.ndarray | None:
        """``rows_of(seq_ids)`` when every sequence already has a row, else None
        (nothing is created)."""
        rows = self._rows
        if not all(s in rows for s in seq_ids):
            return None
        return self._existing_rows(seq_ids)

    def _existing_rows(self, seq_ids: Sequence[int]) -> np.ndarray:
        """Rows of sequences that must already exist (KeyError otherwise)."""
        return np.fromiter(map(self._rows.__getitem__, seq_ids), dtype=np.int64,
                           count=len(seq_ids))

    def num_tokens_many(self, seq_ids: Sequence[int], rows: np.ndarray | None = None) -> np.ndarray:
        """``num_tokens`` of each sequence (0 for unknown ones), int64."""
        if rows is not None:
            return self._ntok[rows]
        get = self._rows.get
        rows = np.fromiter((get(s, -1) for s in seq_ids), dtype=np.int64, count=len(seq_ids))
        out = np.zeros(len(seq_ids), dtype=np.int64)
        known = rows >= 0
        out[known] = self._ntok[rows[known]]
        return out

    def _ensure_columns(self, n: int) -> None:
        if n > self._table.shape[1]:
            extra = max(n - self._table.shape[1], self._table.shape[1])
            self._table = np.concatenate(
                [self._table, np.zeros((self._table.shape[0], extra), np.int32)], axis=1
            )

    # -- sequence lifecycle ----------------------------------------------
    def append(self, seq_id: int, num_new_tokens: int) -> list[int]:
        """Reserve slots for ``num_new_tokens`` and return their physical ids."""
        return self.append_many([seq_id], [num_new_tokens]).tolist()

    def append_many(self, seq_ids: Sequence[int], counts: Sequence[int] | np.ndarray,
                    rows: np.ndarray | None = None) -> np.ndarray:
        """Vectorised ``append``: slots of every new token, sequence by sequence.

        All-or-nothing: raises :class:`OutOfCacheMemory` before touching any
        table if the pool cannot hold every sequence's new blocks.  ``rows``:
        the (distinct) sequences' ``rows_of`` result, when the caller has it.
        """
        counts = np.ascontiguousarray(counts, dtype=np.int64)
        if rows is None:
            if len(set(seq_ids)) != len(seq_ids):
                raise ValueError("append_many: a sequence appears twice in one batch")
            rows = self.rows_of(seq_ids)
        if counts.size == 0:
            return np.zeros(0, dtype=np.int64)
        rows = np.ascontiguousarray(rows, dtype=np.int64)
        if counts.shape != rows.shape:
            raise ValueError("append_many: one count per sequence")
        lib = _lib.load()
        widest = ctypes.c_int64(0)
        total = int(lib.ms_host_blocks_needed(_addr(rows), _addr(counts), len(rows),
                                              _addr(self._ntok), _addr(self._nblk),
                                              self.block_size, ctypes.addressof(widest)))
        if total > self.allocator.num_free:
            raise OutOfCacheMemory(f"need {total} blocks, {self.allocator.num_free} free")
        if total:
            self._ensure_columns(int(widest.value))
        # sequence i takes the next blocks it needs, in batch order
        blocks = np.asarray(self.allocator.allocate_many(total), dtype=np.int32)
        slots = np.empty(int(counts.sum()), dtype=np.int64)
        rc = lib.ms_host_append(_addr(rows), _addr(counts), len(rows), _addr(self._ntok),
                                _addr(self._nblk), _addr(self._table), self._table.shape[1],
                                self.block_size, _addr(blocks), total, _addr(slots))
        if rc != 0:
            raise RuntimeError(lib.ms_last_error().decode())
        return slots

    def free(self, seq_id: int) -> None:
        row = self._rows.pop(seq_id, None)
        if row is None:
            return
        for block in self._table[row, : self._nblk[row]].tolist():
            self.allocator.free(block)
        self._nblk[row] = 0
        self._ntok[row] = 0
        self._free_rows.append(row)
        self.generation += 1

    def fork(self, parent_id: int, child_id: int) -> None:
        """Let ``child_id`` share every block of ``parent_id`` (copy-on-write
        prefix sharing, reference cache.py:180-187): the blocks gain a
        reference, nothing is copied."""
        if child_id in self._rows:
            raise ValueError(f"sequence {child_id} already exists")
        parent = self._rows[parent_id]
        n = int(self._nblk[parent])
        blocks = self._table[parent, :n].copy()
        for block in blocks.tolist():
            self.allocator.incref(block)
        child = self._row_of(child_id)
        self._table[child, :n] = blocks
        self._nblk[child] = n
        self._ntok[child] = self._ntok[parent]

    def unshare_last_block(self, seq_id: int) -> None:
        """Give ``seq_id`` its own copy of its last block when another
        sequence still references it (reference cache.py:189-204), so that
        appending to it leaves the other sequence's keys and values alone.
        The block's K/V are copied for every layer in one device copy; a
        cache without a device only updates its tables."""
        row = self._rows[seq_id]
        n = int(self._nblk[row])
        if n == 0:
            return
        old = int(self._table[row, n - 1])
        if self.allocator.refcount(old) == 1:
            return
        new = self.allocator.allocate()
        if self.pool is not None:
            self.pool[:, :, new].copy_(self.pool[:, :, old])
        self._table[row, n - 1] = new
        self.allocator.free(old)

    def truncate(self, seq_id: int, num_tokens: int) -> None:
        """Shrink a sequence to ``num_tokens``, releasing blocks past the end."""
        if seq_id not in self._rows:
            raise KeyError(seq_id)
        self.truncate_many([seq_id], [num_tokens])

    def reserve_many(self, seq_ids: Sequence[int], capacity: Sequence[int] | np.ndarray,
                     rows: np.ndarray | None = None) -> bool:
        """Give every sequence blocks for ``capacity[i]`` tokens without
        changing its token count (later appends within it take no block).
        All-or-nothing: False, and no change, if the pool is short."""
        if rows is None:
            rows = self._existing_rows(seq_ids)
        rows = np.ascontiguousarray(rows, dtype=np.int64)
        cap = np.ascontiguousarray(capacity, dtype=np.int64)
        have = self._nblk[rows].astype(np.int64)
        need = np.maximum(0, (cap + self.block_size - 1) // self.block_size - have)
        total = int(need.sum())
        if total == 0:
            return True
        if total > self.allocator.num_free:
            return False
        self._ensure_columns(int((have + need).max()))
        blocks = np.asarray(self.allocator.allocate_many(total), dtype=np.int32)
        first = np.repeat(np.cumsum(need) - need, need)
        cols = np.repeat(have, need) + (np.arange(total) - first)
        self._table[np.repeat(rows, need), cols] = blocks
        self._nblk[rows] = (have + need).astype(np.int32)
        return True

    def truncate_many(self, seq_ids: Sequence[int], num_tokens: Sequence[int] | np.ndarray,
                      rows: np.ndarray | None = None, keep_blocks: bool = False) -> None:
        """Vectorised ``truncate`` (speculative rollback, reference cache.py:210-222).
        ``keep_blocks``: only the token counts shrink; the blocks past the
        new ends stay with their sequences as reserved capacity."""
        if rows is None:
            rows = self._existing_rows(seq_ids)
        rows = np.ascontiguousarray(rows, dtype=np.int64)
        n = np.ascontiguousarray(num_tokens, dtype=np.int64)
        if n.shape != rows.shape:
            raise ValueError("truncate_many: one token count per sequence")
        if keep_blocks:
            if np.any(n > self._ntok[rows]) or np.any(n < 0):
                raise ValueError("truncate cannot grow a sequence")
            self._ntok[rows] = n
            return
        lib = _lib.load()
        for _ in range(2):
            freed = self._freed
            k = int(lib.ms_host_truncate(
                _addr(rows), _addr(n), len(rows), _addr(self._ntok), _addr(self._nblk),
                _addr(self._table), self._table.shape[1], self.block_size, _addr(freed),
                freed.size))
            if k != -2:
                break
            # shared blocks can appear in several rows: make room for every entry
            self._freed = np.empty(int(self._nblk[rows].sum()) + 1, dtype=np.int32)
        if k == -1:
            raise ValueError("truncate cannot grow a sequence")
        if k < 0:
            raise RuntimeError("truncate_many: bad sizes")
        if k:
            # blocks past the new end, sequence by sequence, in table order
            self.allocator.free_many(freed[:k])

    def reset(self) -> None:
        """Drop every sequence and return all blocks to the pool."""
        for seq_id in list(self._rows):
            self.free(seq_id)

    # -- batch tables --------------------------------------------------------
    def table_rows(self, seq_ids: Sequence[int],
                   rows: np.ndarray | None = None) -> tuple[np.ndarray, np.ndarray, int]:
        """Host ``(B, max_blocks)`` int32 tables, ``(B,)`` token counts and the width."""
        if rows is None:
            rows = self._existing_rows(seq_ids)
        width = max(1, int(self._nblk[rows].max())) if len(rows) else 1
        return self._table[rows, :width], self._ntok[rows].copy(), width

    def build_block_tables(self, seq_ids: list[int]) -> tuple[torch.Tensor, torch.Tensor]:
        """Padded ``(B, max_blocks)`` block ids and ``(B,)`` context lengths (int64)."""
        tables, lens, _ = self.table_rows(seq_ids)
        dev = self.device if self.pool is not None else torch.device("cpu")
        # rows past a sequence's last block are stale ids: zero them as the reference does
        tables = tables.copy()
        nblk = self._nblk[[self._rows[s] for s in seq_ids]] if seq_ids else np.zeros(0, np.int32)
        cols = np.arange(tables.shape[1])[None, :]
        tables[cols >= nblk[:, None]] = 0
        return (
            torch.from_numpy(tables.astype(np.int64)).to(dev),
            torch.from_numpy(lens.astype(np.int64)).to(dev),
        )

    # -- tensor plumbing -----------------------------------------------------
    def write(self, layer: int, slots: torch.Tensor, keys: torch.Tensor, values: torch.Tensor) -> None:
        """Scatter ``(T, n_kv_heads, d_head)`` keys/values into the pools at ``slots``."""
        c = self.c_struct()
        slots32 = slots.to(device=self.device, dtype=torch.int32).contiguous()
        k = keys.to(device=self.device, dtype=torch.float32).contiguous()
        v = values.to(device=self.device, dtype=torch.float32).contiguous()
        _lib.call("ms_kv_write", ctypes.byref(c), layer, slots32.data_ptr(), int(slots32.numel()),
                  k.data_ptr(), v.data_ptr(), _lib.stream_ptr(self.device))

    def gather(
        self, layer: int, block_tables: torch.Tensor, max_context: int
    ) -> tuple[torch.Tensor, torch.Tensor]:
        """Materialise ``(B, max_context, n_kv_heads, d_head)`` float32 K and V."""
        c = self.c_struct()
        bt = block_tables.to(device=self.device, dtype=torch.int32).contiguous()
        bsz, max_blocks = bt.shape
        shape = (bsz, max_context, self.model_cfg.kv_heads, self.model_cfg.d_head)
        keys = torch.empty(shape, dtype=torch.float32, device=self.device)
        values = torch.empty(shape, dtype=torch.float32, device=self.device)
        _lib.call("ms_kv_gather", ctypes.byref(c), layer, bt.data_ptr(), bsz, max_blocks,
                  max_context, keys.data_ptr(), values.data_ptr(), _lib.stream_ptr(self.device))
        return keys, values
