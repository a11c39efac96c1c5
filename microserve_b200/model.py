"""Device transformer with the reference's paged-forward API.

Reference: src/microserve/model.py.  Same architecture (pre-norm RMSNorm,
half-split RoPE, SwiGLU, tied embeddings, GPT-2 style init) and the same
``forward_paged(batch, cache) -> (T, vocab)`` float32 logits, computed by
``ms_forward`` in libmicroserve_b200 (one C call per pass).  Additions:
grouped-query attention (``ModelConfig.n_kv_heads``), bf16 weights
(``ModelConfig.dtype``) and ``logit_rows`` to compute logits only for the rows
a caller reads.

Device weight layout:
* ``w_qkv[l]`` = ``[q_proj; k_proj; v_proj]`` stacked along the output dim;
* ``w_gate_up[l]`` interleaves gate and up in groups of 8 rows (rows 16g..16g+7
  are gate 8g..8g+7, rows 16g+8..16g+15 up 8g..8g+7) so the GEMM epilogue sees
  each gate column next to its up column;
* norm weights and RoPE tables are float32.
"""

from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass
from pathlib import Path
from typing import Any

import numpy as np
import torch

from . import _lib
from .cache import PagedKVCache
from .config import ModelConfig


@dataclass
class PagedBatch:
    """Flattened description of one paged pass (reference model.py:33-66).

    Sequence ``b`` contributes ``q_lens[b]`` consecutive tokens.  Device
    arrays are int32 (the kernels' index type); ``max_q`` and ``n_tokens``
    are host integers so no device sync is needed to launch.
    """

    input_ids: torch.Tensor  # (T,) int32
    positions: torch.Tensor  # (T,) int32 absolute positions
    slot_mapping: torch.Tensor  # (T,) int32 physical slots
    block_tables: torch.Tensor  # (B, max_blocks) int32
    context_lens: torch.Tensor  # (B,) int32, context after this pass's writes
    q_lens: torch.Tensor  # (B,) int32
    q_start: torch.Tensor  # (B + 1,) int32 prefix sums of q_lens
    max_q: int
    n_tokens: int
    max_context: int = 0  # max of context_lens (0: unknown, bounded by the table)

    @property
    def batch_size(self) -> int:
        return int(self.q_lens.numel())

    def scatter_index(self) -> torch.Tensor:
        """Flat token index -> row-major index into a ``(B, max_q)`` grid."""
        dev = self.q_lens.device
        ql = self.q_lens.long()
        rows = torch.repeat_interleave(torch.arange(self.batch_size, device=dev), ql)
        starts = torch.repeat_interleave(self.q_start[:-1].long(), ql)
        cols = torch.arange(self.n_tokens, device=dev) - starts
        return rows * self.max_q + cols

    def c_struct(self) -> _lib.MsBatch:
        return _lib.MsBatch(
            self.n_tokens,
            self.batch_size,
            int(self.block_tables.shape[1]),
            self.max_q,
            self.max_context,
            0,
            self.input_ids.data_ptr(),
            self.positions.data_ptr(),
            self.slot_mapping.data_ptr(),
            self.q_start.data_ptr(),
            self.context_lens.data_ptr(),
            self.block_tables.data_ptr(),
        )


def rope_tables(d_head: int, max_seq_len: int, theta: float) -> tuple[torch.Tensor, torch.Tensor]:
    """float32 cos/sin tables, computed on the host by reference model.py:92-98's formula."""
    if d_head % 2 != 0:
        raise ValueError("rotary embeddings need an even head dimension")
    inv_freq = 1.0 / (theta ** (torch.arange(0, d_head, 2, dtype=torch.float32) / d_head))
    pos = torch.arange(max_seq_len, dtype=torch.float32)
    angles = torch.outer(pos, inv_freq)
    return angles.cos().contiguous(), angles.sin().contiguous()


def interleave_gate_up(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    ff, d = gate.shape
    if ff % 8:
        raise ValueError(f"d_ff must be a multiple of 8 (got {ff})")
    return torch.stack([gate.reshape(ff // 8, 8, d), up.reshape(ff // 8, 8, d)], dim=1).reshape(
        2 * ff, d
    )


def split_gate_up(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    two_ff, d = w.shape
    v = w.reshape(two_ff // 16, 2, 8, d)
    return v[:, 0].reshape(-1, d), v[:, 1].reshape(-1, d)


# ModelConfig fields the reference's config class does not have; a checkpoint
# stores them under EXTRA_CONFIG_KEY so the reference can still load it.
ADDED_CONFIG_FIELDS = ("n_kv_heads", "dtype")
EXTRA_CONFIG_KEY = "microserve_b200_config"


def checkpoint_payload(cfg: ModelConfig, state: dict[str, torch.Tensor],
                       extra: dict[str, Any] | None = None) -> dict[str, Any]:
    """``{"config": ..., "state_dict": ..., EXTRA_CONFIG_KEY: ..., **extra}``:
    the reference's checkpoint layout (model.py:357-363), with ``config``
    limited to the reference's ``ModelConfig`` fields."""
    c = dict(cfg.__dict__)
    added = {k: c.pop(k) for k in ADDED_CONFIG_FIELDS}
    return {"config": c, "state_dict": state, EXTRA_CONFIG_KEY: added, **(extra or {})}


def load_checkpoint(path: str | Path, dtype: str | None = None
                    ) -> tuple[ModelConfig, dict[str, torch.Tensor]]:
    """The config and state dict of a checkpoint in the reference's format
    (reference model.py:356-373).  Read with ``weights_only=True``: plain
    values and tensors load, any other pickled object is refused.  The
    ``ModelConfig`` fields this package adds (``n_kv_heads``, ``dtype``) are
    read from the payload's ``EXTRA_CONFIG_KEY`` entry when present, else
    keep their defaults; ``dtype`` overrides the stored one."""
    payload = torch.load(path, map_location="cpu", weights_only=True)
    kw = dict(payload["config"])
    kw.update(payload.get(EXTRA_CONFIG_KEY, {}))
    if dtype is not None:
        kw["dtype"] = dtype
    return ModelConfig(**kw), payload["state_dict"]


class Transformer:
    """Decoder on one CUDA device; ``forward_paged`` is the hot path."""

    def __init__(
        self,
        cfg: ModelConfig,
        device: str | torch.device = "cuda",
        seed: int | None = 0,
        init: bool = True,
    ) -> None:
        if not cfg.tie_weights:
            raise ValueError("only tied input/output embeddings are supported")
        self.device = _lib.require_cuda(device)
        self.cfg = cfg
        self.dtype_code = _lib.DTYPE_CODES[cfg.dtype]
        self.dtype = _lib.TORCH_DTYPES[self.dtype_code]
        self._ws: torch.Tensor | None = None
        self._empty_rows: torch.Tensor | None = None
        if init:
            self._random_init(seed)

    # -- weights -------------------------------------------------------------
    def _random_init(self, seed: int | None) -> None:
        """N(0, 0.02) everywhere, N(0, 0.02/sqrt(2L)) for o_proj and down_proj,
        ones for norms (reference model.py:279-299), drawn on the device."""
        cfg = self.cfg
        gen = torch.Generator(device=self.device)
        gen.manual_seed(0 if seed is None else seed)
        d, hq, hkv, dh, ff = cfg.d_model, cfg.n_heads, cfg.kv_heads, cfg.d_head, cfg.ffn_hidden

        def normal(shape: tuple[int, ...], std: float) -> torch.Tensor:
            t = torch.randn(shape, generator=gen, device=self.device, dtype=torch.float32)
            return (t * std).to(self.dtype)

        res = 0.02 / math.sqrt(2 * cfg.n_layers)
        self.embed = normal((cfg.vocab_size, d), 0.02)
        self.w_qkv = [normal(((hq + 2 * hkv) * dh, d), 0.02) for _ in range(cfg.n_layers)]
        self.w_o = [normal((d, hq * dh), res) for _ in range(cfg.n_layers)]
        self.w_gate_up = [normal((2 * ff, d), 0.02) for _ in range(cfg.n_layers)]
        self.w_down = [normal((d, ff), res) for _ in range(cfg.n_layers)]
        ones = lambda: torch.ones(d, dtype=torch.float32, device=self.device)  # noqa: E731
        self.attn_norm = [ones() for _ in range(cfg.n_layers)]
        self.ffn_norm = [ones() for _ in range(cfg.n_layers)]
        self.final_norm = ones()
        self._finish()

    @classmethod
    def from_state_dict(
        cls, cfg: ModelConfig, state: dict[str, Any], device: str | torch.device = "cuda"
    ) -> Transformer:
        """Load a reference-format state dict (``blocks.{i}.attn.q_proj.weight`` ...)."""
        m = cls(cfg, device, init=False)

        def get(name: str, dtype: torch.dtype) -> torch.Tensor:
            t = state[name]
            t = torch.as_tensor(np.asarray(t)) if not isinstance(t, torch.Tensor) else t
            return t.detach().to(device=m.device, dtype=dtype).contiguous()

        dt = m.dtype
        m.embed = get("embed.weight", dt)
        m.w_qkv, m.w_o, m.w_gate_up, m.w_down, m.attn_norm, m.ffn_norm = [], [], [], [], [], []
        for i in range(cfg.n_layers):
            p = f"blocks.{i}."
            q, k, v = (get(p + f"attn.{n}_proj.weight", dt) for n in "qkv")
            m.w_qkv.append(torch.cat([q, k, v], 0).contiguous())
            m.w_o.append(get(p + "attn.o_proj.weight", dt))
            m.w_gate_up.append(
                interleave_gate_up(get(p + "ffn.gate_proj.weight", dt), get(p + "ffn.up_proj.weight", dt))
                .contiguous()
            )
            m.w_down.append(get(p + "ffn.down_proj.weight", dt))
            m.attn_norm.append(get(p + "attn_norm.weight", torch.float32))
            m.ffn_norm.append(get(p + "ffn_norm.weight", torch.float32))
        m.final_norm = get("norm.weight", torch.float32)
        m._finish()
        return m

    # -- checkpoints (reference model.py:356-373) ------------------------------
    def save(self, path: str | Path, extra: dict[str, Any] | None = None) -> None:
        """Write the reference's checkpoint format: ``{"config": ...,
        "state_dict": ..., **extra}`` with float32 weights.

        ``config`` holds only the reference's ``ModelConfig`` fields, so the
        reference's ``ModelConfig(**payload["config"])`` (model.py:369-370)
        loads the file; the fields this package adds go under
        ``EXTRA_CONFIG_KEY``, which the reference ignores."""
        torch.save(checkpoint_payload(self.cfg, self.state_dict(), extra), path)

    @classmethod
    def from_checkpoint(
        cls, path: str | Path, device: str | torch.device = "cuda", dtype: str | None = None
    ) -> Transformer:
        """Load a checkpoint written by the reference's ``Transformer.save`` (or
        :meth:`save`).  ``dtype`` overrides the stored compute dtype."""
        cfg, state = load_checkpoint(path, dtype)
        return cls.from_state_dict(cfg, state, device)

    def state_dict(self) -> dict[str, torch.Tensor]:
        """Reference-format float32 state dict on the host (for the checker)."""
        cfg = self.cfg
        hq, hkv, dh = cfg.n_heads, cfg.kv_heads, cfg.d_head
        f = lambda t: t.detach().float().cpu()  # noqa: E731
        embed = f(self.embed)
        # tied: one storage under both names, as the reference's module shares it
        out = {"embed.weight": embed, "norm.weight": f(self.final_norm), "lm_head.weight": embed}
        for i in range(cfg.n_layers):
            p = f"blocks.{i}."
            qkv = f(self.w_qkv[i])
            out[p + "attn.q_proj.weight"] = qkv[: hq * dh]
            out[p + "attn.k_proj.weight"] = qkv[hq * dh : (hq + hkv) * dh]
            out[p + "attn.v_proj.weight"] = qkv[(hq + hkv) * dh :]
            out[p + "attn.o_proj.weight"] = f(self.w_o[i])
            gate, up = split_gate_up(f(self.w_gate_up[i]))
            out[p + "ffn.gate_proj.weight"] = gate
            out[p + "ffn.up_proj.weight"] = up
            out[p + "ffn.down_proj.weight"] = f(self.w_down[i])
            out[p + "attn_norm.weight"] = f(self.attn_norm[i])
            out[p + "ffn_norm.weight"] = f(self.ffn_norm[i])
        return out

    def _finish(self) -> None:
        cfg = self.cfg
        cos, sin = rope_tables(cfg.d_head, cfg.max_seq_len, cfg.rope_theta)
        self.rope_cos = cos.to(self.device)
        self.rope_sin = sin.to(self.device)
        self._arrays = {
            "attn_norm": _lib.pointer_array(self.attn_norm),
            "w_qkv": _lib.pointer_array(self.w_qkv),
            "w_o": _lib.pointer_array(self.w_o),
            "ffn_norm": _lib.pointer_array(self.ffn_norm),
            "w_gate_up": _lib.pointer_array(self.w_gate_up),
            "w_down": _lib.pointer_array(self.w_down),
        }
        cast = lambda a: ctypes.cast(a, ctypes.POINTER(ctypes.c_void_p))  # noqa: E731
        a = self._arrays
        self._c_model = _lib.MsModel(
            cfg.vocab_size, cfg.d_model, cfg.n_layers, cfg.n_heads, cfg.kv_heads, cfg.d_head,
            cfg.ffn_hidden, cfg.max_seq_len, self.dtype_code, cfg.norm_eps,
            self.embed.data_ptr(), self.final_norm.data_ptr(), self.rope_cos.data_ptr(),
            self.rope_sin.data_ptr(), cast(a["attn_norm"]), cast(a["w_qkv"]), cast(a["w_o"]),
            cast(a["ffn_norm"]), cast(a["w_gate_up"]), cast(a["w_down"]),
        )

    # -- module-like conveniences ---------------------------------------------
    def eval(self) -> Transformer:
        return self

    def num_parameters(self) -> int:
        return self.cfg.n_params()

    def weight_bytes(self) -> int:
        ts = [self.embed, *self.w_qkv, *self.w_o, *self.w_gate_up, *self.w_down]
        return sum(t.numel() * t.element_size() for t in ts)

    # -- forward ---------------------------------------------------------------
    def _placeholder(self) -> torch.Tensor:
        """A 4-byte device buffer whose pointer stands for an empty argument."""
        if self._empty_rows is None:
            self._empty_rows = torch.zeros(1, dtype=torch.int32, device=self.device)
        return self._empty_rows

    def workspace(self, n_tokens: int, n_rows: int, attn_scratch: int = 0) -> torch.Tensor:
        """Grow-only device workspace: ms_forward's carve plus ``attn_scratch``
        bytes for the attention's split-KV partials."""
        need = int(_lib.load().ms_forward_workspace_size(ctypes.byref(self._c_model), n_tokens,
                                                           n_rows))
        need += attn_scratch
        if self._ws is None or self._ws.numel() < need:
            self._ws = torch.empty(max(need, 1), dtype=torch.uint8, device=self.device)
        return self._ws

    def forward_paged(
        self,
        batch: PagedBatch,
        cache: PagedKVCache,
        logit_rows: torch.Tensor | None = None,
        out: torch.Tensor | None = None,
        out_row_stride: int = 0,
    ) -> torch.Tensor:
        """Paged forward; returns float32 logits ``(rows, vocab)``.

        ``logit_rows`` (int32, device) selects which flat token rows get
        logits (default: all, as the reference).  ``out`` may be a
        preallocated buffer whose rows are ``out_row_stride`` apart.
        """
        n_rows = batch.n_tokens if logit_rows is None else int(logit_rows.numel())
        if out is None:
            out = torch.empty((n_rows, self.cfg.vocab_size), dtype=torch.float32,
                              device=self.device)
            out_row_stride = 0
        rows_ptr, out_ptr = _lib.ptr(logit_rows), out.data_ptr()
        if logit_rows is not None and n_rows == 0:
            # No logits wanted.  An empty tensor's data pointer is null, and a
            # null row list means "every row": pass a real (unused) row list
            # and output of length 0 instead.
            rows_ptr, out_ptr = self._placeholder().data_ptr(), self._placeholder().data_ptr()
        cb = batch.c_struct()
        cc = cache.c_struct()
        scratch = int(_lib.load().ms_attention_scratch_size(ctypes.byref(cc), self.cfg.n_heads,
                                                            ctypes.byref(cb)))
        ws = self.workspace(batch.n_tokens, n_rows, scratch)
        _lib.call(
            "ms_forward", ctypes.byref(self._c_model), ctypes.byref(cache.c_struct()),
            ctypes.byref(cb), rows_ptr, n_rows, out_ptr, out_row_stride,
            ws.data_ptr(), ws.numel(), _lib.stream_ptr(self.device),
        )
        return out
