"""Configuration dataclasses, field-for-field compatible with MicroServe's.

Reference: src/microserve/config.py.  The same names, defaults and
validation, so that an ``EngineConfig`` written for MicroServe loads here
unchanged.  Two additions for the B200 path:

* ``ModelConfig.n_kv_heads`` -- grouped-query attention (``None`` = one KV
  head per query head, the reference's multi-head attention);
* ``ModelConfig.dtype`` -- weight/activation dtype of the device model
  (``"float32"`` or ``"bfloat16"``); the KV cache must use the same dtype.

``EngineConfig.device`` defaults to ``"cuda"``: there is no CPU compute path.
"""

from __future__ import annotations

import json
from dataclasses import asdict, dataclass, field, fields
from pathlib import Path
from typing import Any

_DTYPES = ("float32", "bfloat16")


def _round_to_multiple(value: float, multiple: int) -> int:
    return int(multiple * round(value / multiple))


@dataclass
class ModelConfig:
    """Shape of a pre-norm RMSNorm/RoPE/SwiGLU decoder (reference config.py:19-65)."""

    vocab_size: int = 65
    n_layers: int = 4
    d_model: int = 128
    n_heads: int = 4
    d_ff: int | None = None
    max_seq_len: int = 1024
    rope_theta: float = 10_000.0
    norm_eps: float = 1e-5
    tie_weights: bool = True
    dropout: float = 0.0
    n_kv_heads: int | None = None
    dtype: str = "float32"

    def __post_init__(self) -> None:
        if self.d_model % self.n_heads != 0:
            raise ValueError(
                f"d_model={self.d_model} not divisible by n_heads={self.n_heads}"
            )
        if self.d_ff is None:
            # SwiGLU has three matrices, so the 4x expansion is scaled by 2/3.
            self.d_ff = _round_to_multiple(8 * self.d_model / 3, 32)
        if self.n_kv_heads is None:
            self.n_kv_heads = self.n_heads
        if self.n_heads % self.n_kv_heads != 0:
            raise ValueError(
                f"n_heads={self.n_heads} not divisible by n_kv_heads={self.n_kv_heads}"
            )
        if self.dtype not in _DTYPES:
            raise ValueError(f"dtype must be one of {_DTYPES}, got {self.dtype!r}")

    @property
    def d_head(self) -> int:
        return self.d_model // self.n_heads

    @property
    def ffn_hidden(self) -> int:
        assert self.d_ff is not None
        return self.d_ff

    @property
    def kv_heads(self) -> int:
        assert self.n_kv_heads is not None
        return self.n_kv_heads

    def n_params(self) -> int:
        """Analytic parameter count (excludes buffers)."""
        kv = self.kv_heads * self.d_head
        emb = self.vocab_size * self.d_model
        attn = self.n_layers * (2 * self.d_model * self.d_model + 2 * self.d_model * kv)
        ffn = self.n_layers * 3 * self.d_model * self.ffn_hidden
        norms = self.n_layers * 2 * self.d_model + self.d_model
        head = 0 if self.tie_weights else self.vocab_size * self.d_model
        return emb + attn + ffn + norms + head


@dataclass
class CacheConfig:
    """Paged KV cache geometry (reference config.py:68-87)."""

    block_size: int = 16
    num_blocks: int = 512
    dtype: str = "float32"

    def bytes_for(self, model: ModelConfig) -> int:
        itemsize = {"float32": 4, "float16": 2, "bfloat16": 2}[self.dtype]
        per_slot = model.kv_heads * model.d_head
        return 2 * model.n_layers * self.num_blocks * self.block_size * per_slot * itemsize

    @property
    def num_slots(self) -> int:
        return self.num_blocks * self.block_size


@dataclass
class SchedulerConfig:
    """Admission control and batching policy (reference config.py:90-108)."""

    policy: str = "fcfs"  # fcfs | sjf | lifo
    batching: str = "continuous"  # continuous | static
    max_batch_size: int = 8
    max_batched_tokens: int = 2048
    watermark: float = 0.01
    preemption_mode: str = "recompute"
    # Chunked prefill (an addition): a prefilling request processes at most
    # this many of its uncomputed tokens per step; None = the whole prompt
    # in one pass, as the reference does.
    prefill_chunk: int | None = None

    def __post_init__(self) -> None:
        if self.prefill_chunk is not None and self.prefill_chunk < 1:
            raise ValueError("prefill_chunk must be at least 1")
        if self.policy not in {"fcfs", "sjf", "lifo"}:
            raise ValueError(f"unknown scheduling policy {self.policy!r}")
        if self.batching not in {"continuous", "static"}:
            raise ValueError(f"unknown batching mode {self.batching!r}")
        if self.preemption_mode != "recompute":
            raise ValueError("only 'recompute' preemption is implemented")


@dataclass
class SamplingConfig:
    """Per-request sampling parameters (reference config.py:111-124)."""

    temperature: float = 1.0
    top_k: int | None = None
    top_p: float | None = None
    max_new_tokens: int = 32
    seed: int | None = None
    stop_token: int | None = None

    @property
    def greedy(self) -> bool:
        return self.temperature == 0.0


@dataclass
class SpeculativeConfig:
    """Draft-then-verify settings; ``gamma`` is the proposal length."""

    enabled: bool = False
    gamma: int = 4
    draft_checkpoint: str | None = None


@dataclass
class EngineConfig:
    """Top-level configuration (reference config.py:156-188)."""

    model: ModelConfig = field(default_factory=ModelConfig)
    cache: CacheConfig = field(default_factory=CacheConfig)
    scheduler: SchedulerConfig = field(default_factory=SchedulerConfig)
    speculative: SpeculativeConfig = field(default_factory=SpeculativeConfig)
    seed: int = 0
    device: str = "cuda"

    def to_dict(self) -> dict[str, Any]:
        return asdict(self)

    @classmethod
    def from_dict(cls, raw: dict[str, Any]) -> EngineConfig:
        known = {f.name for f in fields(cls)}
        table = {
            "model": ModelConfig,
            "cache": CacheConfig,
            "scheduler": SchedulerConfig,
            "speculative": SpeculativeConfig,
        }
        kwargs: dict[str, Any] = {}
        for key, value in raw.items():
            if key not in known:
                raise ValueError(f"unknown config key {key!r}")
            kwargs[key] = table[key](**value) if key in table else value
        return cls(**kwargs)

    def save(self, path: str | Path) -> None:
        Path(path).write_text(json.dumps(self.to_dict(), indent=2), encoding="utf-8")


def load_config(path: str | Path) -> EngineConfig:
    """Load an :class:`EngineConfig` from ``.json`` or ``.yaml``."""
    p = Path(path)
    text = p.read_text(encoding="utf-8")
    if p.suffix in {".yaml", ".yml"}:
        import yaml

        raw = yaml.safe_load(text)
    else:
        raw = json.loads(text)
    return EngineConfig.from_dict(raw or {})
