"""ctypes binding of libmicroserve_b200.so (the C ABI in include/microserve_b200.h).

The library is built in-tree (``python -m microserve_b200.csrc.build`` or
``__graft_entry__.build()``).  There is no fallback: every compute path of the
package goes through this library on a CUDA device, and a missing library or
device raises immediately.
"""

from __future__ import annotations

import ctypes
from ctypes import POINTER, c_float, c_int, c_int32, c_int64, c_size_t, c_uint64, c_void_p
from pathlib import Path

import numpy as np
import torch

LIB_PATH = Path(__file__).resolve().with_name("libmicroserve_b200.so")

MS_OK = 0
MS_ERR_INVALID = 1
MS_ERR_CUDA = 2
MS_ERR_UNSUPPORTED = 3
MS_ERR_TOO_LARGE = 4

DTYPE_F32 = 0
DTYPE_BF16 = 1

LANE_SAMPLE = 0
LANE_DRAFT = 0
LANE_ACCEPT = 64
LANE_RESAMPLE = 128

TORCH_DTYPES = {DTYPE_F32: torch.float32, DTYPE_BF16: torch.bfloat16}
DTYPE_CODES = {"float32": DTYPE_F32, "bfloat16": DTYPE_BF16}


class MicroserveError(RuntimeError):
    """A non-zero status from the CUDA library."""

    def __init__(self, func: str, code: int, message: str) -> None:
        super().__init__(f"{func} failed (status {code}): {message}")
        self.code = code


# numpy mirrors of the C structs that live in device arrays
SAMPLING_PARAMS_DTYPE = np.dtype(
    [("temperature", "<f4"), ("top_p", "<f4"), ("top_k", "<i4"), ("pad_", "<i4"),
     ("seed", "<u8"), ("step", "<u8")],
    align=True,
)
assert SAMPLING_PARAMS_DTYPE.itemsize == 32
ROW_STATS_DTYPE = np.dtype([("max", "<f4"), ("thresh", "<f4"), ("z", "<f4"), ("argmax", "<i4")])
assert ROW_STATS_DTYPE.itemsize == 16


class MsKVCache(ctypes.Structure):
    _fields_ = [
        ("n_layers", c_int32),
        ("num_blocks", c_int32),
        ("block_size", c_int32),
        ("n_kv_heads", c_int32),
        ("d_head", c_int32),
        ("dtype", c_int32),
        ("k_pool", POINTER(c_void_p)),
        ("v_pool", POINTER(c_void_p)),
    ]


class MsModel(ctypes.Structure):
    _fields_ = [
        ("vocab_size", c_int32),
        ("d_model", c_int32),
        ("n_layers", c_int32),
        ("n_heads", c_int32),
        ("n_kv_heads", c_int32),
        ("d_head", c_int32),
        ("d_ff", c_int32),
        ("max_seq_len", c_int32),
        ("dtype", c_int32),
        ("norm_eps", c_float),
        ("embed", c_void_p),
        ("final_norm", c_void_p),
        ("rope_cos", c_void_p),
        ("rope_sin", c_void_p),
        ("attn_norm", POINTER(c_void_p)),
        ("w_qkv", POINTER(c_void_p)),
        ("w_o", POINTER(c_void_p)),
        ("ffn_norm", POINTER(c_void_p)),
        ("w_gate_up", POINTER(c_void_p)),
        ("w_down", POINTER(c_void_p)),
    ]


class MsBatch(ctypes.Structure):
    _fields_ = [
        ("n_tokens", c_int32),
        ("n_seqs", c_int32),
        ("max_blocks", c_int32),
        ("max_q_len", c_int32),
        ("max_context", c_int32),
        ("reserved_", c_int32),
        ("input_ids", c_void_p),
        ("positions", c_void_p),
        ("slot_mapping", c_void_p),
        ("q_start", c_void_p),
        ("context_lens", c_void_p),
        ("block_tables", c_void_p),
    ]


# name -> (restype, argtypes)
_SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "ms_version": (c_int, []),
    "ms_last_error": (ctypes.c_char_p, []),
    "ms_launch_count": (c_uint64, []),
    "ms_device_error": (c_int, [c_void_p, POINTER(c_int32)]),
    "ms_profile_start": (c_int, [c_int]),
    "ms_profile_stop": (c_int, [POINTER(ctypes.c_double), POINTER(c_int64)]),
    "ms_philox_uniforms": (c_int, [c_void_p, c_void_p, c_int, c_int, c_void_p, c_void_p]),
    "ms_sample": (
        c_int,
        [c_void_p, c_int64, c_int, c_int, c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_void_p,
         c_void_p, c_void_p, c_void_p],
    ),
    "ms_spec_accept": (
        c_int,
        [c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_int, c_void_p, c_void_p, c_int, c_int,
         c_int, c_void_p, c_void_p, c_void_p],
    ),
    "ms_spec_chain_size": (c_int64, [c_int, c_int]),
    "ms_spec_chain_plan": (
        c_int,
        [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_void_p, c_int,
         c_int, c_void_p, c_void_p, c_void_p],
    ),
    "ms_verify_probs": (
        c_int,
        [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_void_p, c_void_p,
         c_void_p],
    ),
    "ms_host_blocks_needed": (c_int64, [c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_int,
                                        c_void_p]),
    "ms_host_append": (c_int, [c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_int64,
                               c_int, c_void_p, c_int64, c_void_p]),
    "ms_host_truncate": (c_int64, [c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_void_p,
                                   c_int64, c_int, c_void_p, c_int64]),
    "ms_kv_write": (c_int, [POINTER(MsKVCache), c_int, c_void_p, c_int, c_void_p, c_void_p, c_void_p]),
    "ms_kv_gather": (
        c_int,
        [POINTER(MsKVCache), c_int, c_void_p, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p],
    ),
    "ms_forward_workspace_size": (c_size_t, [POINTER(MsModel), c_int, c_int]),
    "ms_forward": (
        c_int,
        [POINTER(MsModel), POINTER(MsKVCache), POINTER(MsBatch), c_void_p, c_int, c_void_p,
         c_int64, c_void_p, c_size_t, c_void_p],
    ),
    "ms_forward_static_scratch": (
        c_int,
        [POINTER(MsModel), POINTER(MsKVCache), POINTER(MsBatch), c_void_p, c_int, c_void_p,
         c_int64, c_void_p],
    ),
    "ms_rmsnorm": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_float, c_int,
                           c_void_p]),
    "ms_gemm": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int64, c_int,
                        c_int, c_int, c_void_p]),
    "ms_gemm_set_policy": (c_int, [c_int]),
    "ms_attention_scratch_size": (c_size_t, [POINTER(MsKVCache), c_int, POINTER(MsBatch)]),
    "ms_paged_attention": (c_int, [c_void_p, POINTER(MsKVCache), c_int, POINTER(MsBatch), c_int,
                                   c_void_p, c_void_p]),
}

_lib: ctypes.CDLL | None = None


def load() -> ctypes.CDLL:
    """Load the library once and bind every declared entry point."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise RuntimeError(
            f"microserve_b200 CUDA library not found at {LIB_PATH}; build it with "
            "`python -m microserve_b200.csrc.build` (there is no CPU fallback)"
        )
    lib = ctypes.CDLL(str(LIB_PATH))
    for name, (restype, argtypes) in _SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = restype
        fn.argtypes = argtypes
    _lib = lib
    return lib


def exported_names() -> list[str]:
    return list(_SIGNATURES)


def check(name: str, rc: int) -> None:
    if rc != MS_OK:
        msg = load().ms_last_error()
        raise MicroserveError(name, rc, msg.decode() if msg else "")


def call(name: str, *args: object) -> None:
    """Call an int-status entry point and raise on failure."""
    check(name, getattr(load(), name)(*args))


def require_cuda(device: torch.device | str) -> torch.device:
    dev = torch.device(device)
    if dev.type != "cuda":
        raise RuntimeError(
            f"microserve_b200 computes on CUDA devices only (got {dev}); there is no CPU path"
        )
    if not torch.cuda.is_available():
        raise RuntimeError("microserve_b200 needs a CUDA device and none is available")
    load()
    return dev


def stream_ptr(device: torch.device | None = None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def launch_count() -> int:
    return int(load().ms_launch_count())


def device_error(device: torch.device | None = None) -> int:
    code = c_int32(0)
    call("ms_device_error", stream_ptr(device), ctypes.byref(code))
    return int(code.value)


def pointer_array(tensors: list[torch.Tensor]) -> ctypes.Array:
    arr = (c_void_p * len(tensors))()
    for i, t in enumerate(tensors):
        arr[i] = t.data_ptr()
    return arr
