"""Philox4x32-10 in numpy -- test infrastructure (checker only).

Published algorithm: J. K. Salmon, M. A. Moraes, R. O. Dror, D. E. Shaw,
"Parallel random numbers: as easy as 1, 2, 3", SC'11.  Ten rounds of
    (hi0, lo0) = mulhilo(0xD2511F53, c0); (hi1, lo1) = mulhilo(0xCD9E8D57, c2)
    c = (hi1 ^ c1 ^ k0, lo1, hi0 ^ c3 ^ k1, lo0)
with the key bumped by (0x9E3779B9, 0xBB67AE85) between rounds.

The device kernels (microserve_b200/csrc/common.cuh) use the same stream:
counter (lane, 0, step_lo, step_hi), key (seed_lo, seed_hi), uniform = top 24
bits of output word 0 times 2^-24 (exact in float32, in [0, 1)).
"""

from __future__ import annotations

import numpy as np

_MASK = np.uint64(0xFFFFFFFF)
_M0 = np.uint64(0xD2511F53)
_M1 = np.uint64(0xCD9E8D57)
_W0 = np.uint64(0x9E3779B9)
_W1 = np.uint64(0xBB67AE85)


def philox4x32_10(
    ctr: tuple[object, object, object, object], key: tuple[object, object]
) -> tuple[np.ndarray, np.ndarray, np.ndarray, np.ndarray]:
    """Vectorised Philox4x32-10; every argument broadcasts, values are uint32."""
    c0, c1, c2, c3 = (np.asarray(v, dtype=np.uint64) & _MASK for v in ctr)
    k0, k1 = (np.asarray(v, dtype=np.uint64) & _MASK for v in key)
    for r in range(10):
        if r:
            k0 = (k0 + _W0) & _MASK
            k1 = (k1 + _W1) & _MASK
        p0 = _M0 * c0
        p1 = _M1 * c2
        hi0, lo0 = p0 >> np.uint64(32), p0 & _MASK
        hi1, lo1 = p1 >> np.uint64(32), p1 & _MASK
        c0, c1, c2, c3 = hi1 ^ c1 ^ k0, lo1, hi0 ^ c3 ^ k1, lo0
    return tuple(np.asarray(v, dtype=np.uint32) for v in (c0, c1, c2, c3))  # type: ignore[return-value]


def uniform(seed: object, step: object, lane: object) -> np.ndarray:
    """float32 uniforms in [0, 1) for (seed, step, lane), broadcasting."""
    seed = np.asarray(seed, dtype=np.uint64)
    step = np.asarray(step, dtype=np.uint64)
    lane = np.asarray(lane, dtype=np.uint64)
    r0, _, _, _ = philox4x32_10(
        (lane, np.uint64(0), step & _MASK, step >> np.uint64(32)),
        (seed & _MASK, seed >> np.uint64(32)),
    )
    return ((r0 >> np.uint32(8)).astype(np.float32) * np.float32(1.0 / 16777216.0)).astype(np.float32)
