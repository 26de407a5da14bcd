"""Counter-based random numbers of the device samplers -- TEST INFRASTRUCTURE.

The reference draws with torch.Generator streams (ssd/engine/tree_drafter.py:
134-145, ssd/engine/verify.py:60-95), which no other implementation can
reproduce; the B200 kernels instead draw from Philox4x32-10 (Salmon, Moraes,
Dror, Shaw, "Parallel random numbers: as easy as 1, 2, 3", SC 2011) keyed by
the 64-bit seed, counter (round, row, index, stream), and turn a draw into a
Gumbel variate. This module restates those published steps in numpy so tests
can check the device's draws index for index, on top of the distributional
(chi-square) checks against the reference's sampling semantics.
"""

from __future__ import annotations

import numpy as np

_M32 = np.uint64(0xFFFFFFFF)
_MUL0, _MUL1 = np.uint64(0xD2511F53), np.uint64(0xCD9E8D57)
_W0, _W1 = np.uint64(0x9E3779B9), np.uint64(0xBB67AE85)


def philox4x32_10(counter, key):
    """Philox4x32-10 over arrays: counter = (c0, c1, c2, c3), key = (k0, k1),
    each broadcastable uint32 values. Returns the four output words."""
    c = [np.asarray(x, dtype=np.uint64) & _M32 for x in counter]
    k = [np.asarray(x, dtype=np.uint64) & _M32 for x in key]
    for _ in range(10):
        p0, p1 = _MUL0 * c[0], _MUL1 * c[2]
        c = [((p1 >> np.uint64(32)) ^ c[1] ^ k[0]) & _M32, p1 & _M32,
             ((p0 >> np.uint64(32)) ^ c[3] ^ k[1]) & _M32, p0 & _M32]
        k = [(k[0] + _W0) & _M32, (k[1] + _W1) & _M32]
    return c


def u01(x) -> np.ndarray:
    """Open-interval uniform from the top 23 bits of a word: (k + 1/2) / 2^23."""
    k = (np.asarray(x, dtype=np.uint64) >> np.uint64(9)).astype(np.float64)
    return ((k + 0.5) / 8388608.0).astype(np.float32)


def gumbel(seed: int, rnd: int, row: int, idx, stream: int) -> np.ndarray:
    """-log(-log(u)) for counter (rnd, row, idx, stream) under key `seed`."""
    idx = np.asarray(idx, dtype=np.uint64)
    zero = np.zeros_like(idx)
    w = philox4x32_10((zero + np.uint64(rnd), zero + np.uint64(row), idx, zero + np.uint64(stream)),
                      (np.uint64(seed & 0xFFFFFFFF), np.uint64((seed >> 32) & 0xFFFFFFFF)))
    u = u01(w[0]).astype(np.float64)
    return -np.log(-np.log(u))


def gumbel_topk(logprobs: np.ndarray, k: int, seed: int, rnd: int, row: int, stream: int) -> list:
    """Indices of the k largest log p(i) + Gumbel(i) over tokens with p > 0, in
    draw order (ties to the lower index): k draws without replacement."""
    lp = np.asarray(logprobs, dtype=np.float64)
    keys = lp + gumbel(seed, rnd, row, np.arange(lp.shape[0]), stream)
    keys[~np.isfinite(lp)] = -np.inf
    order = np.lexsort((np.arange(lp.shape[0]), -keys))
    return [int(i) for i in order[:k] if np.isfinite(keys[i])]
