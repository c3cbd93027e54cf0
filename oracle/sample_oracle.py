"""ORACLE -- test infrastructure, not product code (see oracle/__init__.py).

Temperature sampling of the decode head, restated on the CPU:

* Philox4x32-10, the counter-based generator of Salmon, Moraes, Dror and
  Shaw, "Parallel random numbers: as easy as 1, 2, 3" (SC 2011): ten rounds
  of (R0, R1, R2, R3) -> (hi(M1 R2) ^ R1 ^ k0, lo(M1 R2), hi(M0 R0) ^ R3 ^
  k1, lo(M0 R0)) with M0 = 0xD2511F53, M1 = 0xCD9E8D57 and the key bumped by
  0x9E3779B9 / 0xBB67AE85 between rounds.  Pinned by the generator's
  published known-answer vectors (tests/test_sample_oracle.py).
* The reference's sampler, generate.py:46-63 without top_k: probs =
  softmax(logits / T), token = argmax(probs / q), q ~ Exp(1).  With q =
  -log(u) this is argmax(logits / T - log(-log(u))), the Gumbel-max form the
  kernel computes, with u from the first Philox word of counter (row, pos
  low, pos high, 0x5EED5A3B) under key (seed low, seed high).
"""
from __future__ import annotations

import numpy as np

_M0, _M1, _W0, _W1 = 0xD2511F53, 0xCD9E8D57, 0x9E3779B9, 0xBB67AE85
_MASK = 0xFFFFFFFF


def philox4x32_10(ctr, key):
    """Four 32-bit words of Philox4x32-10 for counter ``ctr`` (4 ints) and key (2 ints)."""
    c0, c1, c2, c3 = (int(v) & _MASK for v in ctr)
    k0, k1 = (int(v) & _MASK for v in key)
    for r in range(10):
        if r:
            k0, k1 = (k0 + _W0) & _MASK, (k1 + _W1) & _MASK
        p0, p1 = _M0 * c0, _M1 * c2
        c0, c1, c2, c3 = ((p1 >> 32) ^ c1 ^ k0) & _MASK, p1 & _MASK, ((p0 >> 32) ^ c3 ^ k1) & _MASK, p0 & _MASK
    return c0, c1, c2, c3


def _philox_first_word(rows: np.ndarray, pos: int, seed: int) -> np.ndarray:
    """First Philox word for every row (vectorised over rows, uint64 arithmetic)."""
    m = np.uint64(_MASK)
    c0 = rows.astype(np.uint64) & m
    c1 = np.full_like(c0, pos & _MASK)
    c2 = np.full_like(c0, (pos >> 32) & _MASK)
    c3 = np.full_like(c0, 0x5EED5A3B)
    k0, k1 = seed & _MASK, (seed >> 32) & _MASK
    for r in range(10):
        if r:
            k0, k1 = (k0 + _W0) & _MASK, (k1 + _W1) & _MASK
        p0 = np.uint64(_M0) * c0
        p1 = np.uint64(_M1) * c2
        c0, c1, c2, c3 = (((p1 >> np.uint64(32)) ^ c1 ^ np.uint64(k0)) & m, p1 & m,
                          ((p0 >> np.uint64(32)) ^ c3 ^ np.uint64(k1)) & m, p0 & m)
    return c0


def gumbel_noise(rows, pos: int, seed: int) -> np.ndarray:
    """Gumbel(0, 1) noise per global vocabulary row (float32), as the kernel draws it."""
    w = _philox_first_word(np.asarray(rows), int(pos), int(seed))
    u = ((w >> np.uint64(8)).astype(np.float32) + np.float32(0.5)) * np.float32(1.0 / 16777216.0)
    return (-np.log(-np.log(u.astype(np.float64)))).astype(np.float32)


def sample_keys(logits_f16: np.ndarray, temperature: float, pos: int, seed: int, row_offset: int = 0) -> np.ndarray:
    """Sampling keys logit / T + noise (float32) of fp16 logits."""
    lg = np.asarray(logits_f16, dtype=np.float32)
    rows = np.arange(lg.shape[0], dtype=np.int64) + row_offset
    return lg * np.float32(1.0 / temperature) + gumbel_noise(rows, pos, seed)


def sample_token(logits_f16: np.ndarray, temperature: float, pos: int, seed: int) -> int:
    """The sampled token (lowest index among equal keys)."""
    return int(np.argmax(sample_keys(logits_f16, temperature, pos, seed)))
