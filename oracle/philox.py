"""Philox4x32-10 and the dropout keep-mask derived from it (numpy restatement).

TEST INFRASTRUCTURE ONLY (see `oracle/__init__.py`).

The reference draws dropout masks with `Tensor.bernoulli_` from the global torch
RNG (`src/tabpackage/nn.py:897-901`), which is neither counter-based nor
reproducible across devices.  The B200 path replaces it with a counter-based
Philox4x32-10 stream (Salmon, Moraes, Dror, Shaw, "Parallel random numbers: as
easy as 1, 2, 3", SC'11), keyed so that a mask element depends only on
(seed, call offset, member id, row, column).  This module is the host
definition of that mask; the CUDA epilogue must agree with it bit for bit.

Key / counter layout (one Philox call covers 8 consecutive columns)::

    key     = (seed & 0xffffffff, seed >> 32)
    counter = (col >> 3, row, member, offset)
    r16     = 16-bit slice (col & 7) of the 128-bit output, little-endian
              within each 32-bit word: word[(col & 7) >> 1] >> (16 * (col & 1))
    p_keep  = float32(1 - p)
    keep    = r16 < floor(p_keep * 65536)
    scale   = float32(1 / p_keep)     (the value `mask.div_(p_keep)` produces)
"""

from __future__ import annotations

import numpy as np

PHILOX_M0 = np.uint64(0xD2511F53)
PHILOX_M1 = np.uint64(0xCD9E8D57)
PHILOX_W0 = np.uint32(0x9E3779B9)
PHILOX_W1 = np.uint32(0xBB67AE85)
_MASK32 = np.uint64(0xFFFFFFFF)


def philox4x32_10(c0, c1, c2, c3, k0, k1):
    """Vectorised Philox4x32 with 10 rounds.

    All arguments are broadcastable uint32 arrays (or scalars).  Returns a tuple
    of four uint32 arrays.
    """
    c0, c1, c2, c3 = (np.asarray(x, dtype=np.uint32) for x in (c0, c1, c2, c3))
    c0, c1, c2, c3 = np.broadcast_arrays(c0, c1, c2, c3)
    c0, c1, c2, c3 = (x.astype(np.uint32, copy=True) for x in (c0, c1, c2, c3))
    k0 = np.uint32(k0)
    k1 = np.uint32(k1)
    with np.errstate(over='ignore'):
        for rnd in range(10):
            p0 = PHILOX_M0 * c0.astype(np.uint64)
            p1 = PHILOX_M1 * c2.astype(np.uint64)
            hi0 = (p0 >> np.uint64(32)).astype(np.uint32)
            lo0 = (p0 & _MASK32).astype(np.uint32)
            hi1 = (p1 >> np.uint64(32)).astype(np.uint32)
            lo1 = (p1 & _MASK32).astype(np.uint32)
            c0, c1, c2, c3 = hi1 ^ c1 ^ k0, lo1, hi0 ^ c3 ^ k1, lo0
            if rnd != 9:
                k0 = np.uint32(k0 + PHILOX_W0)
                k1 = np.uint32(k1 + PHILOX_W1)
    return c0, c1, c2, c3


def keep_threshold(p: np.ndarray) -> np.ndarray:
    """uint32 threshold floor(float32(1 - p) * 2**16) per member."""
    p_keep = (np.float32(1.0) - np.asarray(p, dtype=np.float32)).astype(np.float32)
    return np.floor(p_keep.astype(np.float32) * np.float32(65536.0)).astype(np.uint32)


def keep_scale(p: np.ndarray) -> np.ndarray:
    """float32 1 / (1 - p), i.e. the kept value of `mask.div_(p_keep)`."""
    p_keep = (np.float32(1.0) - np.asarray(p, dtype=np.float32)).astype(np.float32)
    return (np.float32(1.0) / p_keep).astype(np.float32)


def dropout_keep_mask(
    *,
    seed: int,
    offset: int,
    members: np.ndarray,
    n_rows: int,
    n_cols: int,
    p: np.ndarray,
) -> np.ndarray:
    """Boolean keep mask of shape (len(members), n_rows, n_cols).

    `members` are the member ids that enter the counter (global ids when the
    pack is sharded); `p` holds one dropout probability per entry of `members`.
    """
    members = np.asarray(members, dtype=np.uint32)
    n_members = len(members)
    k0 = seed & 0xFFFFFFFF
    k1 = (seed >> 32) & 0xFFFFFFFF
    n_groups = (n_cols + 7) // 8
    g = np.arange(n_groups, dtype=np.uint32)[None, None, :]
    r = np.arange(n_rows, dtype=np.uint32)[None, :, None]
    m = members[:, None, None]
    w = philox4x32_10(g, r, m, np.uint32(offset & 0xFFFFFFFF), k0, k1)
    words = np.stack(w, axis=-1)  # (M, R, G, 4) uint32
    halves = np.stack([words & np.uint32(0xFFFF), words >> np.uint32(16)], axis=-1)
    r16 = halves.reshape(n_members, n_rows, n_groups * 8)[:, :, :n_cols]
    thr = keep_threshold(p)[:, None, None]
    return r16 < thr


def permutation_keys(*, seed: int, epoch: int, members: np.ndarray, n_rows: int) -> np.ndarray:
    """(len(members), n_rows) int32 batch-order keys: 31 bits of Philox4x32-10 word 0 with
    key = seed and counter = (row, member, epoch, 0x9E3779B9).  A member's stable argsort
    of its keys is its batch order in every epoch, whatever the sharding."""
    members = np.asarray(members, dtype=np.uint32)
    r = np.arange(n_rows, dtype=np.uint32)[None, :]
    w = philox4x32_10(r, members[:, None], np.uint32(epoch), np.uint32(0x9E3779B9),
                      seed & 0xFFFFFFFF, (seed >> 32) & 0xFFFFFFFF)[0]
    return (w >> np.uint32(1)).astype(np.int32)
