"""Per-member metric reductions (numpy restatement of `src/tabpackage/metrics.py`).

TEST INFRASTRUCTURE ONLY (see `oracle/__init__.py`).

Predictions carry one pack dimension first; labels without a pack dimension are
shared by all members (`metrics.py:1-15`).  Means accumulate in float64 and are
cast to the prediction dtype at the end.
"""

from __future__ import annotations

import numpy as np


def _mean_nonpack(x):
    """`_mean_nonpack` (`metrics.py:49-60`)."""
    if x.ndim == 1:
        return x
    return x.reshape(x.shape[0], -1).astype(np.float64).mean(1)


def accuracy_pack(y_true, y_pred):
    """`accuracy_pack` (`metrics.py:76-84`)."""
    return _mean_nonpack((np.broadcast_to(y_true, y_pred.shape) == y_pred).astype(np.float32)).astype(np.float32)


def mse_pack(y_true, y_pred):
    """`mse_pack` (`metrics.py:190-200`)."""
    d = y_pred.astype(np.float64) - np.broadcast_to(y_true, y_pred.shape)
    return _mean_nonpack(d * d).astype(y_pred.dtype)


def mae_pack(y_true, y_pred):
    """`mae_pack` (`metrics.py:203-213`)."""
    d = y_pred.astype(np.float64) - np.broadcast_to(y_true, y_pred.shape)
    return _mean_nonpack(np.abs(d)).astype(y_pred.dtype)


def binary_cross_entropy_pack(y_true, y_proba):
    """`binary_cross_entropy_pack` (`metrics.py:153-167`): torch BCE clamps each
    log term at -100."""
    y = np.broadcast_to(y_true, y_proba.shape).astype(np.float64)
    p = y_proba.astype(np.float64)
    with np.errstate(divide='ignore'):
        lp = np.maximum(np.log(p), -100.0)
        l1p = np.maximum(np.log1p(-p), -100.0)
    return _mean_nonpack(-(y * lp + (1 - y) * l1p)).astype(y_proba.dtype)


def multiclass_cross_entropy_pack(y_true, y_proba):
    """`multiclass_cross_entropy_pack` (`metrics.py:170-187`)."""
    idx = np.broadcast_to(y_true, y_proba.shape[:-1])[..., None]
    pc = np.take_along_axis(y_proba, idx, axis=-1)[..., 0].astype(np.float64)
    with np.errstate(divide='ignore'):
        return _mean_nonpack(-np.maximum(np.log(pc), -100.0)).astype(y_proba.dtype)


def r2_pack(y_true, y_pred, force_finite=True):
    """`r2_pack` (`metrics.py:216-253`) for labels shared by all members."""
    yp = y_pred.astype(np.float64)
    yt = np.broadcast_to(y_true, y_pred.shape[1:]).astype(np.float64)
    num = ((yp - yt[None]) ** 2).reshape(yp.shape[0], -1).sum(1)
    den = ((yt - np.asarray(y_true, np.float64).mean()) ** 2).sum()
    with np.errstate(divide='ignore', invalid='ignore'):
        ratio = num / den
    if force_finite:
        ratio = np.where(num == 0.0, 0.0, np.where(den == 0.0, 1.0, ratio))
    n_obj = y_pred.size // y_pred.shape[0]
    out = np.full_like(ratio, np.nan) if n_obj < 2 else 1.0 - ratio
    return out.astype(y_pred.dtype)


def _midranks(x_sorted):
    """`_midranks_pack` (`metrics.py:87-114`) for one sorted row."""
    n = len(x_sorted)
    ranks = np.empty(n, np.float64)
    i = 0
    while i < n:
        j = i
        while j + 1 < n and x_sorted[j + 1] == x_sorted[i]:
            j += 1
        ranks[i : j + 1] = (i + j) / 2 + 1
        i = j + 1
    return ranks


def binary_roc_auc_pack(y_true, y_score):
    """`binary_roc_auc_pack` (`metrics.py:117-150`): Mann-Whitney U with midranks."""
    y_true = np.asarray(y_true, np.int64)
    npos = int(y_true.sum())
    nneg = len(y_true) - npos
    out = np.empty(y_score.shape[0], np.float64)
    for m in range(y_score.shape[0]):
        order = np.argsort(y_score[m], kind='stable')
        r = _midranks(y_score[m][order])
        u = (r * y_true[order]).sum() - npos * (npos + 1) / 2
        out[m] = np.nan if npos * nneg == 0 else u / (npos * nneg)
    return out.astype(y_score.dtype)
