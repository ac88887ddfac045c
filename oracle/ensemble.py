"""Ensemble selection (numpy restatement of `src/tabpackage/ensemble.py`).

TEST INFRASTRUCTURE ONLY (see `oracle/__init__.py`).

`score_fn` maps a stacked prediction array `(C, *)` to higher-is-better scores
`(C,)`, as in the reference.
"""

from __future__ import annotations

import numpy as np

from oracle.optim import lerp


def ensemble_mean(member_predictions, member_weights=None):
    """`compute_unsanitized_ensemble_predictions` (`ensemble.py:25-61`)."""
    if member_weights is None:
        return member_predictions.astype(np.float64).mean(0).astype(member_predictions.dtype)
    w = np.asarray(member_weights, np.float64)
    w = w / w.sum()
    flat = member_predictions.reshape(len(member_predictions), -1).astype(np.float64)
    return (w @ flat).reshape(member_predictions.shape[1:]).astype(member_predictions.dtype)


def topk_ensemble(predictions, score_fn, k):
    """`topk_ensemble` (`ensemble.py:64-92`): stable descending sort of scores."""
    s = score_fn(predictions)
    if k == 1:
        return np.array([int(np.argmax(s))])
    order = sorted(range(len(s)), key=lambda i: (-s[i], i))
    return np.array(order[:k])


def greedy_ensemble(predictions, score_fn, init_top_k=1, max_ensemble_size=None,
                    with_replacement=False):
    """`greedy_ensemble` (`ensemble.py:95-263`).

    Returns `(idx, weights)` like the reference (weights None without
    replacement).  The candidate update is the reference's
    `candidate.lerp_(ensemble, w/(w+1))` in float32.
    """
    predictions = np.asarray(predictions, np.float32)
    C = len(predictions)
    ind_scores = score_fn(predictions)
    init_idx = topk_ensemble(predictions, lambda _: ind_scores, init_top_k)
    mask = np.zeros(C, bool)
    mask[init_idx] = True
    weights = None
    if with_replacement:
        weights = np.zeros(C, np.float32)
        weights[init_idx] = 1.0
    ens = predictions[init_idx].astype(np.float64).mean(0).astype(np.float32)
    ens_score = score_fn(ens[None])[0]
    size = len(init_idx)
    wsum = size
    limit = (C if max_ensemble_size is None
             else max_ensemble_size if with_replacement
             else min(C, max_ensemble_size))
    while wsum < limit:
        cand_idx = np.arange(C) if with_replacement else np.nonzero(~mask)[0]
        cand = lerp(predictions[cand_idx], ens[None], np.float32(wsum / (wsum + 1)))
        scores = score_fn(cand)
        best = scores.max()
        if not best > ens_score:
            break
        local = np.nonzero(scores == best)[0]
        if len(local) == 0:
            raise ValueError('NaN score')
        if len(local) == 1:
            li = local[0]
        else:
            li = local[int(np.argmax(ind_scores[cand_idx[local]]))]
        bi = cand_idx[li]
        mask[bi] = True
        if weights is not None:
            weights[bi] += 1.0
        ens_score = scores[li]
        ens = cand[li].copy()
        if weights is None or weights[bi] == 1.0:
            size += 1
        wsum += 1
    idx = np.nonzero(mask)[0]
    return idx, (None if weights is None else weights[idx])
