"""Ensembling on the GPU (`src/tabpackage/ensemble.py`).

`greedy_ensemble` keeps the reference's signature.  With a `PackScore` score function
the whole selection loop runs on the device (fused candidate scoring, selection and
ensemble update per iteration, one host synchronisation at the end).  An arbitrary
score callable -- e.g. the closure `tabpackage.train` builds around a metric -- runs
the reference's loop on the device tensors instead.
"""

from __future__ import annotations

import torch
from torch import Tensor

from tabpack_b200 import ops
from tabpack_b200.metrics import PackScore


def _validate(predictions: Tensor) -> None:
    if predictions.ndim < 2:
        raise ValueError("Predictions must have a dimension for ensemble members and at least one dimension for "
                         "each member's predictions")
    if predictions.numel() == 0:
        raise ValueError('Predictions must not be empty')


def compute_unsanitized_ensemble_predictions(member_predictions: Tensor, member_weights: Tensor | None) -> Tensor:
    """`compute_unsanitized_ensemble_predictions` (`ensemble.py:25-61`)."""
    _validate(member_predictions)
    K = member_predictions.shape[0]
    if member_weights is not None:
        if member_weights.ndim != 1:
            raise ValueError('`member_weights` must be a one-dimensional tensor')
        if len(member_weights) != K:
            raise ValueError('The number of member weights must match the number of ensemble members')
    flat = member_predictions.reshape(K, -1).to(torch.float32)
    idx = torch.arange(K, device=flat.device, dtype=torch.int32)
    out = ops.ensemble_mean(flat, idx, member_weights)
    return out.view(member_predictions.shape[1:]).to(member_predictions.dtype)


def topk_ensemble(predictions: Tensor, *, score_fn, k: int) -> Tensor:
    """`topk_ensemble` (`ensemble.py:64-92`)."""
    _validate(predictions)
    if k <= 0:
        raise ValueError('`k` must be positive to select at least one ensemble member')
    s = score_fn(predictions)
    if s.ndim != 1:
        raise ValueError('The scoring function must return a one-dimensional tensor of scores')
    if len(s) != len(predictions):
        raise ValueError('The scoring function must return one score per prediction')
    return torch.argmax(s)[None] if k == 1 else torch.argsort(s, descending=True, stable=True)[:k]


def _greedy_reference_loop(predictions, score_fn, init_top_k, max_ensemble_size, with_replacement):
    """The reference's loop (`ensemble.py:180-263`) for score callables that cannot be fused."""
    device = predictions.device
    ps = score_fn(predictions)
    init_idx = topk_ensemble(predictions, score_fn=lambda _: ps, k=init_top_k)
    n = len(predictions)
    rng = torch.arange(n, device=device)
    mask = torch.zeros(n, dtype=torch.bool, device=device)
    mask[init_idx] = True
    weights = None
    if with_replacement:
        weights = torch.zeros(n, dtype=predictions.dtype, device=device)
        weights[init_idx] = 1.0
    ens = predictions[init_idx].mean(0)
    ens_score = score_fn(ens[None])[0]
    size = len(init_idx)
    wsum = size
    limit = n if max_ensemble_size is None else max_ensemble_size if with_replacement else min(n, max_ensemble_size)
    while wsum < limit:
        cand_idx = rng if with_replacement else torch.nonzero_static(~mask, size=n - size)[:, 0]
        cand = predictions.clone() if with_replacement else predictions.index_select(0, cand_idx)
        cand.lerp_(ens[None], wsum / (wsum + 1))
        sc = score_fn(cand)
        best = sc.max()
        if best <= ens_score:
            break
        local_mask = sc == best
        local = torch.nonzero(local_mask)[:, 0]
        bidx = cand_idx[local_mask]
        if len(bidx) == 0:
            raise ValueError('Cannot select the best ensemble candidate because the scoring function returned a '
                             'NaN score')
        if len(bidx) == 1:
            li, bi = local[0], bidx[0]
        else:
            li = local[torch.argmax(ps[bidx])]
            bi = cand_idx[li]
        mask[bi] = True
        if weights is not None:
            weights[bi] += 1.0
        ens_score = sc[li]
        ens = cand[li].clone()
        del cand
        if weights is None or weights[bi].item() == 1.0:
            size += 1
        wsum += 1
    idx = torch.nonzero_static(mask, size=size)[:, 0]
    return idx, (None if weights is None else weights[idx])


def greedy_ensemble(predictions: Tensor, *, score_fn, init_top_k: int = 1, max_ensemble_size: int | None = None,
                    with_replacement: bool = False) -> tuple[Tensor, Tensor | None]:
    """`greedy_ensemble` (`ensemble.py:95-263`)."""
    _validate(predictions)
    if not torch.is_floating_point(predictions):
        raise TypeError('Predictions must be floating-point values')
    if init_top_k <= 0:
        raise ValueError('`init_top_k` must be positive to initialize the ensemble with at least one member')
    if with_replacement and max_ensemble_size is None:
        raise ValueError('Set `max_ensemble_size` to limit the number of ensemble members when '
                         '`with_replacement=True`')
    if max_ensemble_size is not None and init_top_k > max_ensemble_size:
        raise ValueError('`init_top_k` must not exceed `max_ensemble_size`')
    if not predictions.is_cuda:
        raise RuntimeError('tabpack_b200 ensembling runs on CUDA devices only')
    if not isinstance(score_fn, PackScore) or score_fn.metric == 'roc_auc':
        # no fused candidate scoring for ROC AUC: each iteration ranks its candidate blends
        # with the per-member sort kernel
        return _greedy_reference_loop(predictions, score_fn, init_top_k, max_ensemble_size, with_replacement)
    k = score_fn.classes(predictions)
    counts, status = ops.greedy_ensemble(
        predictions.reshape(len(predictions), -1), score_fn.y_true.reshape(-1), metric=score_fn.metric,
        maximize=score_fn.maximize, classes=k, init_top_k=init_top_k, max_ensemble_size=max_ensemble_size,
        with_replacement=with_replacement)
    st = status.cpu()  # the one synchronisation of the call
    if int(st[2]) != 0:
        raise ValueError('Cannot select the best ensemble candidate because the scoring function returned a NaN score')
    idx = torch.nonzero_static(counts > 0, size=int(st[1]))[:, 0]
    return idx, (counts[idx].to(predictions.dtype) if with_replacement else None)
