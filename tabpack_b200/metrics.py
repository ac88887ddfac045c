"""Per-member metrics on the GPU (`src/tabpackage/metrics.py`).

Same functions and signatures as the reference's `*_pack` metrics: the pack dimension
comes first and labels without a pack dimension are shared by every member.  Each call
is one kernel launch with one block per member (fp32 terms, fp64 sums).  `PackScore`
wraps a metric as a score function that `tabpack_b200.ensemble.greedy_ensemble`
recognises and runs fully fused on the device.
"""

from __future__ import annotations

import torch
from torch import Tensor

from tabpack_b200 import ops


def _is_integer(t: Tensor) -> bool:
    return not torch.is_floating_point(t) and not torch.is_complex(t) and t.dtype != torch.bool


def _check_shapes(y_true: Tensor, y_pred: Tensor, n_trailing: int) -> None:
    """`_check_y_shapes` (`metrics.py:26-46`) for labels shared by all members."""
    if y_pred.ndim < 1 + n_trailing:
        raise ValueError('The prediction tensor has too few dimensions to represent a pack of outputs')
    if y_true.ndim > y_pred.ndim - n_trailing:
        raise ValueError('Labels have too many dimensions for the provided predictions')
    end = y_pred.ndim - n_trailing
    if y_true.ndim > 0 and y_true.shape != y_pred.shape[end - y_true.ndim: end]:
        raise ValueError('The label and prediction shapes are incompatible; only missing leading label dimensions '
                         'may be broadcast')
    if y_pred.numel() == 0:
        raise ValueError('Predictions must not be empty')
    if y_true.ndim == y_pred.ndim - n_trailing:
        raise NotImplementedError('per-member labels: pass labels shared by all members')


def _flat(y_true: Tensor, y_pred: Tensor, n_trailing: int = 0):
    P = y_pred.shape[0]
    rows = y_pred.numel() // P
    if n_trailing:
        rows //= y_pred.shape[-1]
    yt = y_true.expand(y_pred.shape[1: y_pred.ndim - n_trailing]).reshape(-1)
    return P, rows, yt


def accuracy_pack(*, y_true: Tensor, y_pred: Tensor) -> Tensor:
    """`accuracy_pack` (`metrics.py:76-84`)."""
    if not _is_integer(y_true):
        raise TypeError('Labels must have an integer data type')
    if y_true.dtype != y_pred.dtype:
        raise TypeError('Labels and predictions must have the same data type')
    _check_shapes(y_true, y_pred, 0)
    P, rows, yt = _flat(y_true, y_pred)
    return ops.metric_pack('accuracy', y_pred.reshape(P, rows), yt)


def _float_metric(name: str, y_true: Tensor, y_pred: Tensor) -> Tensor:
    if not torch.is_floating_point(y_true):
        raise TypeError('Labels must be floating-point values')
    if y_true.dtype != y_pred.dtype:
        raise TypeError('Labels and predictions must have the same data type')
    _check_shapes(y_true, y_pred, 0)
    P, rows, yt = _flat(y_true, y_pred)
    return ops.metric_pack(name, y_pred.reshape(P, rows), yt).to(y_pred.dtype)


def mse_pack(*, y_true: Tensor, y_pred: Tensor) -> Tensor:
    """`mse_pack` (`metrics.py:190-200`)."""
    return _float_metric('mse', y_true, y_pred)


def mae_pack(*, y_true: Tensor, y_pred: Tensor) -> Tensor:
    """`mae_pack` (`metrics.py:203-213`)."""
    return _float_metric('mae', y_true, y_pred)


def r2_pack(*, y_true: Tensor, y_pred: Tensor, force_finite: bool = True) -> Tensor:
    """`r2_pack` (`metrics.py:216-253`) for labels shared by all members (force_finite)."""
    if not force_finite:
        raise NotImplementedError('r2_pack runs with force_finite=True')
    return _float_metric('r2', y_true, y_pred)


def binary_cross_entropy_pack(*, y_true: Tensor, y_proba: Tensor) -> Tensor:
    """`binary_cross_entropy_pack` (`metrics.py:153-167`)."""
    if not _is_integer(y_true):
        raise TypeError('Labels must have an integer data type')
    if not torch.is_floating_point(y_proba):
        raise TypeError('Probabilities must be floating-point values')
    _check_shapes(y_true, y_proba, 0)
    P, rows, yt = _flat(y_true, y_proba)
    return ops.metric_pack('bce', y_proba.reshape(P, rows), yt).to(y_proba.dtype)


def multiclass_cross_entropy_pack(*, y_true: Tensor, y_proba: Tensor) -> Tensor:
    """`multiclass_cross_entropy_pack` (`metrics.py:170-187`)."""
    if y_true.dtype != torch.int64:
        raise TypeError('Labels must have the int64 data type')
    if not torch.is_floating_point(y_proba):
        raise TypeError('Probabilities must be floating-point values')
    _check_shapes(y_true, y_proba, 1)
    P, rows, yt = _flat(y_true, y_proba, 1)
    return ops.metric_pack('ce', y_proba.reshape(P, rows, y_proba.shape[-1]), yt, y_proba.shape[-1]).to(y_proba.dtype)


def binary_roc_auc_pack(*, y_true: Tensor, y_score: Tensor) -> Tensor:
    """`binary_roc_auc_pack` (`metrics.py:117-150`): per-member ROC AUC as the Mann-Whitney U
    statistic with midranks, one sort per member on the device (`tp_binary_roc_auc`).
    Labels are {0, 1}; a nonzero label counts as positive."""
    if y_true.dtype != torch.int64:
        raise TypeError('Labels must have the data type `torch.int64`')
    if y_score.dtype not in (torch.float32, torch.float64):
        raise TypeError('Scores must have the data type `torch.float32` or `torch.float64`')
    if y_true.ndim != 1:
        raise ValueError('The label tensor must have one dimension')
    if y_score.ndim != 2:
        raise ValueError('The score tensor must have two dimensions')
    if y_true.shape[-1] != y_score.shape[-1]:
        raise ValueError('Labels and scores must have the same batch size')
    if y_score.numel() == 0:
        raise ValueError('Scores must not be empty')
    return ops.binary_roc_auc(y_score, y_true)


_PACK_FNS = {'mse': mse_pack, 'mae': mae_pack, 'bce': binary_cross_entropy_pack, 'ce': multiclass_cross_entropy_pack}


class PackScore:
    """A higher-is-better score function over stacked predictions, as `greedy_ensemble`
    and `topk_ensemble` take it (`ensemble.py:9-12`), backed by a fused metric.

    metric: 'mse', 'mae', 'bce', 'ce', 'accuracy_argmax' or 'roc_auc' (binary scores, scored
    by `binary_roc_auc_pack`; greedy selection then scores each iteration's candidate blends
    with it instead of the fused scoring kernel); `y_true` shared labels; `maximize`: whether
    larger metric values are better (the score is -metric otherwise).
    """

    def __init__(self, metric: str, y_true: Tensor, *, maximize: bool) -> None:
        if metric not in ('mse', 'mae', 'bce', 'ce', 'accuracy_argmax', 'roc_auc'):
            raise ValueError(f'unsupported fused metric {metric!r}')
        self.metric = metric
        self.y_true = y_true
        self.maximize = maximize

    def classes(self, predictions: Tensor) -> int:
        return predictions.shape[-1] if self.metric in ('ce', 'accuracy_argmax') else 1

    def __call__(self, predictions: Tensor) -> Tensor:
        C = predictions.shape[0]
        if self.metric == 'roc_auc':
            v = ops.binary_roc_auc(predictions.reshape(C, -1).float(), self.y_true.reshape(-1).to(torch.int64))
            return v if self.maximize else -v
        k = self.classes(predictions)
        flat = predictions.reshape(C, -1, k) if k > 1 else predictions.reshape(C, -1)
        v = ops.metric_pack(self.metric, flat, self.y_true.reshape(-1), k)
        return v if self.maximize else -v
