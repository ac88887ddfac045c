"""Metric reductions and greedy ensemble selection on the GPU against the reference.

Metric values agree with the reference to 1e-5 relative; ensemble member indices and
selection counts are bit-exact (the fixture includes an exact duplicate prediction,
i.e. exact score ties broken by individual score and then by index).
"""

import numpy as np
import pytest
import torch

from oracle import ensemble as oe
from oracle import metrics as om

pytestmark = pytest.mark.gpu


@pytest.fixture(scope='module', autouse=True)
def _gpu():
    if not torch.cuda.is_available():
        pytest.skip('needs a GPU')


def _t(a):
    return torch.from_numpy(np.asarray(a)).cuda()


def test_metrics_match_reference(golden):
    from tabpack_b200 import metrics as M

    g = golden('metrics.npz')
    chk = lambda got, want, rtol=1e-5: np.testing.assert_allclose(got.cpu().numpy(), want, rtol=rtol, atol=1e-7)  # noqa: E731
    chk(M.mse_pack(y_true=_t(g['yr']), y_pred=_t(g['pr'])), g['mse'])
    chk(M.mae_pack(y_true=_t(g['yr']), y_pred=_t(g['pr'])), g['mae'])
    chk(M.r2_pack(y_true=_t(g['yr']), y_pred=_t(g['pr'])), g['r2'], 1e-4)
    chk(M.binary_cross_entropy_pack(y_true=_t(g['yb']), y_proba=_t(g['pb'])), g['bce'])
    chk(M.multiclass_cross_entropy_pack(y_true=_t(g['ym']), y_proba=_t(g['pm'])), g['ce'])
    chk(M.accuracy_pack(y_true=_t(g['ym']), y_pred=_t(g['lab'])), g['acc'], 1e-7)


REG_KWS = [dict(), dict(init_top_k=3), dict(max_ensemble_size=4),
           dict(with_replacement=True, max_ensemble_size=12),
           dict(with_replacement=True, max_ensemble_size=20, init_top_k=2)]


@pytest.mark.parametrize('j', range(len(REG_KWS)))
@pytest.mark.parametrize('fused', [True, False])
def test_greedy_regression_matches_reference(golden, j, fused):
    from tabpack_b200 import ensemble as E
    from tabpack_b200 import metrics as M

    g = golden('ensemble.npz')
    y, preds = _t(g['reg.y']), _t(g['reg.preds'])
    score = M.PackScore('mse', y, maximize=False) if fused else (lambda p: -M.mse_pack(y_true=y, y_pred=p))
    idx, w = E.greedy_ensemble(preds, score_fn=score, **REG_KWS[j])
    np.testing.assert_array_equal(idx.cpu().numpy(), g[f'reg.k{j}.idx'])
    if f'reg.k{j}.w' in g.files:
        np.testing.assert_array_equal(w.cpu().numpy(), g[f'reg.k{j}.w'])
    else:
        assert w is None


def test_greedy_classification_and_topk_match_reference(golden):
    from tabpack_b200 import ensemble as E
    from tabpack_b200 import metrics as M

    g = golden('ensemble.npz')
    yc, probs = _t(g['cls.y']), _t(g['cls.probs'])
    idx, _ = E.greedy_ensemble(probs, score_fn=M.PackScore('ce', yc, maximize=False), max_ensemble_size=6)
    np.testing.assert_array_equal(idx.cpu().numpy(), g['cls.idx'])
    y, preds = _t(g['reg.y']), _t(g['reg.preds'])
    top = E.topk_ensemble(preds, score_fn=M.PackScore('mse', y, maximize=False), k=3)
    np.testing.assert_array_equal(top.cpu().numpy(), g['reg.top3'])
    out = E.compute_unsanitized_ensemble_predictions(probs[:4], _t(g['mean.w']))
    np.testing.assert_allclose(out.cpu().numpy(), g['mean.out'], rtol=1e-6)
    out = E.compute_unsanitized_ensemble_predictions(probs[:4], None)
    np.testing.assert_allclose(out.cpu().numpy(), g['mean.out_eq'], rtol=1e-6)


@pytest.mark.parametrize('metric', ['mse', 'bce', 'accuracy_argmax'])
def test_greedy_large_matches_oracle(metric):
    from tabpack_b200 import ensemble as E
    from tabpack_b200 import metrics as M

    rng = np.random.default_rng(11)
    C, N = 96, 3000
    if metric == 'mse':
        y = rng.standard_normal(N).astype(np.float32)
        preds = (y[None] + rng.standard_normal((C, N)) * rng.uniform(0.2, 1.5, (C, 1))).astype(np.float32)
        score_np = lambda p: -om.mse_pack(y, p)  # noqa: E731
        kw = dict(max_ensemble_size=32)
    elif metric == 'bce':
        y = rng.integers(0, 2, N)
        logit = (2 * y - 1)[None] * rng.uniform(0.1, 2.0, (C, 1)) + rng.standard_normal((C, N))
        preds = (1 / (1 + np.exp(-logit))).astype(np.float32)
        score_np = lambda p: -om.binary_cross_entropy_pack(y, p)  # noqa: E731
        kw = dict(max_ensemble_size=32)
    else:
        K = 5
        y = rng.integers(0, K, N)
        logits = rng.standard_normal((C, N, K)) + 1.5 * np.eye(K)[y][None] * rng.uniform(0, 1, (C, 1, 1))
        preds = (np.exp(logits) / np.exp(logits).sum(-1, keepdims=True)).astype(np.float32)

        def score_np(p):
            return (np.argmax(p, -1) == y[None]).mean(-1)
        kw = dict(max_ensemble_size=16, with_replacement=True)
    want_idx, want_w = oe.greedy_ensemble(preds, score_np, **kw)
    score = M.PackScore(metric, _t(y), maximize=metric == 'accuracy_argmax')
    idx, w = E.greedy_ensemble(_t(preds), score_fn=score, **kw)
    np.testing.assert_array_equal(idx.cpu().numpy(), want_idx)
    if want_w is not None:
        np.testing.assert_array_equal(w.cpu().numpy(), want_w)


def test_roc_auc_matches_reference(golden):
    """Golden vectors of the reference's binary_roc_auc_pack (scores rounded to 0.1: ties)."""
    from tabpack_b200 import metrics as M

    g = golden('metrics.npz')
    got = M.binary_roc_auc_pack(y_true=_t(g['yb']), y_score=_t(g['sc']))
    assert got.dtype == torch.float32
    np.testing.assert_allclose(got.cpu().numpy(), g['auc'], rtol=1e-6)


@pytest.mark.parametrize('dtype', [np.float32, np.float64])
def test_roc_auc_large_with_ties_nans_and_signed_zeros(dtype):
    """Against the oracle at 50 003 rows: coarse scores (large tie groups), a constant member
    (AUC 0.5), NaN scores (ranked last, never tied), -0.0 next to +0.0 (tied)."""
    from tabpack_b200 import metrics as M

    rng = np.random.default_rng(11)
    N = 50003
    y = (rng.random(N) < 0.3).astype(np.int64)
    sc = np.stack([
        rng.standard_normal(N) + y,                      # distinct scores, informative
        np.round(rng.standard_normal(N) + 0.5 * y, 1),   # ~80 tie groups
        np.full(N, 0.25),                                # one group: AUC = 0.5
        np.where(rng.random(N) < 0.01, np.nan, rng.standard_normal(N) - y),
        np.where(rng.random(N) < 0.3 + 0.4 * y, 1.0, np.where(rng.random(N) < 0.5, -0.0, 0.0)),
    ]).astype(dtype)
    got = M.binary_roc_auc_pack(y_true=_t(y), y_score=_t(sc))
    want = om.binary_roc_auc_pack(y, sc)
    assert got.dtype == torch.from_numpy(sc).dtype
    np.testing.assert_allclose(got.cpu().numpy(), want, rtol=1e-6 if dtype == np.float32 else 1e-12)
    assert abs(float(got[2]) - 0.5) < 1e-12


def test_roc_auc_absent_class_is_nan_and_errors():
    from tabpack_b200 import metrics as M

    sc = torch.randn(3, 17, device='cuda')
    out = M.binary_roc_auc_pack(y_true=torch.zeros(17, dtype=torch.int64, device='cuda'), y_score=sc)
    assert torch.isnan(out).all()
    with pytest.raises(TypeError):
        M.binary_roc_auc_pack(y_true=torch.zeros(17, dtype=torch.int32, device='cuda'), y_score=sc)
    with pytest.raises(ValueError):
        M.binary_roc_auc_pack(y_true=torch.zeros(16, dtype=torch.int64, device='cuda'), y_score=sc)


def test_greedy_with_roc_auc_matches_oracle():
    """Greedy selection scored by ROC AUC (the reference's loop order, the AUC kernel as the
    score function) selects the same members as the oracle's greedy with the oracle's AUC."""
    from tabpack_b200.ensemble import greedy_ensemble
    from tabpack_b200.metrics import PackScore

    rng = np.random.default_rng(3)
    C, N = 12, 4000
    y = (rng.random(N) < 0.4).astype(np.int64)
    preds = (y[None] + rng.standard_normal((C, N)) * np.linspace(0.6, 2.0, C)[:, None]).astype(np.float32)
    idx, _ = greedy_ensemble(_t(preds), score_fn=PackScore('roc_auc', _t(y), maximize=True), init_top_k=2,
                             max_ensemble_size=6)
    want, _ = oe.greedy_ensemble(preds, lambda p: om.binary_roc_auc_pack(y, p).astype(np.float64), init_top_k=2,
                                 max_ensemble_size=6)
    assert sorted(idx.cpu().tolist()) == sorted(np.asarray(want).tolist())
