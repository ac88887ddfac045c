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
