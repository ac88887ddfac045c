"""Pin the numpy oracle against golden vectors produced by the reference itself.

The fixtures come from `tests/golden/make_golden.py`, which runs the unmodified
reference (`tabpackage`) with the Philox keep mask injected into
`DropoutPack.forward`.
"""

import numpy as np
import pytest

from oracle import ensemble as oe
from oracle import layers as ol
from oracle import metrics as om
from oracle import optim as oo
from oracle.philox import dropout_keep_mask, philox4x32_10


def test_philox_known_answers():
    # Published Philox4x32-10 known-answer vectors (Random123 distribution).
    assert [int(x) for x in philox4x32_10(0, 0, 0, 0, 0, 0)] == [
        0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8]
    assert [int(x) for x in philox4x32_10(*([0xFFFFFFFF] * 6))] == [
        0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD]
    assert [int(x) for x in philox4x32_10(
        0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344, 0xA4093822, 0x299F31D0)] == [
        0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1]


def test_dropout_mask_statistics_and_edges():
    p = np.array([0.0, 0.1, 0.5, 0.9], np.float32)
    keep = dropout_keep_mask(seed=9, offset=3, members=np.arange(4), n_rows=256, n_cols=517, p=p)
    assert keep.shape == (4, 256, 517)
    assert keep[0].all()  # p = 0 keeps everything
    rates = keep.reshape(4, -1).mean(1)
    np.testing.assert_allclose(rates, 1 - p, atol=6e-3)
    # member ids, offsets and seeds give independent streams
    k2 = dropout_keep_mask(seed=9, offset=4, members=np.arange(4), n_rows=256, n_cols=517, p=p)
    assert (keep[2] != k2[2]).mean() > 0.3
    k3 = dropout_keep_mask(seed=9, offset=3, members=np.arange(4) + 1, n_rows=256, n_cols=517, p=p)
    assert np.array_equal(k3[0, :, :], dropout_keep_mask(
        seed=9, offset=3, members=np.array([1]), n_rows=256, n_cols=517, p=p[:1])[0])


@pytest.mark.parametrize('name,rtol', [('block_fp64.npz', 1e-12), ('block_fp32.npz', 2e-5)])
def test_block_forward_backward(golden, name, rtol):
    g = golden(name)
    dt = g['x'].dtype
    P, B, _ = g['x'].shape
    max_out = g['weight'].shape[1]
    mv = ol.dropout_mask_values(seed=int(g['seed']), offset=int(g['offset']), members=np.arange(P),
                                n_rows=B, n_cols=max_out, p=g['p'], dtype=dt)
    y, pre = ol.block_forward(g['x'], g['weight'], g['bias'], g['out_features'], mask_values=mv)
    scale = np.abs(g['y']).max()
    np.testing.assert_allclose(y, g['y'], rtol=rtol, atol=rtol * scale)
    dx, dW, db = ol.block_backward(g['x'], g['weight'], g['out_features'], pre, g['dy'], mask_values=mv)
    for got, want in ((dx, g['dx']), (dW, g['dweight']), (db, g['dbias'])):
        np.testing.assert_allclose(got, want, rtol=rtol, atol=rtol * np.abs(want).max())


@pytest.mark.parametrize('name', ['tabpack_fp64.npz', 'tabpack_indexed_fp64.npz'])
def test_tabpack_forward_backward(golden, name):
    g = golden(name)
    P = g['x_num'].shape[0]
    nb = int(g['n_blocks'].max())
    x_cat = ol.one_hot_encode(g['x_cat'], g['cards'], np.float64)
    x = np.concatenate([g['x_num'], x_cat], -1)
    blocks, masks = [], []
    for i in range(nb):
        pre = f'param.backbone.blocks.{i}.'
        w, b = g[pre + 'linear.weight'], g[pre + 'linear.bias']
        blocks.append((w, b, g[pre + 'linear.out_features']))
        masks.append(ol.dropout_mask_values(seed=int(g['seed']), offset=i, members=np.arange(P),
                                            n_rows=x.shape[1], n_cols=w.shape[1], p=g['dropout'],
                                            dtype=np.float64))
    h, cache = ol.mlp_forward_dense(x, blocks, g['n_blocks'], masks=masks)
    y = ol.linear_forward(h, g['param.output.weight'], g['param.output.bias'])
    np.testing.assert_allclose(y, g['y'], rtol=1e-12, atol=1e-12)
    dh, dWo, dbo = ol.linear_backward(h, g['param.output.weight'], None, g['dy'])
    np.testing.assert_allclose(dWo, g['grad.output.weight'], rtol=1e-11, atol=1e-11)
    np.testing.assert_allclose(dbo, g['grad.output.bias'], rtol=1e-11, atol=1e-11)
    _, grads = ol.mlp_backward_dense(blocks, cache, dh, g['n_blocks'])
    for i, (dW, db) in enumerate(grads):
        pre = f'grad.backbone.blocks.{i}.linear.'
        np.testing.assert_allclose(dW, g[pre + 'weight'], rtol=1e-10, atol=1e-10)
        np.testing.assert_allclose(db, g[pre + 'bias'], rtol=1e-10, atol=1e-10)


def _hp(g, case, key, per_member):
    v = g[f'c{case}.hp.{key}']
    return v.astype(np.float32) if per_member else float(v)


@pytest.mark.parametrize('case', [0, 1, 2, 3])
def test_adamw(golden, case):
    g = golden('adamw.npz')
    pm = bool(g[f'c{case}.per_member'])
    sr = bool(g[f'c{case}.support_replacement'])
    hp = {k: _hp(g, case, k, pm) for k in ('lr', 'beta1', 'beta2', 'eps', 'weight_decay')}
    w = g[f'c{case}.w0'].copy()
    b = g[f'c{case}.b0'].copy()
    sw, sb = {}, {}
    for s in range(3):
        oo.adamw_step(w, g[f'c{case}.s{s}.gw'], sw, support_replacement=sr, **hp)
        oo.adamw_step(b, g[f'c{case}.s{s}.gb'], sb, support_replacement=sr, **hp)
        np.testing.assert_allclose(w, g[f'c{case}.s{s}.w'], rtol=2e-6, atol=2e-7)
        np.testing.assert_allclose(b, g[f'c{case}.s{s}.b'], rtol=2e-6, atol=2e-7)
        np.testing.assert_allclose(sw['exp_avg'], g[f'c{case}.s{s}.m_w'], rtol=2e-6, atol=1e-9)
        np.testing.assert_allclose(sw['exp_avg_sq'], g[f'c{case}.s{s}.v_w'], rtol=2e-6, atol=1e-12)


def test_newton_schulz(golden):
    g = golden('newton_schulz.npz')
    for j in range(3):
        X = oo.newton_schulz5(g[f'G{j}'], 5)
        want = g[f'X{j}']
        # bf16 arithmetic: the CPU reference and the restatement may round a
        # handful of intermediate values differently
        err = np.abs(X - want).max() / np.abs(want).max()
        assert err < 2e-2, err


def test_newton_schulz_ragged_matches_padded():
    rng = np.random.default_rng(0)
    outs, ins = np.array([32, 16, 8, 40]), np.array([24, 40, 32, 40])
    G = np.zeros((4, 40, 40), np.float32)
    for i in range(4):
        G[i, :outs[i], :ins[i]] = rng.standard_normal((outs[i], ins[i])) * 0.02
    a = oo.newton_schulz5(G)
    b = oo.newton_schulz5_ragged(G, outs, ins)
    assert np.abs(a - b).max() / np.abs(a).max() < 2e-2


def test_muon(golden):
    g = golden('muon.npz')
    w = g['w0'].copy()
    st = {}
    scale = oo.muon_update_scale(g['out_features'], g['in_features'], 32, 32)
    np.testing.assert_allclose(scale, g['scale'], rtol=1e-7)
    lr = np.array([0.02, 0.01, 0.05], np.float32)
    mu = np.array([0.95, 0.9, 0.8], np.float32)
    wd = np.array([1e-2, 0.0, 1e-3], np.float32)
    for s in range(2):
        gr = g[f's{s}.g'].copy()
        oo.muon_step(w, gr, st, lr=lr, momentum=mu, weight_decay=wd, nesterov=True, update_scale=scale)
        np.testing.assert_allclose(st['muon_momentum_buffer'], g[f's{s}.mom'], rtol=1e-5, atol=1e-12)
        err = np.abs(w - g[f's{s}.w']).max() / np.abs(g[f's{s}.w']).max()
        assert err < 1e-3, err


def test_metrics(golden):
    g = golden('metrics.npz')
    np.testing.assert_allclose(om.mse_pack(g['yr'], g['pr']), g['mse'], rtol=1e-6)
    np.testing.assert_allclose(om.mae_pack(g['yr'], g['pr']), g['mae'], rtol=1e-6)
    np.testing.assert_allclose(om.r2_pack(g['yr'], g['pr']), g['r2'], rtol=1e-5)
    np.testing.assert_allclose(om.binary_cross_entropy_pack(g['yb'], g['pb']), g['bce'], rtol=1e-5)
    np.testing.assert_allclose(om.multiclass_cross_entropy_pack(g['ym'], g['pm']), g['ce'], rtol=1e-5)
    np.testing.assert_allclose(om.accuracy_pack(g['ym'], g['lab']), g['acc'], rtol=1e-7)
    np.testing.assert_allclose(om.binary_roc_auc_pack(g['yb'], g['sc']), g['auc'], rtol=1e-6)


def test_ensemble(golden):
    g = golden('ensemble.npz')
    y, preds = g['reg.y'], g['reg.preds']
    score = lambda p: -om.mse_pack(y, p)  # noqa: E731
    kws = [dict(), dict(init_top_k=3), dict(max_ensemble_size=4),
           dict(with_replacement=True, max_ensemble_size=12),
           dict(with_replacement=True, max_ensemble_size=20, init_top_k=2)]
    for j, kw in enumerate(kws):
        idx, w = oe.greedy_ensemble(preds, score, **kw)
        np.testing.assert_array_equal(idx, g[f'reg.k{j}.idx'])
        if w is not None:
            np.testing.assert_array_equal(w, g[f'reg.k{j}.w'])
    np.testing.assert_array_equal(oe.topk_ensemble(preds, score, 3), g['reg.top3'])
    yc, probs = g['cls.y'], g['cls.probs']
    idx, _ = oe.greedy_ensemble(probs, lambda p: -om.multiclass_cross_entropy_pack(yc, p), max_ensemble_size=6)
    np.testing.assert_array_equal(idx, g['cls.idx'])
    np.testing.assert_allclose(oe.ensemble_mean(probs[:4], g['mean.w']), g['mean.out'], rtol=1e-6)
    np.testing.assert_allclose(oe.ensemble_mean(probs[:4]), g['mean.out_eq'], rtol=1e-6)


@pytest.mark.parametrize('name, rtol', [('cosine_fp64.npz', 1e-12), ('cosine_fp32.npz', 2e-5)])
def test_cosine_embeddings(golden, name, rtol):
    g = golden(name)
    prm = [g['param.' + k] for k in ('weight', 'bias', 'elementwise_affine_weight', 'elementwise_affine_bias')]
    y, cache = ol.cosine_embeddings_forward(g['x'], *prm, g['d_embedding'])
    np.testing.assert_allclose(y, g['y'], rtol=rtol, atol=rtol * np.abs(g['y']).max())
    grads = ol.cosine_embeddings_backward(cache, g['dy'])
    for got, k in zip(grads, ('weight', 'bias', 'elementwise_affine_weight', 'elementwise_affine_bias')):
        want = g['grad.' + k]
        np.testing.assert_allclose(got, want, rtol=rtol * 10, atol=rtol * 10 * np.abs(want).max(), err_msg=k)


def test_tabpack_cosine_forward_backward(golden):
    """TabPack with per-member cosine embedding sizes and one-hot features: the first
    layer multiplies its full padded input width (`nn.py:792-816` ignores in_features)."""
    g = golden('tabpack_cosine_fp64.npz')
    P = g['x_num'].shape[0]
    pre = 'param.num_module.'
    prm = [g[pre + k] for k in ('weight', 'bias', 'elementwise_affine_weight', 'elementwise_affine_bias')]
    emb, cache = ol.cosine_embeddings_forward(g['x_num'], *prm, g[pre + 'd_embedding'])
    cards = [3, 2]
    x = np.concatenate([emb.reshape(*emb.shape[:2], -1), ol.one_hot_encode(g['x_cat'], cards, np.float64)], -1)
    nb = g['param.backbone.n_blocks']
    blocks, masks = [], []
    for i in range(int(nb.max())):
        p = f'param.backbone.blocks.{i}.'
        w = g[p + 'linear.weight']
        blocks.append((w, g[p + 'linear.bias'], g[p + 'linear.out_features']))
        masks.append(ol.dropout_mask_values(seed=int(g['seed']), offset=i, members=np.arange(P), n_rows=x.shape[1],
                                            n_cols=w.shape[1], p=g[f'param.backbone.blocks.{i}.dropout.p'],
                                            dtype=np.float64))
    h, bcache = ol.mlp_forward_dense(x, blocks, nb, masks=masks)
    y = ol.linear_forward(h, g['param.output.weight'], g['param.output.bias'])
    np.testing.assert_allclose(y, g['y'], rtol=1e-12, atol=1e-12)
    dh, _, _ = ol.linear_backward(h, g['param.output.weight'], None, g['dy'])
    dx, grads = ol.mlp_backward_dense(blocks, bcache, dh, nb)
    for i, (dW, db) in enumerate(grads):
        p = f'grad.backbone.blocks.{i}.linear.'
        np.testing.assert_allclose(dW, g[p + 'weight'], rtol=1e-10, atol=1e-10)
        np.testing.assert_allclose(db, g[p + 'bias'], rtol=1e-10, atol=1e-10)
    F, D = prm[2].shape[1:]
    demb = dx[..., :F * D].reshape(P, -1, F, D)
    for got, k in zip(ol.cosine_embeddings_backward(cache, demb),
                      ('weight', 'bias', 'elementwise_affine_weight', 'elementwise_affine_bias')):
        np.testing.assert_allclose(got, g['grad.num_module.' + k], rtol=1e-10, atol=1e-10, err_msg=k)
