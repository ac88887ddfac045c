"""Cosine numerical embeddings on the GPU against the reference.

`CosineEmbeddingsPack` outputs and parameter gradients must match the reference's own
fixtures (ragged `d_embedding`) to the fp32 tolerance (1e-4 relative to the largest
element), the row-segmented backward must match the numpy oracle on a batch large enough
to split, and a whole `TabPack` with cosine embeddings of per-member size and one-hot
features must reproduce the reference's training step (output and every gradient).
"""

import numpy as np
import pytest
import torch

from oracle import layers as ol

pytestmark = pytest.mark.gpu

KEYS = ('weight', 'bias', 'elementwise_affine_weight', 'elementwise_affine_bias')


@pytest.fixture(scope='module', autouse=True)
def _gpu():
    if not torch.cuda.is_available():
        pytest.skip('needs a GPU')


def _rel(a, b):
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


def _module_from(params, d_embedding, device='cuda'):
    from tabpack_b200.nn import CosineEmbeddingsPack

    P, F, D = params['elementwise_affine_weight'].shape
    emb = CosineEmbeddingsPack(F, [int(v) for v in d_embedding], max_d_embedding=D, init_scale=[0.1] * P,
                               pack_size=P).to(device)
    with torch.no_grad():
        for k in KEYS:
            getattr(emb, k).copy_(torch.from_numpy(np.asarray(params[k])).float())
    return emb


@pytest.mark.parametrize('name', ['cosine_fp64.npz', 'cosine_fp32.npz'])
def test_cosine_embeddings_match_reference(golden, name):
    g = golden(name)
    emb = _module_from({k: g['param.' + k] for k in KEYS}, g['d_embedding'])
    x = torch.from_numpy(g['x']).float().cuda()
    y = emb(x)
    assert y.shape == g['y'].shape
    assert _rel(y.detach().cpu().numpy(), g['y']) < 1e-4
    (y * torch.from_numpy(g['dy']).float().cuda()).sum().backward()
    for k in KEYS:
        got = getattr(emb, k).grad.cpu().numpy()
        assert _rel(got, g['grad.' + k]) < 1e-4, k


@pytest.mark.parametrize('shared', [False, True])
def test_cosine_embeddings_segmented_backward_matches_oracle(shared):
    """3000 rows over 6 members: the backward splits the rows into segments whose fp64 sums
    are added in order by a second launch."""
    rng = np.random.default_rng(4)
    P, B, F, D = 6, 3000, 20, 16
    prm = {'weight': rng.standard_normal((P, F, D - 1)) * 0.3, 'bias': rng.standard_normal((P, F, D - 1)),
           'elementwise_affine_weight': rng.standard_normal((P, F, D)),
           'elementwise_affine_bias': rng.standard_normal((P, F, D))}
    prm = {k: v.astype(np.float32) for k, v in prm.items()}
    d = np.array([16, 3, 9, 1, 12, 16])
    x = rng.standard_normal((B, F) if shared else (P, B, F)).astype(np.float32)
    emb = _module_from(prm, d)
    yx = emb(torch.from_numpy(x).cuda().expand(P, B, F) if shared else torch.from_numpy(x).cuda())
    gy = rng.standard_normal((P, B, F, D)).astype(np.float32)
    (yx * torch.from_numpy(gy).cuda()).sum().backward()
    xs = np.broadcast_to(x, (P, B, F)).astype(np.float64)
    want, cache = ol.cosine_embeddings_forward(xs, *[prm[k].astype(np.float64) for k in KEYS], d)
    assert _rel(yx.detach().cpu().numpy(), want) < 1e-4
    for k, w in zip(KEYS, ol.cosine_embeddings_backward(cache, gy.astype(np.float64))):
        assert _rel(getattr(emb, k).grad.cpu().numpy(), w) < 1e-4, k


def test_cosine_embeddings_bf16_output_and_gradient():
    """bf16 output (first layer's dtype under autocast) and a bf16 upstream gradient."""
    from tabpack_b200 import ops

    rng = np.random.default_rng(5)
    P, B, F, D = 3, 257, 7, 5
    t = lambda a: torch.from_numpy(a.astype(np.float32)).cuda().contiguous()  # noqa: E731
    w, b = t(rng.standard_normal((P, F, D - 1))), t(rng.standard_normal((P, F, D - 1)))
    aw, ab = t(rng.standard_normal((P, F, D))), t(rng.standard_normal((P, F, D)))
    x = t(rng.standard_normal((P, B, F)))
    out = torch.zeros(P, B, F * D + 6, dtype=torch.bfloat16, device='cuda')  # wider: a one-hot block follows
    ops.cos_emb_forward(x, w, b, aw, ab, None, out=out)
    want, cache = ol.cosine_embeddings_forward(x.cpu().double().numpy(), *[v.cpu().double().numpy()
                                                                           for v in (w, b, aw, ab)])
    got = out[..., : F * D].float().cpu().numpy().reshape(P, B, F, D)
    assert _rel(got, want) < 2 ** -7
    assert torch.count_nonzero(out[..., F * D:]) == 0
    gy = torch.from_numpy(rng.standard_normal((P, B, F * D)).astype(np.float32)).cuda().bfloat16()
    grads = ops.cos_emb_backward(x, w, b, aw, ab, None, gy)
    for got, wt in zip(grads, ol.cosine_embeddings_backward(cache, gy.float().cpu().double().numpy()
                                                            .reshape(P, B, F, D))):
        assert _rel(got.cpu().numpy(), wt) < 1e-4


def test_tabpack_with_cosine_embeddings_matches_reference(golden):
    """A TabPack training step with per-member embedding sizes and one-hot features: the
    first layer multiplies the full padded input width, like the reference."""
    from tabpack_b200 import nn as bnn

    g = golden('tabpack_cosine_fp64.npz')
    P = g['x_num'].shape[0]
    model = bnn.TabPack(
        n_numerical_features=g['x_num'].shape[-1], categorical_cardinalities=[3, 2], d_out=g['y'].shape[-1],
        n_blocks=[2, 1, 2], d_block=[16, 8, 12], dropout=[0.1, 0.0, 0.2], pack_size=P,
        numerical_embeddings={'type': bnn.CosineEmbeddingsPack, 'd_embedding': [4, 6, 3], 'max_d_embedding': 6,
                              'init_scale': [0.1, 0.05, 0.2]})
    sd = {k[len('param.'):]: torch.from_numpy(g[k]) for k in g.files if k.startswith('param.')}
    assert set(sd) == set(model.state_dict()), sorted(set(sd) ^ set(model.state_dict()))
    model.load_state_dict(sd)
    model.cuda().train()
    model.backbone._stream.seed = int(g['seed'])
    y = model(torch.from_numpy(g['x_num']).float().cuda(), torch.from_numpy(g['x_cat']).cuda())
    assert _rel(y.detach().cpu().numpy(), g['y']) < 1e-4
    (y * torch.from_numpy(g['dy']).float().cuda()).sum().backward()
    for k, p in model.named_parameters():
        assert _rel(p.grad.cpu().numpy(), g['grad.' + k]) < 1e-4, k


def _cosine_model(P=4):
    from tabpack_b200 import nn as bnn

    return bnn.TabPack(
        n_numerical_features=6, categorical_cardinalities=[5, 3, 9], d_out=2, n_blocks=[1, 2, 3, 2][:P],
        d_block=[32, 16, 48, 24][:P], dropout=[0.1, 0.2, 0.0, 0.3][:P], pack_size=P, max_d_block=48,
        numerical_embeddings={'type': bnn.CosineEmbeddingsPack, 'd_embedding': [4, 8, 3, 6][:P], 'max_d_embedding': 8,
                              'init_scale': [0.1, 0.05, 0.2, 0.1][:P]}).cuda()


@pytest.mark.parametrize('rows', [False, True])
def test_embedded_first_layer_input_equals_concat(rows):
    """Under bf16 autocast the first layer's input [embeddings | one-hot] is built in one bf16
    buffer and the embedding gradient is read from the input's gradient in place; outputs and
    every gradient equal the generic path (embedding, one-hot, concat, cast) bit for bit."""
    torch.manual_seed(2)
    model = _cosine_model().train()
    g = torch.Generator(device='cuda').manual_seed(4)
    N, B = 300, 200
    x_num = torch.randn(N, 6, device='cuda', generator=g)
    x_cat = torch.stack([torch.randint(0, c + 1, (N,), device='cuda', generator=g) for c in (5, 3, 9)], -1)
    idx = torch.randint(0, N, (4, B), device='cuda', generator=g)
    dy = torch.randn(4, B if rows else N, 2, device='cuda', generator=g)

    def run(embedded):
        model.zero_grad(set_to_none=True)
        model.backbone._stream.seed, model.backbone._stream.calls = 11, 0
        if not embedded:
            model._embedded_input = lambda *a, **k: None
        try:
            with torch.autocast('cuda', dtype=torch.bfloat16):
                y = model.forward_rows(x_num, x_cat, idx) if rows else model(x_num, x_cat)
            (y.float() * dy).sum().backward()
        finally:
            model.__dict__.pop('_embedded_input', None)
        return y.detach(), {k: p.grad.clone() for k, p in model.named_parameters() if p.grad is not None}

    y1, g1 = run(True)
    y0, g0 = run(False)
    assert torch.equal(y1, y0)
    assert set(g1) == set(g0)
    for k in g0:
        assert torch.equal(g1[k], g0[k]), k


def test_cosine_embeddings_model_predicts_in_eval_mode():
    """A shared 2-D batch is a valid evaluation input with numerical embeddings (the
    per-member embedding is internal); a per-member 3-D batch still needs training mode."""
    model = _cosine_model().eval()
    g = torch.Generator(device='cuda').manual_seed(7)
    x_num = torch.randn(50, 6, device='cuda', generator=g)
    x_cat = torch.stack([torch.randint(0, c, (50,), device='cuda', generator=g) for c in (5, 3, 9)], -1)
    with torch.autocast('cuda', dtype=torch.bfloat16):
        y = model(x_num, x_cat)
    assert y.shape == (4, 50, 2) and torch.isfinite(y).all()
    with torch.no_grad():
        y32 = model(x_num, x_cat)
    assert (y.float() - y32).abs().max() < 5e-2 * y32.abs().max()
    with pytest.raises(RuntimeError, match='training mode'):
        model(x_num.expand(4, 50, 6), x_cat.expand(4, 50, 3))
