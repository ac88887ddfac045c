"""The gathered one-hot first layer (bf16) against the dense one-hot first layer.

Under bf16 autocast a TabPack with categorical features can run its first layer as a
gather-sum: the dense columns on the tensor cores with K = n_dense, one weight column per
categorical feature and row added before the bias / ReLU / dropout, and the one-hot columns
of the weight gradient as segmented sums over each category's rows.  Forwards without a
backward use it by default; training uses it with `gather_one_hot_in_training`.  Both paths
round the same fp32 sums to bf16 once, so outputs and gradients must agree to the bf16
tolerance (2e-2 relative, the bar for bf16 work).
"""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope='module', autouse=True)
def _gpu():
    if not torch.cuda.is_available():
        pytest.skip('needs a GPU')


def _rel(a, b):
    a, b = a.detach().float().cpu().numpy(), b.detach().float().cpu().numpy()
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


def _run(model, x_num, x_cat, gathered: bool, seed=7, row_index=None):
    """Output and parameter gradients of one bf16 training step, on the gathered or the
    dense one-hot path (the same dropout masks either way)."""
    model.gather_one_hot_in_training = True
    model.zero_grad(set_to_none=True)
    model.backbone._stream.seed, model.backbone._stream.calls = seed, 0
    if not gathered:
        model._gathered = lambda *a, **k: None
    try:
        with torch.autocast('cuda', dtype=torch.bfloat16):
            y = model.forward_rows(x_num, x_cat, row_index) if row_index is not None else model(x_num, x_cat)
        g = torch.Generator(device='cuda').manual_seed(5)
        dy = torch.randn(y.shape, device='cuda', generator=g)
        (y.float() * dy).sum().backward()
    finally:
        model.__dict__.pop('_gathered', None)
        model.gather_one_hot_in_training = False
    return y.detach(), {k: p.grad.detach().clone() for k, p in model.named_parameters() if p.grad is not None}


def _compare(model, x_num, x_cat, row_index=None, bar=2e-2):
    y1, g1 = _run(model, x_num, x_cat, True, row_index=row_index)
    y0, g0 = _run(model, x_num, x_cat, False, row_index=row_index)
    assert y1.shape == y0.shape
    assert _rel(y1, y0) < bar
    assert set(g1) == set(g0)
    for k in g0:
        assert _rel(g1[k], g0[k]) < bar, k
    return y1, g1


@pytest.mark.parametrize('shared', [True, False])
def test_gathered_first_layer_matches_dense_one_hot(shared):
    """Ragged widths and depths, dropout, unknown / out-of-range categories, a feature of
    cardinality 1 and a batch that is not a power of two."""
    from tabpack_b200 import nn as bnn

    torch.manual_seed(0)
    P, B = 5, 300
    cards = [4, 1, 13, 2, 37]
    model = bnn.TabPack(n_numerical_features=7, categorical_cardinalities=cards, d_out=3,
                        n_blocks=[1, 2, 3, 2, 1], d_block=[32, 64, 16, 48, 24], dropout=[0.1, 0.0, 0.3, 0.2, 0.05],
                        pack_size=P, max_d_block=64).cuda().train()
    g = torch.Generator(device='cuda').manual_seed(1)
    lead = (B,) if shared else (P, B)
    x_num = torch.randn(*lead, 7, device='cuda', generator=g)
    # values up to card + 1: `card` is the unknown category, card + 1 lies outside the encoding
    x_cat = torch.stack([torch.randint(0, c + 2, lead, device='cuda', generator=g) for c in cards], -1)
    x_cat[..., 1] = torch.where(x_cat[..., 1] > 1, 1, x_cat[..., 1])  # card 1: values {0, 1(unknown)}
    _compare(model, x_num, x_cat)


def test_gathered_first_layer_forward_rows_and_many_features():
    """Dataset rows gathered per member (forward_rows) with 40 categorical features (more than
    one warp's worth in the gather) and no numerical features; the result equals gathering the
    batch first and running the same path."""
    from tabpack_b200 import nn as bnn

    torch.manual_seed(1)
    P, N, B = 3, 700, 129
    cards = [int(c) for c in np.random.default_rng(2).integers(1, 30, 40)]
    model = bnn.TabPack(n_numerical_features=0, categorical_cardinalities=cards, d_out=1, n_blocks=[2, 1, 3],
                        d_block=[40, 24, 56], dropout=[0.2, 0.1, 0.0], pack_size=P, max_d_block=56).cuda().train()
    g = torch.Generator(device='cuda').manual_seed(3)
    x_cat = torch.stack([torch.randint(0, c + 1, (N,), device='cuda', generator=g) for c in cards], -1)
    idx = torch.randint(0, N, (P, B), device='cuda', generator=g)
    y1, g1 = _compare(model, None, x_cat, row_index=idx)
    y2, g2 = _run(model, None, x_cat[idx], True)
    assert torch.equal(y1, y2)
    for k in g1:
        assert torch.equal(g1[k], g2[k]), k


def test_gathered_first_layer_with_cosine_embeddings():
    """Cosine numerical embeddings of per-member size before the one-hot block: the dense
    columns' gradient flows back into the embedding parameters."""
    from tabpack_b200 import nn as bnn

    torch.manual_seed(2)
    P, B = 4, 200
    model = bnn.TabPack(
        n_numerical_features=6, categorical_cardinalities=[5, 3, 9], d_out=2, n_blocks=[1, 2, 3, 2],
        d_block=[32, 16, 48, 24], dropout=[0.1, 0.2, 0.0, 0.3], pack_size=P, max_d_block=48,
        numerical_embeddings={'type': bnn.CosineEmbeddingsPack, 'd_embedding': [4, 8, 3, 6], 'max_d_embedding': 8,
                              'init_scale': [0.1, 0.05, 0.2, 0.1]}).cuda().train()
    g = torch.Generator(device='cuda').manual_seed(4)
    x_num = torch.randn(B, 6, device='cuda', generator=g)
    x_cat = torch.stack([torch.randint(0, c + 1, (B,), device='cuda', generator=g) for c in (5, 3, 9)], -1)
    _, grads = _compare(model, x_num, x_cat)
    assert any(k.startswith('num_module') for k in grads)


def test_gathered_first_layer_at_benchmark_shapes():
    """64 members, 1024 rows, 100 numerical features and 10 categorical features with
    cardinalities log-uniform in [2, 1000] (the one-hot block of the benchmarked model), widths
    U{128..1024 step 8}: each CTA runs several gathered tiles, and outputs and gradients must
    agree with the dense one-hot path."""
    from tabpack_b200 import nn as bnn

    torch.manual_seed(4)
    rng = np.random.default_rng(4)
    P, B = 64, 1024
    cards = [int(c) for c in np.exp(rng.uniform(np.log(2), np.log(1000), 10)).astype(int)]
    widths = [int(w) for w in rng.integers(16, 129, P) * 8]
    model = bnn.TabPack(n_numerical_features=100, categorical_cardinalities=cards, d_out=1,
                        n_blocks=[int(v) for v in rng.integers(1, 3, P)], d_block=widths,
                        dropout=[float(v) for v in rng.uniform(0, 0.5, P)], pack_size=P,
                        max_d_block=max(widths)).cuda().train()
    g = torch.Generator(device='cuda').manual_seed(8)
    x_num = torch.randn(B, 100, device='cuda', generator=g)
    x_cat = torch.stack([torch.randint(0, c + 1, (B,), device='cuda', generator=g) for c in cards], -1)
    _compare(model, x_num, x_cat)


def test_onehot_wgrad_is_the_segmented_sum():
    """dW over the one-hot columns equals sum over each category's rows of the
    pre-activation gradient, exactly as fp32 sums in ascending row order (no dropout, no
    ReLU: the pre-activation gradient is dy itself, rounded to bf16)."""
    from tabpack_b200 import ops

    P, B, max_out, n_dense = 2, 77, 24, 8
    cards = [3, 1, 6]
    offs = torch.tensor([0, 3, 4, 10], dtype=torch.int32, device='cuda')
    n_onehot = 10
    g = torch.Generator(device='cuda').manual_seed(9)
    W = torch.randn(P, max_out, n_dense + n_onehot, device='cuda', generator=g)
    outf = torch.tensor([24, 17], dtype=torch.int32, device='cuda')
    x = torch.randn(P, B, n_dense, device='cuda', generator=g).bfloat16()
    x_cat = torch.stack([torch.randint(0, c + 1, (P, B), device='cuda', generator=g) for c in cards], -1)
    wd = torch.zeros(P, max_out, n_dense, dtype=torch.bfloat16, device='cuda')
    ops.weight_cast(W, wd, out_features=outf, src_cols=n_dense)
    wt = torch.empty(P, n_onehot, max_out, dtype=torch.bfloat16, device='cuda')
    ops.weight_cast_transposed(W, wt, col0=n_dense, ncols=n_onehot, out_features=outf)
    y, st = ops.onehot_linear_forward(x, wd, None, x_cat=x_cat, cat_offsets=offs, n_dense=n_dense, w_onehot_t=wt,
                                      out_features=outf)
    dy = torch.randn(P, B, max_out, device='cuda', generator=g).bfloat16()
    _, dw, _ = ops.onehot_linear_backward(dy, x, wd, y, st, out_features=outf, need_db=False, dw_rows=max_out,
                                          db_cols=max_out)
    gm = dy.float().cpu()
    for m in range(P):
        o = int(outf[m])
        gm[m, :, o:] = 0
        for f, c in enumerate(cards):
            for v in range(c):
                rows = (x_cat[m, :, f] == v).nonzero().flatten().cpu().tolist()
                want = torch.zeros(max_out)
                for r in rows:
                    want += gm[m, r]
                assert torch.equal(dw[m, :, n_dense + int(offs[f]) + v].cpu(), want), (m, f, v)
    # forward: y = x Wd^T + sum of the gathered columns (rounded to bf16 once)
    wb = W.bfloat16().float()
    for m in range(P):
        o = int(outf[m])
        want = x[m].float() @ wb[m, :, :n_dense].T
        for f, c in enumerate(cards):
            v = x_cat[m, :, f]
            ok = v < c
            col = n_dense + int(offs[f]) + torch.clamp(v, max=c - 1)
            want += torch.where(ok[:, None], wb[m][:, col].T, 0.0)
        assert _rel(y[m, :, :o], want[:, :o].bfloat16()) < 2 ** -7
        assert torch.count_nonzero(y[m, :, o:]) == 0


def test_gathered_forward_is_the_default_without_grad():
    """Evaluation (no_grad, bf16) takes the gathered path, with no category sort, and agrees
    with the dense one-hot forward."""
    from tabpack_b200 import nn as bnn
    from tabpack_b200 import ops

    torch.manual_seed(3)
    P, B = 4, 333
    cards = [7, 2, 19]
    model = bnn.TabPack(n_numerical_features=5, categorical_cardinalities=cards, d_out=2, n_blocks=[1, 2, 3, 2],
                        d_block=[32, 16, 48, 24], dropout=[0.1] * P, pack_size=P, max_d_block=48).cuda().eval()
    g = torch.Generator(device='cuda').manual_seed(6)
    x_num = torch.randn(B, 5, device='cuda', generator=g)
    x_cat = torch.stack([torch.randint(0, c + 1, (B,), device='cuda', generator=g) for c in cards], -1)
    calls = []
    orig = ops.onehot_linear_forward

    def spy(*a, **k):
        calls.append(k.get('need_sort'))
        return orig(*a, **k)

    ops.onehot_linear_forward = spy
    try:
        with torch.no_grad(), torch.autocast('cuda', dtype=torch.bfloat16):
            y1 = model(x_num, x_cat)
    finally:
        ops.onehot_linear_forward = orig
    assert calls == [False]
    model._gathered = lambda *a, **k: None
    with torch.no_grad(), torch.autocast('cuda', dtype=torch.bfloat16):
        y0 = model(x_num, x_cat)
    del model._gathered
    assert _rel(y1, y0) < 2e-2
