"""Generate the golden fixtures in this directory by running the reference itself.

Run from the repository root, in a container where the reference's sources are
available (they are pure Python on top of PyTorch):

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden.py PATH/TO/tabpack/src [FIXTURE ...]

The reference (Abusagit/tabpack, package `tabpackage` 0.0.1) is imported
unmodified.  Its only source of nondeterminism on the hot path is the dropout
draw `torch.empty_like(x).bernoulli_(p_keep)` in `DropoutPack.forward`
(`src/tabpackage/nn.py:897-901`); for the fixtures that call is replaced by the
counter-based Philox keep mask of `oracle.philox`, injected as the same
`mask / p_keep` tensor the reference would have multiplied with.  Everything
else (padded `baddbmm`, masking, depth `where`, autograd, optimizer packs,
metrics, greedy selection) is the reference's own code path.

Each fixture is an `.npz` of small arrays; `tests/test_oracle_golden.py` pins
the numpy oracle against them and the GPU tests pin the CUDA path against the
oracle.
"""

from __future__ import annotations

import functools
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))


def _import_reference(src: str):
    sys.path.insert(0, src)
    sys.path.insert(0, ROOT)
    import tabpackage  # noqa: F401
    import tabpackage.ensemble
    import tabpackage.metrics
    import tabpackage.nn
    import tabpackage.optim

    return tabpackage


def _np(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().numpy().copy()


class _PhiloxDropout:
    """Context manager replacing the Bernoulli draw of `DropoutPack.forward` by
    the Philox keep mask; the k-th training-mode call uses offset k."""

    def __init__(self, tp, seed: int):
        self.tp = tp
        self.seed = seed
        self.calls = 0

    def __enter__(self):
        from oracle.layers import dropout_mask_values

        DropoutPack = self.tp.nn.DropoutPack
        self.orig = DropoutPack.forward
        ctx = self

        def forward(mod, x, pack_idx=None):
            if isinstance(mod.p, (int, float)) or not mod.training:
                return ctx.orig(mod, x, pack_idx)
            p = mod.p if pack_idx is None else mod.p[pack_idx]
            members = (np.arange(x.shape[0]) if pack_idx is None else _np(pack_idx)).astype(np.uint32)
            mv = dropout_mask_values(
                seed=ctx.seed, offset=ctx.calls, members=members, n_rows=x.shape[1],
                n_cols=x.shape[2], p=_np(p), dtype=np.float64,
            )
            ctx.calls += 1
            return torch.from_numpy(mv).to(x.dtype) * x

        DropoutPack.forward = forward
        return self

    def __exit__(self, *exc):
        self.tp.nn.DropoutPack.forward = self.orig


def make_block(tp, dtype, name):
    torch.manual_seed(1)
    P, B, max_in, max_out = 6, 37, 40, 48
    in_f = [40, 16, 33, 8, 24, 40]
    out_f = [48, 16, 20, 47, 9, 32]
    p = [0.0, 0.1, 0.25, 0.5, 0.3, 0.05]
    blk = tp.nn.MLPBackbonePack.Block(
        in_features=in_f, out_features=out_f, max_in_features=max_in,
        max_out_features=max_out, activation={'type': torch.nn.ReLU}, dropout=p,
        pack_size=P,
    ).to(dtype)
    blk.train()
    x = torch.randn(P, B, max_in, dtype=dtype)
    x = x * (torch.arange(max_in)[None] < torch.tensor(in_f)[:, None]).to(dtype)[:, None, :]
    x.requires_grad_(True)
    seed = 0x1234_5678_9ABC
    with _PhiloxDropout(tp, seed) as _:
        y = blk(x)
    dy = torch.randn_like(y)
    (y * dy).sum().backward()
    np.savez_compressed(
        os.path.join(HERE, name),
        x=_np(x), weight=_np(blk.linear.weight), bias=_np(blk.linear.bias),
        in_features=np.array(in_f, np.int32), out_features=np.array(out_f, np.int32),
        p=np.array(p, np.float32), seed=np.uint64(seed), offset=np.uint32(0),
        y=_np(y), dy=_np(dy), dx=_np(x.grad), dweight=_np(blk.linear.weight.grad),
        dbias=_np(blk.linear.bias.grad),
    )


def make_tabpack(tp, dtype, name, forward_impl='dense'):
    torch.manual_seed(2)
    P, B = 5, 29
    n_num, cards, d_out = 5, [3, 4], 3
    n_blocks = [1, 3, 2, 3, 1]
    d_block = [8, 24, 16, 32, 12]
    dropout = [0.1, 0.0, 0.3, 0.2, 0.45]
    model = tp.nn.TabPack(
        n_numerical_features=n_num, categorical_cardinalities=cards, d_out=d_out,
        n_blocks=n_blocks, d_block=d_block, dropout=dropout, pack_size=P,
        forward_impl=forward_impl,
    ).to(dtype)
    model.train()
    x_num = torch.randn(P, B, n_num, dtype=dtype)
    x_cat = torch.stack([torch.randint(0, c + 1, (P, B)) for c in cards], -1)
    seed = 77
    torch.set_default_dtype(dtype)
    try:
        with _PhiloxDropout(tp, seed):
            y = model(x_num, x_cat)
    finally:
        torch.set_default_dtype(torch.float32)
    dy = torch.randn_like(y)
    (y * dy).sum().backward()
    arrays = {
        'x_num': _np(x_num), 'x_cat': _np(x_cat), 'y': _np(y), 'dy': _np(dy),
        'n_blocks': np.array(n_blocks, np.int32), 'd_block': np.array(d_block, np.int32),
        'dropout': np.array(dropout, np.float32), 'cards': np.array(cards, np.int32),
        'seed': np.uint64(seed),
    }
    for k, v in model.state_dict().items():
        arrays['param.' + k] = _np(v)
    for k, v in model.named_parameters():
        arrays['grad.' + k] = _np(v.grad)
    np.savez_compressed(os.path.join(HERE, name), **arrays)


def _randomize_cosine(emb, gen):
    """The affine parameters start at zero (`nn.py:1742-1753`), which would make the
    embedding output and most gradients vanish; give them random values."""
    with torch.no_grad():
        for prm in (emb.bias, emb.elementwise_affine_weight, emb.elementwise_affine_bias):
            prm.copy_(torch.randn(prm.shape, generator=gen, dtype=prm.dtype))


def make_cosine(tp, dtype, name):
    """`CosineEmbeddingsPack` forward/backward with per-member embedding sizes."""
    torch.manual_seed(8)
    gen = torch.Generator().manual_seed(9)
    P, B, F = 4, 23, 6
    emb = tp.nn.CosineEmbeddingsPack(F, [3, 5, 8, 2], max_d_embedding=8, init_scale=[0.01, 0.1, 1.0, 0.3],
                                     pack_size=P).to(dtype)
    _randomize_cosine(emb, gen)
    x = torch.randn(P, B, F, dtype=dtype, generator=gen)
    y = emb(x)
    dy = torch.randn(y.shape, dtype=dtype, generator=gen)
    (y * dy).sum().backward()
    arrays = {'x': _np(x), 'y': _np(y), 'dy': _np(dy), 'd_embedding': _np(emb.d_embedding).astype(np.int32)}
    for k in ('weight', 'bias', 'elementwise_affine_weight', 'elementwise_affine_bias'):
        arrays['param.' + k] = _np(getattr(emb, k))
        arrays['grad.' + k] = _np(getattr(emb, k).grad)
    np.savez_compressed(os.path.join(HERE, name), **arrays)


def make_tabpack_cosine(tp, dtype, name):
    """`TabPack` with cosine numerical embeddings of per-member size and one-hot
    categorical features: the first layer's input is not a masked prefix (each member's
    embedding columns sit at f * max_d + k, the one-hot block after them)."""
    torch.manual_seed(10)
    gen = torch.Generator().manual_seed(11)
    P, B = 3, 31
    n_num, cards, d_out = 4, [3, 2], 2
    model = tp.nn.TabPack(
        n_numerical_features=n_num, categorical_cardinalities=cards, d_out=d_out,
        n_blocks=[2, 1, 2], d_block=[16, 8, 12], dropout=[0.1, 0.0, 0.2], pack_size=P,
        numerical_embeddings={'type': tp.nn.CosineEmbeddingsPack, 'd_embedding': [4, 6, 3], 'max_d_embedding': 6,
                              'init_scale': [0.1, 0.05, 0.2]},
    ).to(dtype)
    _randomize_cosine(model.num_module, gen)
    model.train()
    x_num = torch.randn(P, B, n_num, dtype=dtype, generator=gen)
    x_cat = torch.stack([torch.randint(0, c + 1, (P, B), generator=gen) for c in cards], -1)
    seed = 91
    torch.set_default_dtype(dtype)
    try:
        with _PhiloxDropout(tp, seed):
            y = model(x_num, x_cat)
    finally:
        torch.set_default_dtype(torch.float32)
    dy = torch.randn(y.shape, dtype=dtype, generator=gen)
    (y * dy).sum().backward()
    arrays = {'x_num': _np(x_num), 'x_cat': _np(x_cat), 'y': _np(y), 'dy': _np(dy), 'seed': np.uint64(seed)}
    for k, v in model.state_dict().items():
        arrays['param.' + k] = _np(v)
    for k, v in model.named_parameters():
        arrays['grad.' + k] = _np(v.grad)
    np.savez_compressed(os.path.join(HERE, name), **arrays)


def make_tabpack_large(tp, name):
    """A larger batch for the bf16 comparison (statistics over 384 rows), computed by
    the reference in fp64 and stored as fp32."""
    torch.manual_seed(8)
    P, B = 4, 384
    n_num, cards, d_out = 24, [6, 9], 2
    n_blocks = [3, 2, 3, 1]
    d_block = [64, 48, 32, 56]
    dropout = [0.1, 0.2, 0.0, 0.3]
    model = tp.nn.TabPack(
        n_numerical_features=n_num, categorical_cardinalities=cards, d_out=d_out,
        n_blocks=n_blocks, d_block=d_block, dropout=dropout, pack_size=P,
    )
    with torch.no_grad():  # parameters exactly representable in fp32
        for prm in model.parameters():
            prm.copy_(prm.float())
    model = model.to(torch.float64)
    model.train()
    x_num = torch.randn(P, B, n_num).double()
    x_cat = torch.stack([torch.randint(0, c + 1, (P, B)) for c in cards], -1)
    seed = 91
    torch.set_default_dtype(torch.float64)
    try:
        with _PhiloxDropout(tp, seed):
            y = model(x_num, x_cat)
    finally:
        torch.set_default_dtype(torch.float32)
    dy = torch.randn_like(y).float().double()
    (y * dy).sum().backward()
    arrays = {
        'x_num': _np(x_num).astype(np.float32), 'x_cat': _np(x_cat), 'y': _np(y).astype(np.float32),
        'dy': _np(dy).astype(np.float32), 'n_blocks': np.array(n_blocks, np.int32),
        'd_block': np.array(d_block, np.int32), 'dropout': np.array(dropout, np.float32),
        'cards': np.array(cards, np.int32), 'seed': np.uint64(seed),
    }
    for k, v in model.state_dict().items():
        v = _np(v)
        arrays['param.' + k] = v.astype(np.float32) if v.dtype == np.float64 else v
    for k, v in model.named_parameters():
        arrays['grad.' + k] = _np(v.grad).astype(np.float32)

    # The same step through the reference's own bf16 path (CPU autocast), the accuracy a
    # bf16 implementation is held to.
    ref16 = tp.nn.TabPack(
        n_numerical_features=n_num, categorical_cardinalities=cards, d_out=d_out,
        n_blocks=n_blocks, d_block=d_block, dropout=dropout, pack_size=P,
    )
    ref16.load_state_dict({k: v.float() if v.is_floating_point() else v for k, v in model.state_dict().items()})
    ref16.train()
    with _PhiloxDropout(tp, seed), torch.autocast('cpu', dtype=torch.bfloat16):
        y16 = ref16(x_num.float(), x_cat)
    (y16.float() * dy.float()).sum().backward()
    arrays['bf16ref.y'] = _np(y16.float())
    for k, v in ref16.named_parameters():
        arrays['bf16ref.grad.' + k] = _np(v.grad).astype(np.float32)
    np.savez_compressed(os.path.join(HERE, name), **arrays)


def make_adamw(tp):
    arrays = {}
    P = 4
    for case, (per_member, support_replacement) in enumerate(
        [(False, False), (True, False), (True, True), (False, True)]
    ):
        torch.manual_seed(10 + case)
        w = tp.nn.ParameterPack(torch.randn(P, 6, 5))
        b = tp.nn.ParameterPack(torch.randn(P, 6))
        if per_member:
            hp = dict(lr=[1e-3, 3e-3, 1e-2, 0.0], beta1=[0.9, 0.8, 0.95, 0.5],
                      beta2=[0.999, 0.95, 0.99, 0.9], eps=[1e-8, 1e-6, 1e-7, 1e-8],
                      weight_decay=[0.0, 1e-2, 1e-1, 1e-3])
        else:
            hp = dict(lr=3e-3, beta1=0.9, beta2=0.999, eps=1e-8, weight_decay=1e-2)
        opt = tp.optim.AdamWPack([w, b], pack_size=P, support_replacement=support_replacement, **hp)
        arrays[f'c{case}.w0'] = _np(w)
        arrays[f'c{case}.b0'] = _np(b)
        for k, v in hp.items():
            arrays[f'c{case}.hp.{k}'] = np.array(v, np.float64)
        for s in range(3):
            gw, gb = torch.randn_like(w) * 0.1, torch.randn_like(b) * 0.1
            w.grad, b.grad = gw.clone(), gb.clone()
            opt.step()
            arrays[f'c{case}.s{s}.gw'] = _np(gw)
            arrays[f'c{case}.s{s}.gb'] = _np(gb)
            arrays[f'c{case}.s{s}.w'] = _np(w)
            arrays[f'c{case}.s{s}.b'] = _np(b)
            arrays[f'c{case}.s{s}.m_w'] = _np(opt.state[w]['exp_avg'])
            arrays[f'c{case}.s{s}.v_w'] = _np(opt.state[w]['exp_avg_sq'])
        arrays[f'c{case}.per_member'] = np.array(per_member)
        arrays[f'c{case}.support_replacement'] = np.array(support_replacement)
    np.savez_compressed(os.path.join(HERE, 'adamw.npz'), **arrays)


def make_newton_schulz(tp):
    torch.manual_seed(3)
    arrays = {}
    for j, (r, c) in enumerate([(48, 32), (32, 48), (40, 40)]):
        G = torch.randn(3, r, c) * 0.02
        X = tp.optim._zeropower_via_newtonschulz5(G, steps=5)
        arrays[f'G{j}'] = _np(G)
        arrays[f'X{j}'] = _np(X.float())
    np.savez_compressed(os.path.join(HERE, 'newton_schulz.npz'), **arrays)


def make_muon(tp):
    torch.manual_seed(4)
    P = 3
    lin = tp.nn.LinearPack([24, 16, 32], [32, 16, 8], max_in_features=32,
                           max_out_features=32, pack_size=P)
    out = tp.nn.LinearPack(32, 2, pack_size=P)
    group = tp.optim.MuonAdamWPack.make_muon_parameter_group(lin)
    opt = tp.optim.MuonAdamWPack(
        [group, {'params': [lin.bias, out.weight, out.bias]}],
        adamw_lr=[1e-3, 2e-3, 5e-3], weight_decay=[1e-2, 0.0, 1e-3],
        muon_lr=[0.02, 0.01, 0.05], muon_momentum=[0.95, 0.9, 0.8], pack_size=P,
        allow_inplace_grad_mutation=True,
    )
    arrays = {'w0': _np(lin.weight), 'in_features': np.array([24, 16, 32], np.int32),
              'out_features': np.array([32, 16, 8], np.int32)}
    mask = (torch.arange(32)[None, :, None] < torch.tensor([32, 16, 8])[:, None, None]) & (
        torch.arange(32)[None, None, :] < torch.tensor([24, 16, 32])[:, None, None])
    for s in range(2):
        g = torch.randn_like(lin.weight) * 1e-3 * mask
        lin.weight.grad = g.clone()
        for prm in (lin.bias, out.weight, out.bias):
            prm.grad = torch.randn_like(prm) * 1e-3
        opt.step()
        arrays[f's{s}.g'] = _np(g)
        arrays[f's{s}.w'] = _np(lin.weight)
        arrays[f's{s}.mom'] = _np(opt.state[lin.weight]['muon_momentum_buffer'])
    arrays['scale'] = _np(group['muon_update_scale'])
    np.savez_compressed(os.path.join(HERE, 'muon.npz'), **arrays)


def make_metrics(tp):
    torch.manual_seed(5)
    M = tp.metrics
    P, N, C = 7, 101, 4
    yr = torch.randn(N)
    pr = torch.randn(P, N)
    yb = torch.randint(0, 2, (N,))
    pb = torch.rand(P, N).clamp(1e-6, 1 - 1e-6)
    pb[0, :3] = 0.0  # exercises the -100 clamp
    ym = torch.randint(0, C, (N,))
    pm = torch.softmax(torch.randn(P, N, C), -1)
    lab = torch.randint(0, C, (P, N))
    sc = torch.randn(P, N).round(decimals=1)  # ties for the midranks
    arrays = dict(yr=_np(yr), pr=_np(pr), yb=_np(yb), pb=_np(pb), ym=_np(ym), pm=_np(pm),
                  lab=_np(lab), sc=_np(sc))
    arrays['mse'] = _np(M.mse_pack(y_true=yr, y_pred=pr))
    arrays['mae'] = _np(M.mae_pack(y_true=yr, y_pred=pr))
    arrays['r2'] = _np(M.r2_pack(y_true=yr, y_pred=pr))
    arrays['bce'] = _np(M.binary_cross_entropy_pack(y_true=yb, y_proba=pb))
    arrays['ce'] = _np(M.multiclass_cross_entropy_pack(y_true=ym, y_proba=pm))
    arrays['acc'] = _np(M.accuracy_pack(y_true=ym, y_pred=lab))
    arrays['auc'] = _np(M.binary_roc_auc_pack(y_true=yb, y_score=sc))
    np.savez_compressed(os.path.join(HERE, 'metrics.npz'), **arrays)


def make_ensemble(tp):
    torch.manual_seed(6)
    E = tp.ensemble
    M = tp.metrics
    arrays = {}
    C, N = 14, 83
    y = torch.randn(N)
    preds = y[None] + torch.randn(C, N) * torch.linspace(0.3, 1.5, C)[:, None]
    preds[5] = preds[2]  # exact duplicate -> exact score ties
    arrays['reg.y'] = _np(y)
    arrays['reg.preds'] = _np(preds)
    score = lambda p: -M.mse_pack(y_true=y, y_pred=p)  # noqa: E731
    for j, kw in enumerate([
        dict(), dict(init_top_k=3), dict(max_ensemble_size=4),
        dict(with_replacement=True, max_ensemble_size=12),
        dict(with_replacement=True, max_ensemble_size=20, init_top_k=2),
    ]):
        idx, w = E.greedy_ensemble(preds, score_fn=score, **kw)
        arrays[f'reg.k{j}.idx'] = _np(idx)
        if w is not None:
            arrays[f'reg.k{j}.w'] = _np(w)
    arrays['reg.top3'] = _np(E.topk_ensemble(preds, score_fn=score, k=3))

    K = 3
    yc = torch.randint(0, K, (N,))
    logits = torch.randn(C, N, K) + 2.0 * torch.nn.functional.one_hot(yc, K)[None] * torch.rand(C, 1, 1)
    probs = torch.softmax(logits, -1)
    arrays['cls.y'] = _np(yc)
    arrays['cls.probs'] = _np(probs)
    score_ce = lambda p: -M.multiclass_cross_entropy_pack(y_true=yc, y_proba=p)  # noqa: E731
    idx, _ = E.greedy_ensemble(probs, score_fn=score_ce, max_ensemble_size=6)
    arrays['cls.idx'] = _np(idx)
    wts = torch.rand(4)
    arrays['mean.w'] = _np(wts)
    arrays['mean.out'] = _np(E.compute_unsanitized_ensemble_predictions(probs[:4], wts))
    arrays['mean.out_eq'] = _np(E.compute_unsanitized_ensemble_predictions(probs[:4], None))
    np.savez_compressed(os.path.join(HERE, 'ensemble.npz'), **arrays)


def make_init(tp):
    """`LinearPack.reset_parameters` (`nn.py:702-747`) from a seeded global RNG: ragged
    per-member input widths, a shared width, and a re-initialisation of selected members."""
    arrays = {}
    torch.manual_seed(12)
    lin = tp.nn.LinearPack([40, 16, 33], [48, 16, 20], max_in_features=40, max_out_features=48, pack_size=3)
    arrays['ragged.weight'], arrays['ragged.bias'] = _np(lin.weight), _np(lin.bias)
    torch.manual_seed(13)
    lin.reset_parameters(pack_idx=torch.tensor([2, 0]))
    arrays['ragged.reset.weight'], arrays['ragged.reset.bias'] = _np(lin.weight), _np(lin.bias)
    torch.manual_seed(14)
    shared = tp.nn.LinearPack(24, 12, pack_size=4)
    arrays['shared.weight'], arrays['shared.bias'] = _np(shared.weight), _np(shared.bias)
    torch.manual_seed(15)
    shared.reset_parameters(pack_idx=torch.tensor([1]))
    arrays['shared.reset.weight'], arrays['shared.reset.bias'] = _np(shared.weight), _np(shared.bias)
    np.savez_compressed(os.path.join(HERE, 'init.npz'), **arrays)


def make_training(tp, dtype=torch.float32, name='train_config1.npz'):
    """The reference's own `train` (`_training.py:3068-3296`) on the 16-member CPU plumbing
    run (`synthetic.py`): AdamW, 20 epochs, per-member best checkpoints by validation
    MSE and an online greedy ensemble (at most 32 members) built and scored on validation
    MSE after every epoch.  Three inputs are injected so that a run of this package can be
    compared with it on the same footing:

    * the initial parameters: this package's `init_member_parameters_` drawn on host
      generators (the same distribution as `LinearPack.reset_parameters`), loaded into the
      reference's `TabPack` right after it is built;
    * the batch order: the stable argsort of the Philox permutation keys
      (`oracle.philox.permutation_keys`) in place of `make_shuffled_batch_indices_pack`'s
      `torch.rand(...).argsort()` (`_training.py:323-338`);
    * the dropout masks: the Philox keep mask (`oracle.layers.dropout_mask_values`) in place
      of `bernoulli_` (`nn.py:897-901`), block i of the k-th training forward at offset
      k * max_n_blocks + i, members keyed by their model id.

    Everything else -- forward, loss, backward, `AdamWPack.step`, evaluation, best-checkpoint
    bookkeeping, `Ensemble.update` and `greedy_ensemble` -- is the reference's code.

    With dtype=float64 the model (parameters, activations, optimizer state) runs in fp64;
    the data stay fp32 as `train` requires and the model's output is cast to fp32 by the
    reference's `forward` (`_training.py:154-167`).  That run is the yardstick for how far
    rounding alone moves this training: the fp32 run's distance from it is the reference's
    own rounding drift.
    """
    sys.path.insert(0, HERE)
    import synthetic

    from oracle.layers import dropout_mask_values
    from oracle.philox import permutation_keys
    from tabpack_b200.nn import TabPack as OwnTabPack
    from tabpack_b200.training import _mix, init_member_parameters_

    seed = 0
    data = synthetic.datasets(0)
    hp = synthetic.hyperparameters(1)
    P = len(hp)
    nb = [h['model']['n_blocks'] for h in hp]
    db = [h['model']['d_block'] for h in hp]
    dp = [h['model']['dropout'] for h in hp]
    lr = [h['optimizer']['lr'] for h in hp]
    max_nb, max_db = max(nb), max(db)
    own = OwnTabPack(n_numerical_features=synthetic.N_NUM, categorical_cardinalities=synthetic.CARDS, d_out=1,
                     n_blocks=nb, d_block=db, dropout=dp, pack_size=P, max_n_blocks=max_nb, max_d_block=max_db)
    init_member_parameters_(own, seed=seed, member_ids=list(range(P)), generator_device='cpu')
    init_state = {k: v.clone() for k, v in own.state_dict().items()}

    ref_tabpack = tp.nn.TabPack
    ref_shuffle = tp._training.make_shuffled_batch_indices_pack
    ref_dropout = tp.nn.DropoutPack.forward
    block_of = {}
    state = {'epoch': 0, 'forwards': 0}

    class InitialisedTabPack(ref_tabpack):
        def __init__(self, **kw):
            # built in fp32 (the reference's initialisation mixes fp32 bounds into the
            # parameters' dtype), then cast; the forward's one-hot block follows the default
            # dtype, which stays `dtype` for the whole run
            prev = torch.get_default_dtype()
            torch.set_default_dtype(torch.float32)
            try:
                super().__init__(**kw)
            finally:
                torch.set_default_dtype(prev)
            self.load_state_dict(init_state, strict=True)
            self.to(dtype)
            for i, b in enumerate(self.backbone.blocks):
                block_of[id(b.dropout)] = i

        def forward(self, x_num=None, x_cat=None, *args, **kw):
            return super().forward(None if x_num is None else x_num.to(dtype), x_cat, *args, **kw)

    def shuffled(*, total_size, batch_size, pack_size, generator=None, device=None):
        keys = permutation_keys(seed=_mix(seed, 0xBA), epoch=state['epoch'], members=np.arange(pack_size),
                                n_rows=total_size)
        state['epoch'] += 1
        order = torch.from_numpy(np.argsort(keys, axis=1, kind='stable')).to(device)
        return list(order.split(batch_size, dim=1))

    def dropout(mod, x, pack_idx=None):
        if not mod.training:
            return ref_dropout(mod, x, pack_idx)
        assert pack_idx is None
        i = block_of[id(mod)]
        if i == 0:
            state['forwards'] += 1
        offset = (state['forwards'] - 1) * max_nb + i
        mv = dropout_mask_values(seed=_mix(seed, 0xD0), offset=offset, members=np.arange(x.shape[0]),
                                 n_rows=x.shape[1], n_cols=x.shape[2], p=_np(mod.p), dtype=np.float32)
        return torch.from_numpy(mv).to(x.dtype) * x

    def mse_loss(y_pred, y):
        return ((y_pred.squeeze(-1) - y) ** 2).mean(1)

    def ensemble_mse(*, y_true, y_pred):
        # an ensemble's metric is a scalar: the pack metric of a one-member pack, as the
        # reference's sklearn layer wraps it (`sklearn/_config.py:221`)
        return tp.metrics.mse_pack(y_true=y_true, y_pred=y_pred.unsqueeze(0))[0]

    torch_data = {k: {n: torch.from_numpy(a) for n, a in v.items()} for k, v in data.items()}
    crit = tp.EvalCriterionConfig(dataset='val', metric='mse', metric_direction='minimize')
    ens = tp.EnsembleConfig(
        algorithm={'type': tp.ensemble.greedy_ensemble, 'max_ensemble_size': 32}, online=True,
        prediction_transform=None, early_stopping_patience=None, algorithm_metric=tp.metrics.mse_pack,
        algorithm_metric_direction='minimize', algorithm_dataset='val', algorithm_device=torch.device('cpu'))
    tp.nn.TabPack = InitialisedTabPack
    tp._training.make_shuffled_batch_indices_pack = shuffled
    tp.nn.DropoutPack.forward = dropout
    torch.set_default_dtype(dtype)
    try:
        res = tp.train(
            datasets=torch_data, model={'d_out': 1, 'categorical_cardinalities': synthetic.CARDS},
            prediction_transform=functools.partial(torch.squeeze, dim=-1), loss_fn=mse_loss,
            optimizer={'type': tp.optim.AdamWPack, 'weight_decay': synthetic.WEIGHT_DECAY},
            batch_size=synthetic.BATCH, max_epochs=20, early_stopping_patience=None, per_model_hyperparameters=hp,
            eval_metrics={'val': {'mse': tp.metrics.mse_pack}}, eval_criterion=crit, ensembles={'greedy': ens},
            ensemble_eval_metrics={'val': {'mse': ensemble_mse}}, ensemble_eval_criterion=crit,
            stop_when_all_ensembles_are_finalized=False, seed=seed, device='cpu', aux_device='cpu',
            autocast_dtype=None, print_progress=False, show_progress_bar=False)
    finally:
        torch.set_default_dtype(torch.float32)
        tp.nn.TabPack = ref_tabpack
        tp._training.make_shuffled_batch_indices_pack = ref_shuffle
        tp.nn.DropoutPack.forward = ref_dropout
    hist = res.load_model_history()
    ids = torch.arange(P)
    arrays = {
        'n_blocks': np.array(nb, np.int32), 'd_block': np.array(db, np.int32), 'dropout': np.array(dp, np.float32),
        'lr': np.array(lr, np.float64), 'seed': np.int64(seed), 'max_epochs': np.int32(20),
        'epoch_step': np.array([h['training_loop_step'] for h in hist], np.int64),
        'epoch_val_mse': np.stack([_np(h['metrics']['val']['mse']) for h in hist]),
        'best_step': _np(res.load_model_steps(ids)),
        'best_val_mse': _np(res.load_model_metrics(ids)['val']['mse']),
        'ensemble_ids': _np(res.load_ensemble_member_ids('greedy')),
        'ensemble_steps': _np(res.load_ensemble_member_steps('greedy')),
        'ensemble_val_mse': np.float64(res.load_ensemble_metrics('greedy')['val']['mse']),
    }
    eh = res.load_ensemble_history('greedy')
    arrays['update_step'] = np.array([u['training_loop_step'] for u in eh], np.int64)
    arrays['update_val_mse'] = np.array([float(u['metrics']['val']['mse']) for u in eh], np.float64)
    arrays['update_sizes'] = np.array([len(u['members']['ids']) for u in eh], np.int32)
    arrays['update_ids'] = np.concatenate([_np(u['members']['ids']) for u in eh])
    arrays['update_steps'] = np.concatenate([_np(u['members']['steps']) for u in eh])
    np.savez_compressed(os.path.join(HERE, name), **arrays)


FIXTURES = {
    'block': lambda tp: (make_block(tp, torch.float64, 'block_fp64.npz'),
                         make_block(tp, torch.float32, 'block_fp32.npz')),
    'tabpack': lambda tp: (make_tabpack(tp, torch.float64, 'tabpack_fp64.npz'),
                           make_tabpack(tp, torch.float64, 'tabpack_indexed_fp64.npz', forward_impl='indexed'),
                           make_tabpack_large(tp, 'tabpack_large.npz')),
    'cosine': lambda tp: (make_cosine(tp, torch.float64, 'cosine_fp64.npz'),
                          make_cosine(tp, torch.float32, 'cosine_fp32.npz'),
                          make_tabpack_cosine(tp, torch.float64, 'tabpack_cosine_fp64.npz')),
    'adamw': lambda tp: make_adamw(tp),
    'newton_schulz': lambda tp: make_newton_schulz(tp),
    'muon': lambda tp: make_muon(tp),
    'metrics': lambda tp: make_metrics(tp),
    'ensemble': lambda tp: make_ensemble(tp),
    'init': lambda tp: make_init(tp),
    'training': lambda tp: make_training(tp),
    'training_fp64': lambda tp: make_training(tp, torch.float64, 'train_config1_fp64.npz'),
}


def main():
    """`make_golden.py SRC [FIXTURE ...]`: SRC is the reference's `src` directory (or set
    TABPACK_REFERENCE_SRC); with no FIXTURE names every fixture is written."""
    args = sys.argv[1:]
    src = args.pop(0) if args else os.environ.get('TABPACK_REFERENCE_SRC')
    if not src:
        sys.exit('usage: make_golden.py REFERENCE_SRC [FIXTURE ...] (or set TABPACK_REFERENCE_SRC); '
                 f'fixtures: {", ".join(FIXTURES)}')
    unknown = [a for a in args if a not in FIXTURES]
    if unknown:
        sys.exit(f'unknown fixtures {unknown}; choose from {", ".join(FIXTURES)}')
    tp = _import_reference(src)
    for name in args or FIXTURES:
        FIXTURES[name](tp)
    print('fixtures written to', HERE)


if __name__ == '__main__':
    main()
