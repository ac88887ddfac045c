"""Member-sharded training on one GPU: shard invariance, training progress, prediction.

Members are keyed by global id everywhere (initialisation, batch order, dropout) and
the kernels are deterministic, so training the pack as one shard or as two shards must
give bit-identical members.
"""

import numpy as np
import pytest
import torch

from oracle.philox import permutation_keys

pytestmark = pytest.mark.gpu


@pytest.fixture(scope='module', autouse=True)
def _gpu():
    if not torch.cuda.is_available():
        pytest.skip('needs a GPU')


def test_permutation_keys_match_oracle():
    from tabpack_b200 import ops

    got = ops.permutation_keys(seed=2**40 + 5, epoch=3, member_base=17, P=5, N=1031, device='cuda')
    want = permutation_keys(seed=2**40 + 5, epoch=3, members=np.arange(17, 22), n_rows=1031)
    assert np.array_equal(got.cpu().numpy(), want)


def _data(n, seed, dev):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(n, 12, generator=g)
    c = torch.randint(0, 4, (n, 2), generator=g)
    w = torch.randn(12, generator=g)
    y = torch.tanh(x @ w / 3) + 0.3 * (c[:, 0] == 1).float() + 0.1 * torch.randn(n, generator=g)
    return {'x_num': x.to(dev), 'x_cat': c.to(dev), 'y': y.to(dev)}


MODEL = dict(n_numerical_features=12, categorical_cardinalities=[3, 3], d_out=1, max_d_block=96, max_n_blocks=3)
PER_MEMBER = [dict(n_blocks=nb, d_block=db, dropout=p) for nb, db, p in
              [(1, 64, 0.1), (3, 96, 0.2), (2, 32, 0.0), (3, 48, 0.3), (2, 96, 0.1), (1, 16, 0.05)]]
# nine models through six slots (the replacement queue): shapes, dropout, Muon learning rate
REPLACE_MODELS = PER_MEMBER + [dict(n_blocks=2, d_block=80, dropout=0.15), dict(n_blocks=1, d_block=96, dropout=0.0),
                               dict(n_blocks=3, d_block=24, dropout=0.25)]
REPLACE_OPT = [dict(muon_lr=lr) for lr in (1e-2, 2e-2, 5e-3, 1e-2, 3e-2, 2e-2, 1.5e-2, 2.5e-2, 8e-3)]
REPLACE_MAX_EPOCHS = [2, 1, 3, 2, 1, 2, 1, 2, 1]


def _trainer(member_range, opt='muon'):
    from tabpack_b200.training import PackTrainer

    optim = (dict(type='muon', adamw_lr=3e-3, weight_decay=1e-4, muon_lr=2e-2) if opt == 'muon'
             else dict(type='adamw', lr=3e-3, weight_decay=1e-4))
    per_opt = [dict(**({'muon_lr': lr} if opt == 'muon' else {'lr': lr * 0.2}))
               for lr in (1e-2, 2e-2, 5e-3, 1e-2, 3e-2, 2e-2)]
    return PackTrainer(n_members=6, model=MODEL, per_member_model=PER_MEMBER, optimizer=optim,
                       per_member_optimizer=per_opt, loss='mse', seed=99, device='cuda', autocast_bf16=True,
                       member_range=member_range)


@pytest.mark.parametrize('opt', ['muon', 'adamw'])
def test_sharding_is_bit_invariant(opt):
    data = _data(640, 0, 'cuda')
    val = _data(300, 1, 'cuda')
    full = _trainer((0, 6), opt)
    a, b = _trainer((0, 4), opt), _trainer((4, 6), opt)
    for epoch in range(2):
        for t in (full, a, b):
            t.fit_epoch(data, batch_size=64, epoch=epoch)
    sd_full = full.model.state_dict()
    for shard, lo in ((a, 0), (b, 4)):
        for k, v in shard.model.state_dict().items():
            w = sd_full[k]
            if v.ndim == 0 or w.shape[1:] != v.shape[1:]:
                continue  # pack maxima (e.g. max widths) differ between shards
            assert torch.equal(v, w[lo: lo + v.shape[0]]), k
    pf = full.predict_local(val)
    pa, pb = a.predict_local(val), b.predict_local(val)
    assert torch.equal(torch.cat([pa, pb]), pf)


def test_training_reduces_loss_and_ensembles():
    from tabpack_b200.training import PackPredictor

    data = _data(2048, 2, 'cuda')
    val = _data(512, 3, 'cuda')
    t = _trainer((0, 6), 'muon')
    first = None
    for epoch in range(4):
        loss = t.fit_epoch(data, batch_size=128, epoch=epoch)
        first = loss if first is None else first
    res = t.evaluate_and_ensemble(val, epoch=3, train_loss=loss, max_ensemble_size=4)
    assert torch.all(loss < first)
    assert torch.isfinite(res.val_metric).all()
    assert 1 <= len(res.ensemble_idx) <= 4
    assert res.ensemble_score <= float(res.val_metric.min()) + 1e-6
    pred = PackPredictor(t, {'greedy': res.ensemble_idx})
    y_pack, heads = pred(val['x_num'], val['x_cat'])
    want = y_pack[res.ensemble_idx].mean(0)
    torch.testing.assert_close(heads['greedy'], want, rtol=1e-6, atol=1e-6)


def test_sharding_is_bit_invariant_with_cosine_embeddings():
    """Per-member embedding sizes and init scales from per-member configs (merged into the
    shared `numerical_embeddings` entry); sharded training equals the unsharded run."""
    from tabpack_b200.nn import CosineEmbeddingsPack
    from tabpack_b200.training import PackTrainer

    model = dict(MODEL, numerical_embeddings={'type': CosineEmbeddingsPack, 'max_d_embedding': 8})
    per = [dict(pm, numerical_embeddings={'d_embedding': d, 'init_scale': s})
           for pm, d, s in zip(PER_MEMBER, [4, 8, 2, 6, 3, 8], [0.1, 0.05, 0.2, 0.1, 0.3, 0.02])]

    def trainer(rng):
        return PackTrainer(n_members=6, model=model, per_member_model=per,
                           optimizer=dict(type='muon', adamw_lr=3e-3, weight_decay=1e-4, muon_lr=2e-2),
                           loss='mse', seed=5, device='cuda', autocast_bf16=True, member_range=rng)

    data = _data(512, 4, 'cuda')
    full, a, b = trainer((0, 6)), trainer((0, 2)), trainer((2, 6))
    first = None
    for epoch in range(2):
        for t in (full, a, b):
            loss = t.fit_epoch(data, batch_size=64, epoch=epoch)
            if t is full:
                first = loss if first is None else first
    sd = full.model.state_dict()
    for shard, lo in ((a, 0), (b, 2)):
        for k, v in shard.model.state_dict().items():
            if v.ndim == 0 or sd[k].shape[1:] != v.shape[1:]:
                continue
            assert torch.equal(v, sd[k][lo: lo + v.shape[0]]), k
    assert torch.isfinite(loss).all()
    assert full.model.num_module.elementwise_affine_weight.abs().sum() > 0  # the embeddings train


def test_member_chunked_prediction_equals_whole_pack():
    """predict_local in member groups (pack_idx selections, bounded activations for wide packs
    on large batches): every grouping gives the same predictions bit for bit, and they agree
    with the whole pack's (whose first layer gathers its one-hot columns) to the bf16
    tolerance; the predictor's ensemble head is the mean of the selected members."""
    from tabpack_b200.training import PackPredictor

    val = _data(300, 3, 'cuda')
    t = _trainer((0, 6), 'muon')
    t.fit_epoch(_data(256, 2, 'cuda'), batch_size=64, epoch=0)
    whole = t.predict_local(val)
    one = t.predict_local(val, member_chunk=1)
    assert torch.equal(t.predict_local(val, member_chunk=4), one)
    assert float((one - whole).abs().max()) < 2e-2 * float(whole.abs().max())
    pred = PackPredictor(t, {'h': torch.tensor([1, 4, 5])})
    y_pack, heads = pred(val['x_num'], val['x_cat'], member_chunk=4)
    assert torch.equal(y_pack, one)
    torch.testing.assert_close(heads['h'], one[[1, 4, 5]].mean(0), rtol=1e-6, atol=1e-6)


def _replace_trainer():
    from tabpack_b200.training import PackTrainer

    return PackTrainer(n_members=6, model=MODEL, per_member_model=REPLACE_MODELS,
                       optimizer=dict(type='muon', adamw_lr=3e-3, weight_decay=1e-4, muon_lr=2e-2),
                       per_member_optimizer=REPLACE_OPT, loss='mse', seed=99, device='cuda', n_models=9)


def test_replacement_gives_the_slot_a_fresh_model():
    """A slot taken over by a new model (`pack_replace`, `_training.py:860-924`): the model's
    shapes, dropout and learning rate, parameters keyed by model id (the same in any slot),
    zeroed optimizer state and the Muon update scale of the new shape; the other slots are
    untouched, and the layers' bf16 compute copies follow the new weights."""
    import math

    data, val = _data(640, 0, 'cuda'), _data(300, 1, 'cuda')
    a, b = _replace_trainer(), _replace_trainer()
    for t in (a, b):
        t.fit_epoch(data, batch_size=64, epoch=0)
    before = {n: p.detach().clone() for n, p in a.model.named_parameters()}
    pred_before = a.predict_local(val)
    a._replace_local([(2, 7)])
    b._replace_local([(4, 7)])
    hp = REPLACE_MODELS[7]
    bb = a.model.backbone
    assert int(bb.n_blocks[2]) == hp['n_blocks']
    assert all(int(blk.linear.out_features[2]) == hp['d_block'] for blk in bb.blocks)
    assert int(a.model.output.in_features[2]) == hp['d_block']
    assert all(abs(float(blk.dropout.p[2]) - hp['dropout']) < 1e-7 for blk in bb.blocks)
    params_b = dict(b.model.named_parameters())
    for n, p in a.model.named_parameters():
        keep = torch.ones(p.shape[0], dtype=torch.bool, device=p.device)
        keep[2] = False
        assert torch.equal(p[keep], before[n][keep]), n
        assert torch.equal(p[2], params_b[n][4]), n  # initialisation keyed by model id, not slot
    for g in a.opt.param_groups:
        if g['muon']:
            assert abs(float(g['muon_lr'][2]) / REPLACE_OPT[7]['muon_lr'] - 1) < 1e-6
            lin = next(blk.linear for blk in bb.blocks if blk.linear.weight is g['params'][0])
            o = int(lin.out_features[2])
            i = lin.max_in_features if lin.in_features is None else int(lin.in_features[2])
            assert abs(float(g['muon_update_scale'][2]) - math.sqrt(max(1.0, o / i))) < 1e-6
        for p in g['params']:
            for v in a.opt.state[p].values():
                if isinstance(v, torch.Tensor) and v.ndim > 0:
                    assert not v[2].any()
    pred = a.predict_local(val)
    assert torch.equal(pred[[0, 1, 3, 4, 5]], pred_before[[0, 1, 3, 4, 5]])
    assert not torch.equal(pred[2], pred_before[2])
    with torch.no_grad():  # every weight's version moves: the compute copies are cast again
        for p in a.model.parameters():
            p.add_(0.0)
    assert torch.equal(a.predict_local(val), pred)
    # the replaced slot trains on
    loss = a.fit_epoch(data, batch_size=64, epoch=1)
    assert torch.isfinite(loss).all()
