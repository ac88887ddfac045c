"""The reference's own training loop on this package's kernels (`tabpack_b200.integration`).

`install()` routes the reference's `MLPBackbonePack.Block` and `LinearPack` forwards through
the fused kernels and `reference_optimizer_packs()` gives optimizer packs that
`make_optimizer_pack` accepts as the reference's own; with both, `tabpackage.train` runs
unchanged.  Checked here: the reference's `TabPack` forward on the kernels against its own
PyTorch forward on the same GPU (fp32, 1e-4), and two epochs of `tabpackage.train` with
Muon + AdamW under bf16 autocast ending with finite member and ensemble metrics that beat
predicting the mean.  These tests need the reference package importable (set
TABPACK_REFERENCE_SRC to its `src` directory) and are skipped where it is not.
"""

import functools

import numpy as np
import pytest
import torch

from tests.golden import synthetic

pytestmark = pytest.mark.gpu


def test_reference_tabpack_forward_on_the_kernels(reference):
    tp = reference
    from tabpack_b200.integration import install

    torch.manual_seed(0)
    model = tp.nn.TabPack(n_numerical_features=6, categorical_cardinalities=[3, 4], d_out=2, n_blocks=[1, 3, 2],
                          d_block=[16, 32, 24], dropout=[0.1, 0.0, 0.2], pack_size=3, max_n_blocks=3,
                          max_d_block=32).cuda().eval()
    x_num, x_cat = torch.randn(64, 6, device='cuda'), torch.randint(0, 4, (64, 2), device='cuda')
    with torch.no_grad():
        want = model(x_num, x_cat)
    undo = install()
    try:
        with torch.no_grad():
            got = model(x_num, x_cat)
    finally:
        undo()
    err = float((got - want).abs().max() / want.abs().max())
    assert err < 1e-4, err


def test_reference_train_with_kernels(reference):
    tp = reference
    from tabpack_b200.integration import install, reference_optimizer_packs

    _, Muon = reference_optimizer_packs()
    data = synthetic.datasets(0)
    dev = torch.device('cuda')
    sets = {'train': {k: torch.from_numpy(v[:4096]).to(dev) for k, v in data['train'].items()},
            'val': {k: torch.from_numpy(v[:1024]).to(dev) for k, v in data['val'].items()}}

    def loss_fn(y_pred, y):
        return ((y_pred.squeeze(-1) - y) ** 2).mean(1)

    def ensemble_mse(*, y_true, y_pred):
        return tp.metrics.mse_pack(y_true=y_true, y_pred=y_pred.unsqueeze(0))[0]

    crit = tp.EvalCriterionConfig(dataset='val', metric='mse', metric_direction='minimize')
    ens = tp.EnsembleConfig(algorithm={'type': tp.ensemble.greedy_ensemble, 'max_ensemble_size': 8}, online=True,
                            prediction_transform=None, early_stopping_patience=None,
                            algorithm_metric=tp.metrics.mse_pack, algorithm_metric_direction='minimize',
                            algorithm_dataset='val', algorithm_device=dev)
    hp = [{'model': {'n_blocks': n, 'd_block': d, 'dropout': p}}
          for n, d, p in [(1, 64, 0.1), (2, 128, 0.0), (3, 96, 0.2), (2, 256, 0.1)]]
    undo = install()
    try:
        res = tp.train(
            datasets=sets, model={'d_out': 1, 'categorical_cardinalities': synthetic.CARDS},
            prediction_transform=functools.partial(torch.squeeze, dim=-1), loss_fn=loss_fn,
            optimizer={'type': Muon, 'adamw_lr': 1e-3, 'muon_lr': 2e-2, 'weight_decay': 1e-5},
            batch_size=256, max_epochs=2, early_stopping_patience=None, per_model_hyperparameters=hp,
            eval_metrics={'val': {'mse': tp.metrics.mse_pack}}, eval_criterion=crit, ensembles={'greedy': ens},
            ensemble_eval_metrics={'val': {'mse': ensemble_mse}}, ensemble_eval_criterion=crit,
            stop_when_all_ensembles_are_finalized=False, seed=0, device=dev, aux_device=dev,
            autocast_dtype=torch.bfloat16, print_progress=False, show_progress_bar=False)
    finally:
        undo()
    ids = torch.arange(len(hp))
    member = res.load_model_metrics(ids)['val']['mse'].float().cpu().numpy()
    ensemble = float(res.load_ensemble_metrics('greedy')['val']['mse'])
    baseline = float(sets['val']['y'].float().var(unbiased=False))
    assert np.isfinite(member).all() and np.isfinite(ensemble)
    assert member.max() < baseline and ensemble < baseline
