"""torchrun worker for tests/test_multigpu_gpu.py: trains a member-sharded pack and writes
rank 0's gathered results.

Modes (argv[2]): 'epochs' (two epochs, then validation predictions, ensemble, predictor
heads) and 'replace' (`PackTrainer.fit` with more models than pack slots: the replacement
queue).  The process group is NCCL with one GPU per rank, or, with TP_TEST_BACKEND=gloo,
gloo with every rank on GPU 0 (collectives staged through host memory; the ranks' kernels
never wait on one another)."""

import datetime
import json
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from tests.test_training_gpu import (MODEL, PER_MEMBER, REPLACE_MAX_EPOCHS, REPLACE_MODELS, REPLACE_OPT,  # noqa: E402
                                     _data)
from tabpack_b200.shard import gather_members  # noqa: E402
from tabpack_b200.training import PackPredictor, PackTrainer  # noqa: E402


def _trainer(world, dev, n_models=None):
    optim = dict(type='muon', adamw_lr=3e-3, weight_decay=1e-4, muon_lr=2e-2)
    if n_models is None:
        return PackTrainer(n_members=6, model=MODEL, per_member_model=PER_MEMBER, optimizer=optim, loss='mse',
                           seed=99, device=dev, autocast_bf16=True, member_range=None if world > 1 else (0, 6))
    return PackTrainer(n_members=6, model=MODEL, per_member_model=REPLACE_MODELS, optimizer=optim,
                       per_member_optimizer=REPLACE_OPT, loss='mse', seed=99, device=dev, autocast_bf16=True,
                       member_range=None if world > 1 else (0, 6), n_models=n_models)


def _epochs(t, dev):
    data, val = _data(640, 0, dev), _data(300, 1, dev)
    for epoch in range(2):
        loss = t.fit_epoch(data, batch_size=64, epoch=epoch)
    res = t.evaluate_and_ensemble(val, epoch=1, train_loss=loss, max_ensemble_size=4)
    local_pred = t.predict_local(val)
    preds = gather_members(local_pred, t.counts, t.group) if t.world > 1 else local_pred
    y_pack, heads = PackPredictor(t, {'greedy': res.ensemble_idx})(val['x_num'], val['x_cat'])
    return {'world': t.world, 'preds': preds.double().cpu().tolist(), 'idx': res.ensemble_idx.tolist(),
            'head': heads['greedy'].double().cpu().tolist(), 'loss': loss.double().cpu().tolist()}


def _replace(t, dev):
    data, val = _data(640, 0, dev), _data(300, 1, dev)
    res = t.fit(data, val, batch_size=64, max_epochs=REPLACE_MAX_EPOCHS)
    preds = t.predict(val)

    def nan_none(v):
        return [None if x != x else x for x in v]

    return {'world': t.world, 'slots': [h['slot_model'] for h in res.history],
            'val_metric': [nan_none(h['val_metric'].tolist()) for h in res.history],
            'best_metric': res.best_metric.tolist(), 'best_step': res.best_step.tolist(),
            'ensemble_keys': [list(k) for k in res.ensemble_keys], 'ensemble_metric': res.ensemble_metric,
            'ensemble_history': [[h['step'], [list(k) for k in h['keys']], h['metric']] for h in res.ensemble_history],
            'preds': preds.double().cpu().tolist()}


def run(out_path: str, mode: str) -> None:
    world = int(os.environ.get('WORLD_SIZE', '1'))
    backend = os.environ.get('TP_TEST_BACKEND', 'nccl')
    local = 0 if backend == 'gloo' else int(os.environ.get('LOCAL_RANK', '0'))
    torch.cuda.set_device(local)
    dev = torch.device('cuda', local)
    if world > 1:
        kw = {'device_id': dev} if backend == 'nccl' else {}
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=120), **kw)
    t = _trainer(world, dev, n_models=len(REPLACE_MODELS) if mode == 'replace' else None)
    out = _replace(t, dev) if mode == 'replace' else _epochs(t, dev)
    if t.rank == 0:
        with open(out_path, 'w') as f:
            json.dump(out, f)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == '__main__':
    run(sys.argv[1], sys.argv[2] if len(sys.argv) > 2 else 'epochs')
