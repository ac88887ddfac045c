"""torchrun worker for tests/test_multigpu_gpu.py: trains a member-sharded pack over NCCL
and writes rank 0's gathered results (validation predictions, ensemble, predictor heads)."""

import json
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from tests.test_training_gpu import MODEL, PER_MEMBER, _data  # noqa: E402
from tabpack_b200.shard import gather_members  # noqa: E402
from tabpack_b200.training import PackPredictor, PackTrainer  # noqa: E402


def run(out_path: str) -> None:
    local = int(os.environ.get('LOCAL_RANK', '0'))
    torch.cuda.set_device(local)
    dev = torch.device('cuda', local)
    world = int(os.environ.get('WORLD_SIZE', '1'))
    if world > 1:
        import datetime

        dist.init_process_group('nccl', device_id=dev, timeout=datetime.timedelta(seconds=120))
    optim = dict(type='muon', adamw_lr=3e-3, weight_decay=1e-4, muon_lr=2e-2)
    t = PackTrainer(n_members=6, model=MODEL, per_member_model=PER_MEMBER, optimizer=optim, loss='mse', seed=99,
                    device=dev, autocast_bf16=True, member_range=None if world > 1 else (0, 6))
    data, val = _data(640, 0, dev), _data(300, 1, dev)
    for epoch in range(2):
        loss = t.fit_epoch(data, batch_size=64, epoch=epoch)
    res = t.evaluate_and_ensemble(val, epoch=1, train_loss=loss, max_ensemble_size=4)
    local_pred = t.predict_local(val)
    preds = gather_members(local_pred, t.counts, t.group) if t.world > 1 else local_pred
    y_pack, heads = PackPredictor(t, {'greedy': res.ensemble_idx})(val['x_num'], val['x_cat'])
    if t.rank == 0:
        with open(out_path, 'w') as f:
            json.dump({'world': t.world, 'preds': preds.double().cpu().tolist(), 'idx': res.ensemble_idx.tolist(),
                       'head': heads['greedy'].double().cpu().tolist(), 'loss': loss.double().cpu().tolist()}, f)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == '__main__':
    run(sys.argv[1])
