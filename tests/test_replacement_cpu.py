"""The model-replacement queue of `PackTrainer.fit` (`src/tabpackage/_training.py:2891-2927`),
on CPU: the bookkeeping of `fit` runs against a stand-in trainer whose validation metric of
model m after e epochs is scripted, so which model trains in which slot, when each model
stops, its best checkpoint and the predictions handed to the ensemble are all known in
advance.  The two-rank case (gloo) checks that both ranks take the same decisions as one
process and that each rank only touches its own slots."""

import math
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from tabpack_b200.shard import assign_replacements, gather_members, member_ranges
from tabpack_b200.training import PackTrainer


def test_assign_replacements_order_and_count():
    assert assign_replacements([5, 1, 3], next_model_id=10, n_pending=2) == [(1, 10), (3, 11)]
    assert assign_replacements([2], next_model_id=7, n_pending=0) == []
    assert assign_replacements([], next_model_id=7, n_pending=4) == []
    assert assign_replacements([4, 0], next_model_id=3, n_pending=9) == [(0, 3), (4, 4)]
    with pytest.raises(ValueError):
        assign_replacements([1, 1], next_model_id=0, n_pending=1)
    with pytest.raises(ValueError):
        assign_replacements([1], next_model_id=0, n_pending=-1)


def _metric(m: int, e: int) -> float:
    """Scripted validation metric (lower is better) of model m after e epochs."""
    table = {
        0: [1.0, 2.0, 3.0, 4.0],          # best at its first evaluation, then worse
        1: [math.nan, 0.5, 0.4, 0.45],    # NaN first: still its first best checkpoint
    }
    if m in table:
        return table[m][min(e, len(table[m])) - 1]
    return 1.0 / (m + e)                  # improves every epoch


class _Trainer:
    """What `PackTrainer.fit` uses of a trainer, with scripted predictions: each slot
    predicts (metric of its model, 1000 * model id + model epoch)."""
    fit = PackTrainer.fit

    def __init__(self, n_slots: int, n_models: int, lo: int, hi: int, group=None):
        self.n_models = n_models
        self.slot_model = list(range(n_slots))
        self.gathered_ids = list(range(n_slots))
        self.lo, self.hi = lo, hi
        self.group = group
        self.counts = [b - a for a, b in member_ranges(n_slots, dist.get_world_size(group))] if group else None
        self.model_epochs = [0] * n_models
        self.calls = []

    def fit_epoch(self, data, *, batch_size, epoch):
        for m in self.slot_model:
            if m >= 0:
                self.model_epochs[m] += 1
        return torch.zeros(len(self.slot_model))

    def predict(self, data, *, eval_batch_size):
        rows = []
        for g in range(self.lo, self.hi):
            m = self.slot_model[g]
            e = self.model_epochs[m] if m >= 0 else 0
            rows.append([_metric(m, e) if m >= 0 else 0.0, 1000.0 * m + e])
        local = torch.tensor(rows, dtype=torch.float64)
        return gather_members(local, self.counts, self.group) if self.group is not None else local

    def _score(self, y):
        return lambda preds: -preds[:, 0]

    def _freeze(self, local_idx):
        self.calls.append(('freeze', sorted(local_idx)))

    def _replace_local(self, pairs):
        self.calls.append(('replace', list(pairs)))


class _Ensemble:
    """Records the candidates and checks that each handed-over prediction belongs to the
    checkpoint key it was asked for (model id, model step; one step per epoch here)."""

    def __init__(self):
        self.member_keys = None
        self.member_weights = None
        self.best_score = None
        self.updates = []

    def is_running(self):
        return True

    def update(self, predictions, finished, running_latest):
        for m, step in list(finished) + list(running_latest):
            assert predictions((m, step))[1].item() == 1000.0 * m + step
        self.updates.append((list(finished), list(running_latest)))
        self.member_keys = list(finished[:1]) + list(running_latest[:1])
        self.best_score = 0.0
        return True


def _run(tr: _Trainer, ens: _Ensemble):
    data = {'y': torch.zeros(8)}
    return tr.fit(data, data, batch_size=8, max_epochs=[4, 3, 3, 1, 2, 1], early_stopping_patience=1,
                  ensemble=ens)


# slot_model per epoch, and the finished keys, derived by hand from `_metric` and max_epochs:
#   epoch 1: slots train models 0 1 2; model 1's first evaluation is NaN (its first best checkpoint)
#   epoch 2: model 0 worsens (1 bad update, patience 1 keeps it); nothing stops
#   epoch 3: model 0 worsens again (2 > patience) and stops with best step 1; model 1 (max 3)
#            and model 2 (max 3) stop at step 3; 3 pending models remain -> slots 0 1 2 take 3 4 5
#   epoch 4: models 3 (max 1) and 5 (max 1) stop; nothing pending -> slots 0 and 2 freeze
#   epoch 5: model 4 (max 2) stops; slot 1 freezes
EXPECTED_SLOTS = [[0, 1, 2], [0, 1, 2], [0, 1, 2], [3, 4, 5], [-1, 4, -1]]
EXPECTED_FINISHED = [(0, 1), (1, 3), (2, 3), (3, 1), (5, 1), (4, 2)]


def test_fit_replacement_bookkeeping_one_process():
    tr, ens = _Trainer(3, 6, 0, 3), _Ensemble()
    res = _run(tr, ens)
    assert [h['slot_model'] for h in res.history] == EXPECTED_SLOTS
    assert ens.updates[-1][0] == EXPECTED_FINISHED
    assert res.best_step.tolist() == [1, 3, 3, 1, 2, 1]
    assert res.best_metric[0].item() == 1.0 and res.best_metric[1].item() == 0.4
    assert tr.calls == [('freeze', []), ('replace', []), ('freeze', []), ('replace', []),
                        ('freeze', []), ('replace', [(0, 3), (1, 4), (2, 5)]),
                        ('freeze', [0, 2]), ('replace', []), ('freeze', [1]), ('replace', [])]
    assert tr.slot_model == [-1, -1, -1]
    # per-model history: NaN for the models not trained in an epoch
    v = torch.stack([h['val_metric'] for h in res.history])
    assert math.isnan(v[0, 1]) and math.isnan(v[0, 3]) and v[3, 3].item() == _metric(3, 1)
    assert math.isnan(v[4, 3]) and v[4, 4].item() == _metric(4, 2)


def _free_port():
    s = socket.socket()
    s.bind(('127.0.0.1', 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    os.environ['MASTER_ADDR'] = '127.0.0.1'
    os.environ['MASTER_PORT'] = str(port)
    dist.init_process_group('gloo', rank=rank, world_size=world)
    try:
        lo, hi = member_ranges(3, world)[rank]
        tr, ens = _Trainer(3, 6, lo, hi, group=dist.group.WORLD), _Ensemble()
        res = _run(tr, ens)
        q.put((rank, lo, [h['slot_model'] for h in res.history], ens.updates, res.best_step.tolist(), tr.calls))
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(120)
def test_fit_replacement_gloo_world2_matches_one_process():
    ctx = mp.get_context('spawn')
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=90) for _ in range(2))
    for p in procs:
        p.join(timeout=30)
        assert p.exitcode == 0
    one = _Trainer(3, 6, 0, 3)
    one_ens = _Ensemble()
    ref = _run(one, one_ens)
    replaced = [pairs for kind, pairs in one.calls if kind == 'replace' and pairs]
    for rank, lo, slots, updates, best_step, calls in res:
        assert slots == EXPECTED_SLOTS
        assert updates == one_ens.updates
        assert best_step == ref.best_step.tolist()
        # each rank re-initialises only its own slots, in local indices
        mine = [[(g - lo, m) for g, m in pairs if lo <= g < lo + (2 if rank == 0 else 1)] for pairs in replaced]
        got = [pairs for kind, pairs in calls if kind == 'replace' and pairs]
        assert got == [p for p in mine if p]
