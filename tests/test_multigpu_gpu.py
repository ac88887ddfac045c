"""Two ranks give exactly the single-process results: over NCCL on two GPUs (run when 2+
GPUs exist), and over gloo with both ranks on one GPU (the same sharded code path with the
collectives staged through host memory), for plain epochs and for `fit` with the model
replacement queue."""

import json
import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
WORKER = os.path.join(ROOT, 'tests', 'mgpu_worker.py')


def _run_pair(tmp_path, mode: str, backend: str, port: int):
    one = tmp_path / f'one_{mode}.json'
    two = tmp_path / f'two_{mode}.json'
    env = dict(os.environ, NCCL_NVLS_ENABLE='0', PYTHONPATH=ROOT, TP_TEST_BACKEND=backend)
    subprocess.run([sys.executable, WORKER, str(one), mode], check=True, env=env, timeout=300)
    subprocess.run(['timeout', '-k', '30', '300', sys.executable, '-m', 'torch.distributed.run', '--nnodes=1',
                    '--nproc-per-node', '2', '--master-addr', '127.0.0.1', '--master-port', str(port),
                    WORKER, str(two), mode], check=True, env=env, timeout=360)
    a, b = json.loads(one.read_text()), json.loads(two.read_text())
    assert a['world'] == 1 and b['world'] == 2
    return a, b


def _check_epochs(a, b):
    assert a['preds'] == b['preds']
    assert a['idx'] == b['idx']
    assert a['loss'] == b['loss']
    assert a['head'] == b['head']


def _check_replace(a, b):
    from tests.test_training_gpu import REPLACE_MAX_EPOCHS

    for k in ('slots', 'val_metric', 'best_metric', 'best_step', 'ensemble_keys', 'ensemble_metric',
              'ensemble_history', 'preds'):
        assert a[k] == b[k], k
    # every model trained in some slot for its max_epochs (no early stopping here) and finished
    trained = {m: 0 for m in range(len(REPLACE_MAX_EPOCHS))}
    for slots in a['slots']:
        for m in slots:
            if m >= 0:
                trained[m] += 1
    assert [trained[m] for m in sorted(trained)] == REPLACE_MAX_EPOCHS
    assert a['slots'][0] == [0, 1, 2, 3, 4, 5]


@pytest.mark.timeout(600)
def test_two_rank_training_matches_single_process(tmp_path):
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip('needs 2 GPUs')
    _check_epochs(*_run_pair(tmp_path, 'epochs', 'nccl', 29533))


@pytest.mark.timeout(600)
def test_two_ranks_on_one_gpu_match_single_process(tmp_path):
    _check_epochs(*_run_pair(tmp_path, 'epochs', 'gloo', 29534))


@pytest.mark.timeout(600)
def test_replacement_queue_two_ranks_match_single_process(tmp_path):
    _check_replace(*_run_pair(tmp_path, 'replace', 'gloo', 29535))
