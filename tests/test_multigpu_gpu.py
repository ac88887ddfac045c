"""Two ranks over NCCL give exactly the single-process results (run when 2+ GPUs exist)."""

import json
import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.timeout(600)
def test_two_rank_training_matches_single_process(tmp_path):
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip('needs 2 GPUs')
    one = tmp_path / 'one.json'
    two = tmp_path / 'two.json'
    env = dict(os.environ, NCCL_NVLS_ENABLE='0', PYTHONPATH=ROOT)
    subprocess.run([sys.executable, os.path.join(ROOT, 'tests', 'mgpu_worker.py'), str(one)], check=True, env=env,
                   timeout=300)
    subprocess.run(['timeout', '-k', '30', '300', sys.executable, '-m', 'torch.distributed.run', '--nnodes=1',
                    '--nproc-per-node', '2', '--master-addr', '127.0.0.1', '--master-port', '29533',
                    os.path.join(ROOT, 'tests', 'mgpu_worker.py'), str(two)], check=True, env=env, timeout=360)
    a, b = json.loads(one.read_text()), json.loads(two.read_text())
    assert a['world'] == 1 and b['world'] == 2
    assert a['preds'] == b['preds']
    assert a['idx'] == b['idx']
    assert a['loss'] == b['loss']
    assert a['head'] == b['head']
