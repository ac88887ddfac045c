"""Seeded synthetic data and hyperparameters of the 16-member CPU plumbing run.

Test infrastructure: used by `make_golden.py` (to run the reference's `train` on CPU)
and by the GPU test that trains the same pack here, so both see the same numbers.

Data (regression): 20 000 train / 5 000 validation rows; 32 numerical features
~N(0, 1); 4 categorical features of cardinality 10, uniform; y = a random two-layer
ReLU teacher MLP (width 64) of [x_num, one-hot(x_cat)] plus N(0, 0.1^2) noise.
Pack: 16 members, depth U{1, 2, 3}, width U{64, 128, 256}, dropout U[0, 0.3],
AdamW learning rate log-U[1e-4, 3e-3]; batch 256.
"""

from __future__ import annotations

import numpy as np

N_TRAIN, N_VAL, N_NUM, CARDS = 20_000, 5_000, 32, [10, 10, 10, 10]
N_MEMBERS, BATCH, WEIGHT_DECAY = 16, 256, 1e-4


def datasets(seed: int = 0) -> dict[str, dict[str, np.ndarray]]:
    rng = np.random.default_rng(seed)
    n = N_TRAIN + N_VAL
    x_num = rng.standard_normal((n, N_NUM)).astype(np.float32)
    x_cat = np.stack([rng.integers(0, c, n) for c in CARDS], 1).astype(np.int64)
    onehot = np.concatenate([np.eye(c, dtype=np.float32)[x_cat[:, i]] for i, c in enumerate(CARDS)], 1)
    feats = np.concatenate([x_num, onehot], 1).astype(np.float64)
    w1 = rng.standard_normal((feats.shape[1], 64)) / np.sqrt(feats.shape[1])
    w2 = rng.standard_normal(64) / np.sqrt(64)
    y = (np.maximum(feats @ w1, 0.0) @ w2 + 0.1 * rng.standard_normal(n)).astype(np.float32)
    split = {'train': slice(0, N_TRAIN), 'val': slice(N_TRAIN, n)}
    return {k: {'x_num': x_num[s], 'x_cat': x_cat[s], 'y': y[s]} for k, s in split.items()}


def hyperparameters(seed: int = 1) -> list[dict]:
    """Per-member hyperparameters in the reference's `per_model_hyperparameters` layout."""
    rng = np.random.default_rng(seed)
    out = []
    for _ in range(N_MEMBERS):
        out.append({
            'model': {'n_blocks': int(rng.integers(1, 4)), 'd_block': int(rng.choice([64, 128, 256])),
                      'dropout': float(rng.uniform(0.0, 0.3))},
            'optimizer': {'lr': float(np.exp(rng.uniform(np.log(1e-4), np.log(3e-3))))},
        })
    return out
