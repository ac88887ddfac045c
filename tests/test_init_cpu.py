"""Parameter initialisation against the reference (`LinearPack.reset_parameters`,
`src/tabpackage/nn.py:702-747`): U(-1/sqrt(in_i), 1/sqrt(in_i)) per member.

`LinearPack.reset_parameters` here draws from the global RNG in the reference's order, so
from the same seed it reproduces the reference's parameters bit for bit (`init.npz`, made by
`make_golden.py init`).  `init_member_parameters_` -- what the trainer uses, one generator per
(seed, global member id, layer) so that sharding does not change the initial weights -- has
the same per-member bounds; its tests check the bounds, that the draws fill them, and the
shard invariance.
"""

import numpy as np
import pytest
import torch

from tabpack_b200.nn import LinearPack, TabPack
from tabpack_b200.training import init_member_parameters_


def test_reset_parameters_matches_the_reference_bit_for_bit(golden):
    g = golden('init.npz')
    torch.manual_seed(12)
    lin = LinearPack([40, 16, 33], [48, 16, 20], max_in_features=40, max_out_features=48, pack_size=3)
    assert np.array_equal(lin.weight.detach().numpy(), g['ragged.weight'])
    assert np.array_equal(lin.bias.detach().numpy(), g['ragged.bias'])
    torch.manual_seed(13)
    lin.reset_parameters(pack_idx=torch.tensor([2, 0]))
    assert np.array_equal(lin.weight.detach().numpy(), g['ragged.reset.weight'])
    assert np.array_equal(lin.bias.detach().numpy(), g['ragged.reset.bias'])
    torch.manual_seed(14)
    shared = LinearPack(24, 12, pack_size=4)
    assert np.array_equal(shared.weight.detach().numpy(), g['shared.weight'])
    assert np.array_equal(shared.bias.detach().numpy(), g['shared.bias'])
    torch.manual_seed(15)
    shared.reset_parameters(pack_idx=torch.tensor([1]))
    assert np.array_equal(shared.weight.detach().numpy(), g['shared.reset.weight'])
    assert np.array_equal(shared.bias.detach().numpy(), g['shared.reset.bias'])


def _model(P=6):
    return TabPack(n_numerical_features=20, categorical_cardinalities=[5, 7], d_out=3, n_blocks=[1, 2, 3, 3, 2, 1][:P],
                   d_block=[64, 128, 256, 96, 32, 256][:P], dropout=[0.1] * P, pack_size=P, max_n_blocks=3,
                   max_d_block=256)


def _linears(model):
    return [m for m in model.modules() if isinstance(m, LinearPack)]


def test_init_member_parameters_per_member_bounds():
    model = _model()
    init_member_parameters_(model, seed=3, member_ids=list(range(6)), generator_device='cpu')
    for lin in _linears(model):
        inf = (lin.in_features.tolist() if lin.in_features is not None
               else [lin.max_in_features] * lin.pack_size)
        for m in range(lin.pack_size):
            bound = inf[m] ** -0.5
            for p in (lin.weight, lin.bias):
                v = p[m].detach().double().numpy()
                assert np.abs(v).max() <= bound * (1 + 1e-6)
                if v.size >= 256:
                    # uniform on the whole interval: both ends reached, mean near zero
                    assert v.max() > 0.95 * bound and v.min() < -0.95 * bound
                    assert abs(v.mean()) < 0.1 * bound


def test_init_member_parameters_is_shard_invariant():
    def uniform():  # members of one shape, so a member's bounds do not depend on its position
        return TabPack(n_numerical_features=20, categorical_cardinalities=[5, 7], d_out=3, n_blocks=[2] * 6,
                       d_block=[96] * 6, dropout=[0.1] * 6, pack_size=6, max_n_blocks=2, max_d_block=96)

    full = uniform()
    init_member_parameters_(full, seed=9, member_ids=list(range(6)), generator_device='cpu')
    part = uniform()
    init_member_parameters_(part, seed=9, member_ids=[3, 4, 0, 1, 2, 5], generator_device='cpu')
    for a, b in zip(_linears(full), _linears(part)):
        # member 0 of `part` has global id 3, and so on
        assert torch.equal(a.weight[3], b.weight[0]) and torch.equal(a.weight[4], b.weight[1])
        assert torch.equal(a.bias[5], b.bias[5])


@pytest.mark.parametrize('seed', [0, 1])
def test_init_member_parameters_differs_per_member_and_seed(seed):
    a = _model()
    init_member_parameters_(a, seed=seed, member_ids=list(range(6)), generator_device='cpu')
    b = _model()
    init_member_parameters_(b, seed=seed + 10, member_ids=list(range(6)), generator_device='cpu')
    la, lb = _linears(a)[1], _linears(b)[1]
    assert not torch.equal(la.weight[2], la.weight[3])
    assert not torch.equal(la.weight[2], lb.weight[2])
