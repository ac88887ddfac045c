"""The drop-in boundary inside the reference's own training code (no GPU needed).

`tabpackage.train` builds its optimizer with `make_optimizer_pack`
(`src/tabpackage/_training.py:228-320`); these tests build optimizers through that function
with the classes of `tabpack_b200.integration.reference_optimizer_packs` and check that they
receive exactly the reference's parameter groups (one Muon group per backbone block, the
no-weight-decay group, the rest), `pack_size` / `support_replacement`, and member
replacement; and that `install()` swaps the module forwards in and out.  They need the
reference package: set TABPACK_REFERENCE_SRC to its `src` directory (skipped otherwise).
"""

import pytest
import torch


def _model(tp):
    torch.manual_seed(0)
    return tp.nn.TabPack(n_numerical_features=6, categorical_cardinalities=[3, 4], d_out=1, n_blocks=[1, 3, 2],
                         d_block=[16, 32, 24], dropout=[0.1, 0.0, 0.2], pack_size=3, max_n_blocks=3, max_d_block=32)


def _group_signature(opt):
    return [(tuple(id(p) for p in g['params']), bool(g.get('muon', False)),
             float(g['weight_decay']) if not isinstance(g['weight_decay'], torch.Tensor) else None)
            for g in opt.param_groups]


def test_muon_shim_gets_the_reference_groups(reference):
    tp = reference
    from tabpack_b200.integration import reference_optimizer_packs

    _, Muon = reference_optimizer_packs()
    assert issubclass(Muon, tp.optim.MuonAdamWPack) and issubclass(Muon, tp.optim.OptimizerPack)
    model = _model(tp)
    kw = dict(adamw_lr=1e-3, muon_lr=2e-2, weight_decay=1e-5)
    ours = tp._training.make_optimizer_pack(model, type=Muon, support_replacement=True, **kw)
    ref = tp._training.make_optimizer_pack(model, type=tp.optim.MuonAdamWPack, support_replacement=True, **kw)
    assert isinstance(ours, tp.optim.MuonAdamWPack)
    assert _group_signature(ours) == _group_signature(ref)
    muon = [g for g in ours.param_groups if g['muon']]
    assert len(muon) == len(model.backbone.blocks)
    for g, block in zip(muon, model.backbone.blocks):
        assert g['params'][0] is block.linear.weight
        assert torch.equal(g['muon_update_scale'], tp.optim.compute_muon_update_scale_pack(block.linear))
        assert g['muon_out_features'].dtype == torch.int32
        assert torch.equal(g['muon_out_features'], block.linear.out_features.to(torch.int32))
        want_in = block.linear.in_features
        assert (g['muon_in_features'] is None) == (want_in is None)
        if want_in is not None:
            assert torch.equal(g['muon_in_features'], want_in.to(torch.int32))
    assert ours._support_replacement


def test_adamw_shim_gets_the_reference_groups(reference):
    tp = reference
    from tabpack_b200.integration import reference_optimizer_packs

    AdamW, _ = reference_optimizer_packs()
    assert issubclass(AdamW, tp.optim.AdamWPack)
    model = _model(tp)
    ours = tp._training.make_optimizer_pack(model, type=AdamW, support_replacement=True, lr=[1e-3, 2e-3, 3e-3],
                                            weight_decay=1e-4)
    ref = tp._training.make_optimizer_pack(model, type=tp.optim.AdamWPack, support_replacement=True,
                                           lr=[1e-3, 2e-3, 3e-3], weight_decay=1e-4)
    assert _group_signature(ours) == _group_signature(ref)
    assert torch.equal(ours.param_groups[0]['lr'], ref.param_groups[0]['lr'])


def test_muon_shim_replace_updates_widths(reference):
    tp = reference
    from tabpack_b200.integration import reference_optimizer_packs

    _, Muon = reference_optimizer_packs()
    model = _model(tp)
    # replaceable hyperparameters are per-member lists (`optim.py:216-237`)
    opt = tp._training.make_optimizer_pack(model, type=Muon, support_replacement=True, adamw_lr=1e-3,
                                           muon_lr=[2e-2] * 3, weight_decay=1e-5)
    idx = torch.tensor([1])
    model.replace(pack_idx=idx, n_blocks=[1], d_block=[8], dropout=[0.3])
    opt.replace(pack_idx=idx, muon_lr=[5e-3], module=model)
    g0 = next(g for g in opt.param_groups if g['muon'])
    assert int(g0['muon_out_features'][1]) == 8
    assert float(g0['muon_lr'][1]) == pytest.approx(5e-3)


def test_install_and_undo_swap_the_forwards(reference):
    tp = reference
    from tabpack_b200.integration import install

    Block, Linear = tp.nn.MLPBackbonePack.Block, tp.nn.LinearPack
    before = (Block.forward, Linear.forward, tp.nn.TabPack.__init__)
    undo = install()
    try:
        assert Block.forward is not before[0] and Linear.forward is not before[1]
        # CPU tensors keep the reference's arithmetic
        model = _model(tp).eval()
        x_num, x_cat = torch.randn(5, 6), torch.randint(0, 3, (5, 2))
        y = model(x_num, x_cat)
    finally:
        undo()
    assert (Block.forward, Linear.forward, tp.nn.TabPack.__init__) == before
    assert torch.equal(y, _model(tp).eval()(x_num, x_cat))
