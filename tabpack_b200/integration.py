"""Optimizer packs that pass as the reference's own, for `tabpackage.train`.

`tabpackage.train` builds its optimizer with `make_optimizer_pack`
(`src/tabpackage/_training.py:228-320`), which decides by `issubclass` against the
reference's classes: only a subclass of `tabpackage.optim.MuonAdamWPack` gets one Muon
parameter group per backbone block (`_training.py:246-258`), and only a subclass of
`tabpackage.optim.OptimizerPack` receives `pack_size` / `support_replacement`
(`_training.py:300-318`) and can replace members (`_training.py:2920-2927`).  The classes
made here derive from the reference's `AdamWPack` / `MuonAdamWPack`, so they pass those
checks and keep the reference's constructor, hyperparameter validation, parameter groups,
state keys and `replace`; only `step` changes: AdamW groups go through the grouped AdamW
kernel and each Muon group through the Muon kernels (batched Newton-Schulz on the tensor
cores).  `make_muon_parameter_group` also records each member's real output and input width,
so Newton-Schulz runs on each member's own block instead of the padded one.

    from tabpack_b200.integration import reference_optimizer_packs
    AdamW, Muon = reference_optimizer_packs()
    tabpackage.train(..., optimizer={'type': Muon, 'adamw_lr': ..., 'muon_lr': ..., ...})

`install()` routes the reference's own module packs through the fused kernels: the forward
of `tabpackage.nn.MLPBackbonePack.Block` (`nn.py:1071-1079`: linear, ReLU and dropout as one
launch) and of `tabpackage.nn.LinearPack` (`nn.py:792-816`, e.g. the output head).  The
replacements read only what the reference's modules hold (weights, biases, width buffers,
dropout probabilities, the activation module); each linear pack gets its bf16 weight cache as
an extra attribute.  Dropout then uses the Philox keep mask with a key drawn from the global
torch RNG per call, in place of `bernoulli_` on the same RNG.  Blocks with another activation,
or a training-mode call on a member subset (`pack_idx`), keep the reference's forward.

The module imports `tabpackage` only when one of these functions is called.
"""

from __future__ import annotations

import functools

import torch

from tabpack_b200.nn import _linear_call, _WeightCache
from tabpack_b200.optim import adamw_step, muon_adamw_step


def _widths(module):
    """(out_features, in_features) of a reference `LinearPack` as int32 tensors, or None where
    every member has the padded width."""
    outf = getattr(module, 'out_features', None)
    inf = getattr(module, 'in_features', None)
    return (None if outf is None else outf.to(torch.int32),
            None if inf is None else inf.to(torch.int32))


@functools.cache
def reference_optimizer_packs() -> tuple[type, type]:
    """(AdamWPack, MuonAdamWPack): subclasses of `tabpackage.optim.AdamWPack` and
    `tabpackage.optim.MuonAdamWPack` whose `step` runs on this package's kernels.  Raises
    ImportError when `tabpackage` cannot be imported."""
    try:
        import tabpackage.nn as ref_nn
        import tabpackage.optim as ref
    except ImportError as err:  # pragma: no cover - depends on the environment
        raise ImportError('reference_optimizer_packs needs the reference package `tabpackage` on the path') from err

    class AdamWPack(ref.AdamWPack):
        """`tabpackage.optim.AdamWPack` (`optim.py:269-427`) stepping on the grouped AdamW kernel."""

        @torch.no_grad()
        def step(self, closure=None):
            loss = closure() if closure is not None else None
            adamw_step(self, support_replacement=self._support_replacement)
            return loss

    class MuonAdamWPack(ref.MuonAdamWPack):
        """`tabpackage.optim.MuonAdamWPack` (`optim.py:495-861`) stepping on the Muon and
        grouped AdamW kernels."""

        @staticmethod
        def make_muon_parameter_group(module):
            group = ref.MuonAdamWPack.make_muon_parameter_group(module)
            group['muon_out_features'], group['muon_in_features'] = _widths(module)
            return group

        def replace(self, *, pack_idx, module, **kw):
            super().replace(pack_idx=pack_idx, module=module, **kw)
            # the replaced members' widths, as the reference recomputes their update scales
            by_weight = {m.weight: m for m in module.modules() if isinstance(m, ref_nn.LinearPack)}
            for g in self.param_groups:
                if g['muon']:
                    g['muon_out_features'], g['muon_in_features'] = _widths(by_weight[g['params'][0]])

        @torch.no_grad()
        def step(self, closure=None):
            loss = closure() if closure is not None else None
            if not hasattr(self, '_b200_workspaces'):
                self._b200_workspaces = {}
            muon_adamw_step(self, workspaces=self._b200_workspaces,
                            allow_inplace_grad_mutation=self._allow_inplace_grad_mutation,
                            support_replacement=self._support_replacement)
            return loss

    AdamWPack.__module__ = MuonAdamWPack.__module__ = __name__
    return AdamWPack, MuonAdamWPack


class _CallKey:
    """Philox key of one training-mode call, drawn from the global torch RNG (where the
    reference's dropout draws its Bernoulli samples), counter offset 0."""

    def __init__(self) -> None:
        self.seed = int(torch.randint(0, 2**62, (1,)).item())
        self.member_base = 0

    def next_offset(self, stride: int = 1) -> int:
        return 0


def _fused_linear(linear, x, pack_idx, *, relu: bool, dropout):
    if '_cache' not in linear.__dict__:
        linear._cache = _WeightCache()
    return _linear_call(linear, x, pack_idx, relu=relu, dropout=dropout, stream=None if dropout is None else _CallKey(),
                        n_blocks=None, block_index=0)


def install():
    """Route `tabpackage.nn.MLPBackbonePack.Block.forward` and `tabpackage.nn.LinearPack.forward`
    through the fused kernels (CUDA tensors only); returns a function that restores the
    reference's forwards."""
    import tabpackage.nn as ref_nn

    Block, LinearPack, TabPack = ref_nn.MLPBackbonePack.Block, ref_nn.LinearPack, ref_nn.TabPack
    orig = (Block.forward, LinearPack.forward, TabPack.__init__)

    def block_forward(self, x, pack_idx=None):
        act = self.activation
        relu = isinstance(act, torch.nn.ReLU)
        p = self.dropout.p
        dropout = None
        if self.training and not (isinstance(p, (int, float)) and p == 0.0):
            dropout = (torch.full((self.linear.weight.shape[0],), float(p), device=x.device)
                       if isinstance(p, (int, float)) else p.to(x.device, torch.float32).contiguous())
        if not x.is_cuda or not (relu or isinstance(act, torch.nn.Identity)) or (
                dropout is not None and pack_idx is not None):
            return orig[0](self, x, pack_idx)
        return _fused_linear(self.linear, x, pack_idx, relu=relu, dropout=dropout)

    def linear_forward(self, x, pack_idx=None):
        if not x.is_cuda:
            return orig[1](self, x, pack_idx)
        return _fused_linear(self, x, pack_idx, relu=False, dropout=None)

    def tabpack_init(self, *args, **kwargs):
        orig[2](self, *args, **kwargs)
        # with numerical embeddings the first layer's valid input columns are not a prefix
        # (the reference multiplies its whole padded input width, `nn.py:792-816`)
        self.backbone.blocks[0].linear.full_width_input = self.num_module is not None

    Block.forward, LinearPack.forward, TabPack.__init__ = block_forward, linear_forward, tabpack_init

    def undo() -> None:
        Block.forward, LinearPack.forward, TabPack.__init__ = orig

    return undo


__all__ = ['reference_optimizer_packs', 'install']
