"""Optimizer packs whose step runs on the sm_100a kernels.

Drop-in counterparts of `tabpackage.optim` (`src/tabpackage/optim.py`): the same
constructors, group values (scalars or per-member `(P,)` tensors), state keys
(`step`, `exp_avg`, `exp_avg_sq`, `muon_momentum_buffer`) and member replacement.
A group's AdamW update is one grouped launch over all its parameter packs; a Muon
group runs momentum + packing, batched Newton-Schulz on tcgen05 tensor cores (each
member on its own out x in block) and the scaled update, with members whose update
is all zero skipped on the device instead of through a host synchronisation.
"""

from __future__ import annotations

import math
from typing import Any, Final

import torch
from torch import Tensor

from tabpack_b200 import ops
from tabpack_b200.nn import (PACK_DIM, LinearPack, ParameterPack, bf16_copy_cache, check_pack_idx,
                             make_complementary_pack_idx)


def _check_lr(v):
    if not math.isfinite(v) or v < 0.0:
        raise ValueError('The learning rate must be finite and non-negative')


def _check_momentum(v):
    if not math.isfinite(v) or v < 0.0 or v >= 1.0:
        raise ValueError('Momentum and moving-average decay coefficients must be finite and in the range [0, 1)')


def _check_weight_decay(v):
    if not math.isfinite(v) or v < 0.0:
        raise ValueError('The weight decay must be finite and non-negative')


def _check_eps(v):
    if not math.isfinite(v) or v <= 0.0:
        raise ValueError('The epsilon value must be finite and positive')


def _group_value(value, pack_size: int, device):
    """`_make_group_value` (`optim.py:70-117`)."""
    if value is None or isinstance(value, (bool, int, float, str, bytes)):
        return value
    if isinstance(value, list):
        if len(value) != pack_size:
            raise ValueError('The size of the hyperparameter list must match the pack size')
        return torch.tensor(value, device=device)
    if isinstance(value, Tensor):
        if value.ndim == 0:
            raise ValueError('Tensors can be used only to specify per-member hyperparameters; use a Python scalar '
                             'to share one value across all members')
        if len(value) != pack_size:
            raise ValueError('The first dimension of a hyperparameter tensor must match the pack size')
        return value.to(device, copy=True)
    raise TypeError(f'Unsupported value type: {type(value)}')


def _defaults(items, *, pack_size):
    out = {}
    for key, value, check in items:
        if isinstance(value, list):
            if len(value) != pack_size:
                raise ValueError('The size of each hyperparameter list must match the pack size')
            for x in value:
                check(x)
        else:
            check(value)
        out[key] = value
    return out


def _hp(v):
    """A group value as the kernels take it: a Python float or a (P,) fp32 CUDA tensor."""
    if isinstance(v, Tensor):
        return v.to(torch.float32).contiguous()
    return float(v)


class OptimizerPack(torch.optim.Optimizer):
    """`OptimizerPack` (`optim.py:158-237`)."""

    def __init__(self, params, defaults: dict[str, Any], *, pack_size: int) -> None:
        super().__init__(params, defaults)
        dev = None
        for g in self.param_groups:
            for p in g['params']:
                dev = p.device
                break
        for k, v in list(self.defaults.items()):
            self.defaults[k] = _group_value(v, pack_size, dev)

    def add_param_group(self, param_group):
        out = super().add_param_group(param_group)
        group = self.param_groups[-1]
        if not group['params']:
            raise ValueError('Empty parameter groups are not supported')
        for p in group['params']:
            if not isinstance(p, ParameterPack):
                raise TypeError('For now, only parameter packs are supported')
        p0 = group['params'][0]
        for k, v in list(group.items()):
            if k != 'params':
                group[k] = _group_value(v, p0.shape[PACK_DIM], p0.device)
        return out

    def _pack_size(self):
        for g in self.param_groups:
            for p in g['params']:
                return p.shape[PACK_DIM]
        return None

    def _replace_impl(self, *, pack_idx: Tensor, items) -> None:
        check_pack_idx(pack_idx, self._pack_size())
        for _, value, check in items:
            if value is not None:
                if len(value) != len(pack_idx):
                    raise ValueError('Each replacement hyperparameter list must contain one value per selected '
                                     'pack member')
                for x in value:
                    check(x)
        for key, value, _ in items:
            if value is None:
                continue
            done = False
            for g in self.param_groups:
                cur = g[key]
                if isinstance(cur, Tensor):
                    cur[pack_idx] = torch.tensor(value, dtype=cur.dtype, device=cur.device)
                    done = True
            if not done:
                raise RuntimeError(f'Replacement is not possible for "{key}"')
        optimizer_pack_reset_state(self, pack_idx=pack_idx)


def _adamw_group(opt: torch.optim.Optimizer, params, *, lr, beta1, beta2, eps, weight_decay,
                 support_replacement: bool) -> None:
    """Grouped AdamW launches over the group's parameter packs (`optim.py:347-427`).

    Parameters whose scalar step counters differ (a parameter that first received a
    gradient later) go to separate launches; per-member step tensors go to one."""
    batches: dict = {}
    for p in params:
        if p.grad is None:
            continue
        if p.grad.is_sparse:
            raise RuntimeError('Sparse gradients are not supported')
        st = opt.state[p]
        if len(st) == 0:
            st['step'] = (torch.zeros(p.shape[PACK_DIM], dtype=torch.int64, device=p.device)
                          if support_replacement else 0)
            st['exp_avg'] = torch.zeros_like(p.data)
            st['exp_avg_sq'] = torch.zeros_like(p.data)
        st['step'] += 1
        key = 'tensor' if isinstance(st['step'], Tensor) else int(st['step'])
        # the parameter itself (not `.data`, whose version counter is separate): the launch bumps
        # its version like an in-place update
        batches.setdefault(key, []).append((p, p.grad.data.contiguous(), st['exp_avg'], st['exp_avg_sq'],
                                            st['step']))
    hp = dict(lr=_hp(lr), beta1=_hp(beta1), beta2=_hp(beta2), eps=_hp(eps), weight_decay=_hp(weight_decay))
    for key, items in batches.items():
        ps, gs, ms, vs, steps = (list(t) for t in zip(*items))
        if key == 'tensor':
            ops.adamw_step(ps, gs, ms, vs, steps=steps, **hp)
        else:
            ops.adamw_step(ps, gs, ms, vs, step=key, **hp)


class AdamWPack(OptimizerPack):
    """`AdamWPack` (`optim.py:269-427`) on the grouped AdamW kernel."""

    def __init__(self, params, *, lr, beta1=0.9, beta2=0.999, eps=1e-8, weight_decay, pack_size: int,
                 support_replacement: bool = False):
        if pack_size <= 0:
            raise ValueError('The pack size must be positive')
        super().__init__(params, _defaults([
            ('lr', lr, _check_lr), ('beta1', beta1, _check_momentum), ('beta2', beta2, _check_momentum),
            ('eps', eps, _check_eps), ('weight_decay', weight_decay, _check_weight_decay)], pack_size=pack_size),
            pack_size=pack_size)
        self._support_replacement: Final = support_replacement

    def replace(self, *, pack_idx: Tensor, lr=None, beta1=None, beta2=None, eps=None, weight_decay=None) -> None:
        if not self._support_replacement:
            raise RuntimeError('Replacing optimizer pack members requires constructing the optimizer with '
                               '`support_replacement=True`')
        self._replace_impl(pack_idx=pack_idx, items=[
            ('lr', lr, _check_lr), ('beta1', beta1, _check_momentum), ('beta2', beta2, _check_momentum),
            ('eps', eps, _check_eps), ('weight_decay', weight_decay, _check_weight_decay)])

    @torch.no_grad()
    def step(self, closure=None):
        loss = closure() if closure is not None else None
        adamw_step(self, support_replacement=self._support_replacement)
        return loss


def compute_muon_update_scale_pack(module: LinearPack) -> Tensor | None:
    """`compute_muon_update_scale_pack` (`optim.py:430-453`)."""
    if module.in_features is None and module.out_features is None:
        return None
    ref = module.in_features if module.in_features is not None else module.out_features
    n, dev = ref.shape[PACK_DIM], ref.device
    o = (torch.full((n,), float(module.max_out_features), device=dev) if module.out_features is None
         else module.out_features.float())
    i = (torch.full((n,), float(module.max_in_features), device=dev) if module.in_features is None
         else module.in_features.float())
    return (o / i).clamp_(min=1.0).sqrt_()


def _widths(module: LinearPack):
    inf = None if module.in_features is None else module.in_features.to(torch.int32)
    outf = None if module.out_features is None else module.out_features.to(torch.int32)
    return outf, inf


class MuonAdamWPack(OptimizerPack):
    """`MuonAdamWPack` (`optim.py:495-861`): Muon for backbone block weights (one
    parameter per group, built with `make_muon_parameter_group`), AdamW for the rest."""

    @staticmethod
    def make_muon_parameter_group(module: LinearPack) -> dict[str, Any]:
        outf, inf = _widths(module)
        return {'params': [module.weight], 'muon': True,
                'muon_update_scale': compute_muon_update_scale_pack(module),
                'muon_out_features': outf, 'muon_in_features': inf}

    def __init__(self, params, *, adamw_lr, adamw_beta1=0.9, adamw_beta2=0.999, adamw_eps=1e-8, weight_decay,
                 muon_lr, muon_momentum=0.95, muon_newton_schulz_steps: int = 5, muon_nesterov: bool = True,
                 muon_skip_zero_updates: bool = False, pack_size: int, support_replacement: bool = False,
                 allow_inplace_grad_mutation: bool, compile_muon_newton_schulz: bool = False):
        if pack_size <= 0:
            raise ValueError('The pack size must be positive')
        del compile_muon_newton_schulz  # the Newton-Schulz iterations always run on the tcgen05 kernels
        super().__init__(params, {
            'muon': False, 'muon_newton_schulz_steps': muon_newton_schulz_steps, 'muon_nesterov': muon_nesterov,
            'muon_skip_zero_updates': muon_skip_zero_updates,
            **_defaults([
                ('adamw_lr', adamw_lr, _check_lr), ('adamw_beta1', adamw_beta1, _check_momentum),
                ('adamw_beta2', adamw_beta2, _check_momentum), ('adamw_eps', adamw_eps, _check_eps),
                ('weight_decay', weight_decay, _check_weight_decay), ('muon_lr', muon_lr, _check_lr),
                ('muon_momentum', muon_momentum, _check_momentum)], pack_size=pack_size)}, pack_size=pack_size)
        self._support_replacement: Final = support_replacement
        self._allow_inplace_grad_mutation: Final = allow_inplace_grad_mutation
        self._workspaces: dict = {}

    def add_param_group(self, param_group):
        out = super().add_param_group(param_group)
        g = self.param_groups[-1]
        if g['muon']:
            if 'muon_update_scale' not in g:
                raise ValueError('The just added parameter group is configured to be optimized with Muon. In this '
                                 'case, it must have the "muon_update_scale" key with the value computed with the '
                                 '`compute_muon_update_scale_pack` function.')
            if len(g['params']) > 1:
                raise ValueError('The just added parameter group configured to be optimized with Muon has more '
                                 'than one parameter, which is not allowed')
        return out

    def replace(self, *, pack_idx: Tensor, adamw_lr=None, adamw_beta1=None, adamw_beta2=None, adamw_eps=None,
                weight_decay=None, muon_lr=None, muon_momentum=None, module) -> None:
        if not self._support_replacement:
            raise RuntimeError('Replacing optimizer pack members requires constructing the optimizer with '
                               '`support_replacement=True`')
        self._replace_impl(pack_idx=pack_idx, items=[
            ('adamw_lr', adamw_lr, _check_lr), ('adamw_beta1', adamw_beta1, _check_momentum),
            ('adamw_beta2', adamw_beta2, _check_momentum), ('adamw_eps', adamw_eps, _check_eps),
            ('weight_decay', weight_decay, _check_weight_decay), ('muon_lr', muon_lr, _check_lr),
            ('muon_momentum', muon_momentum, _check_momentum)])
        by_weight = {m.weight: m for m in module.modules() if isinstance(m, LinearPack)}
        for g in self.param_groups:
            if g['muon']:
                lin = by_weight[g['params'][0]]
                g['muon_update_scale'] = compute_muon_update_scale_pack(lin)
                g['muon_out_features'], g['muon_in_features'] = _widths(lin)

    @torch.no_grad()
    def step(self, closure=None):
        loss = closure() if closure is not None else None
        muon_adamw_step(self, workspaces=self._workspaces, allow_inplace_grad_mutation=self._allow_inplace_grad_mutation,
                        support_replacement=self._support_replacement)
        return loss


def _muon_workspace(workspaces: dict, p: Tensor) -> Tensor:
    """Newton-Schulz workspace of `p`'s device, grown to fit `p`."""
    P, mo, mi = p.shape
    n = ops.muon_workspace_size(P, mo, mi)
    key = (p.device, 'single')
    ws = workspaces.get(key)
    if ws is None or ws.numel() < n:
        ws = torch.empty(n, dtype=torch.uint8, device=p.device)
        workspaces[key] = ws
    return ws


def _muon_kwargs(opt: torch.optim.Optimizer, g: dict, *, allow_inplace_grad_mutation: bool):
    """`MuonAdamWPack._step_muon` (`optim.py:682-774`) for one single-parameter Muon group, as
    the arguments of `ops.muon_step` (weight decay, momentum, Nesterov blend, batched
    Newton-Schulz and the scaled update run in the Muon kernels), or None when the parameter
    has no gradient.  Per-member widths (`muon_out_features` / `muon_in_features`) keep each
    member's Newton-Schulz on its own out x in block; without them it runs on the padded block
    (the reference's arithmetic: zero padding rows and columns do not change the result).  The
    second value is the bf16 compute-copy cache to close after the step."""
    p = g['params'][0]
    if p.ndim != 3:
        raise ValueError('Parameters optimized with Muon must have three dimensions')
    if p.grad is None:
        return None, None
    if p.grad.is_sparse:
        raise RuntimeError('Sparse gradients are not supported')
    st = opt.state[p]
    if len(st) == 0:
        st['muon_momentum_buffer'] = torch.zeros_like(p)
    scale = g.get('muon_update_scale')
    # the layer's bf16 compute copy, refreshed in the pass that writes the weights (otherwise the
    # next forward casts the whole weight pack again)
    cache = bf16_copy_cache(p)
    copy = cache.begin_update(p) if cache is not None else None
    # without in-place mutation the kernel leaves the gradient as it is (the reference blends
    # into a copy), so no copy is made here
    kw = dict(p=p, grad=p.grad.data, momentum_buffer=st['muon_momentum_buffer'],
              out_features=g.get('muon_out_features'), in_features=g.get('muon_in_features'),
              lr=_hp(g['muon_lr']), momentum=_hp(g['muon_momentum']), weight_decay=_hp(g['weight_decay']),
              update_scale=None if scale is None else scale.to(torch.float32).contiguous(),
              nesterov=bool(g['muon_nesterov']), mutate_grad=allow_inplace_grad_mutation,
              ns_steps=int(g['muon_newton_schulz_steps']), p_bf16=copy, n_blocks=g.get('muon_n_blocks'),
              block_index=int(g.get('muon_block_index', 0)),
              gated_momentum_zero=bool(g.get('muon_gated_momentum_zero', False)))
    return kw, (cache, copy)


def _close_copy(kw: dict, closing) -> None:
    cache, copy = closing
    if copy is not None:
        cache.end_update(kw['p'], copy)


def _muon_group(opt: torch.optim.Optimizer, g: dict, *, workspaces: dict, allow_inplace_grad_mutation: bool) -> None:
    """One Muon group in its own call (`tp_muon_step`)."""
    kw, closing = _muon_kwargs(opt, g, allow_inplace_grad_mutation=allow_inplace_grad_mutation)
    if kw is None:
        return
    ops.muon_step(**kw, workspace=_muon_workspace(workspaces, kw['p']))
    _close_copy(kw, closing)


def _muon_groups(opt: torch.optim.Optimizer, groups: list, *, workspaces: dict,
                 allow_inplace_grad_mutation: bool) -> None:
    """The Muon groups of one device in one grouped call (`tp_muon_step_grouped`): the same
    results as one call per group, with the Newton-Schulz GEMMs of all groups in shared
    launches (fewer and fuller launches: the tails of one group's launches no longer leave
    SMs idle)."""
    built = [_muon_kwargs(opt, g, allow_inplace_grad_mutation=allow_inplace_grad_mutation) for g in groups]
    built = [(kw, c) for kw, c in built if kw is not None]
    if not built:
        return
    steps = [kw for kw, _ in built]
    if len({kw['ns_steps'] for kw in steps}) > 1:
        for kw, closing in built:
            ops.muon_step(**kw, workspace=_muon_workspace(workspaces, kw['p']))
            _close_copy(kw, closing)
        return
    need = ops.muon_grouped_workspace_size([tuple(kw['p'].shape) for kw in steps])
    dev = steps[0]['p'].device
    key = (dev, 'grouped')
    ws = workspaces.get(key)
    if ws is None or ws.numel() < need:
        ws = torch.empty(need, dtype=torch.uint8, device=dev)
        workspaces[key] = ws
    ops.muon_step_grouped(steps, workspace=ws)
    for kw, closing in built:
        _close_copy(kw, closing)


def adamw_step(opt: torch.optim.Optimizer, *, support_replacement: bool) -> None:
    """`AdamWPack.step` (`optim.py:347-427`) over every group of `opt` (keys `lr`, `beta1`,
    `beta2`, `eps`, `weight_decay`), one grouped AdamW launch per group."""
    for g in opt.param_groups:
        _adamw_group(opt, g['params'], lr=g['lr'], beta1=g['beta1'], beta2=g['beta2'], eps=g['eps'],
                     weight_decay=g['weight_decay'], support_replacement=support_replacement)


def muon_adamw_step(opt: torch.optim.Optimizer, *, workspaces: dict, allow_inplace_grad_mutation: bool,
                    support_replacement: bool) -> None:
    """`MuonAdamWPack.step` (`optim.py:495-861`) over every group of `opt`: Muon groups through
    the Muon kernels, the others through the grouped AdamW kernel (`adamw_*` keys).

    The Muon groups of one device go to one grouped call when there are several (unless the
    optimizer's `grouped_muon` is False, e.g. to time each group's launches on their own)."""
    by_device: dict = {}
    for g in opt.param_groups:
        if g['muon'] and g['params'][0].grad is not None:
            by_device.setdefault(g['params'][0].device, []).append(g)
    for dev, groups in by_device.items():
        if len(groups) > 1 and dev.type == 'cuda' and getattr(opt, 'grouped_muon', True):
            _muon_groups(opt, groups, workspaces=workspaces, allow_inplace_grad_mutation=allow_inplace_grad_mutation)
        else:
            for g in groups:
                _muon_group(opt, g, workspaces=workspaces, allow_inplace_grad_mutation=allow_inplace_grad_mutation)
    for g in opt.param_groups:
        if not g['muon']:
            _adamw_group(opt, g['params'], lr=g['adamw_lr'], beta1=g['adamw_beta1'], beta2=g['adamw_beta2'],
                         eps=g['adamw_eps'], weight_decay=g['weight_decay'], support_replacement=support_replacement)


def optimizer_pack_remove(optimizer, *, pack_idx: Tensor, old_to_new_parameters) -> None:
    """`optimizer_pack_remove` (`optim.py:867-910`)."""
    if not old_to_new_parameters:
        raise ValueError('The mapping from old parameters to new parameters must not be empty')
    P = None
    for g in optimizer.param_groups:
        for p in g['params']:
            if isinstance(p, ParameterPack):
                P = p.shape[PACK_DIM]
                break
        if P is not None:
            break
    if P is None:
        raise ValueError('Failed to infer the pack size')
    check_pack_idx(pack_idx, P)
    keep = make_complementary_pack_idx(pack_idx, pack_size=P)
    for g in optimizer.param_groups:
        for k, v in list(g.items()):
            if isinstance(v, Tensor) and v.ndim > 0:
                g[k] = v[keep]
        for i, p in list(enumerate(g['params'])):
            if isinstance(p, ParameterPack):
                st = optimizer.state.pop(p, None)
                if st is not None:
                    for k, v in list(st.items()):
                        if isinstance(v, Tensor) and v.ndim > 0:
                            st[k] = v[keep]
                new_p = old_to_new_parameters[p]
                g['params'][i] = new_p
                if st is not None:
                    optimizer.state[new_p] = st


def optimizer_pack_reset_state(optimizer, *, pack_idx: Tensor) -> None:
    """`optimizer_pack_reset_state` (`optim.py:913-926`)."""
    for g in optimizer.param_groups:
        for p in g['params']:
            st = optimizer.state.get(p)
            if st is not None:
                for v in st.values():
                    if isinstance(v, Tensor) and v.ndim > 0:
                        v[pack_idx] = 0


def should_skip_weight_decay(module_name: str, module, parameter_name: str, parameter) -> bool:
    """`should_skip_weight_decay` (`optim.py:929-943`) for the packs of this package: biases
    and the frequencies of cosine embeddings take no weight decay."""
    del module_name
    from tabpack_b200.nn import CosineEmbeddingsPack

    return parameter_name.endswith('bias') or (isinstance(module, CosineEmbeddingsPack) and parameter is module.weight)


def split_weight_decay(model) -> tuple[list, list]:
    """(parameters with weight decay, parameters without) by `should_skip_weight_decay`."""
    decay, no_decay = [], []
    for mname, mod in model.named_modules():
        for pname, p in mod.named_parameters(recurse=False):
            (no_decay if should_skip_weight_decay(mname, mod, pname, p) else decay).append(p)
    return decay, no_decay
