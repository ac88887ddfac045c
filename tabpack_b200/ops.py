"""Torch-facing wrappers of the C ABI.

These functions only validate tensors, allocate outputs with PyTorch's caching
allocator and pass raw pointers plus the current CUDA stream to the library.
All arithmetic happens in the CUDA kernels; CPU tensors are rejected.
"""

from __future__ import annotations

import ctypes

import torch
from torch import Tensor
from torch.autograd.graph import increment_version

from tabpack_b200 import _lib
from tabpack_b200._lib import TP_DTYPE_BF16, TP_DTYPE_F32, check, load


class KernelTimes:
    """Per-family device time of this library's kernel launches (`tp_profile_start` /
    `tp_profile_stop`): `with KernelTimes() as kt: ...` then `kt.ms` and `kt.launches`, dicts
    keyed by family name (`_lib.TP_PROF_KINDS`).  Each launch is bracketed by two CUDA events
    on its stream; the totals are read once the block ends (a synchronisation)."""

    def __init__(self, capacity: int = 1 << 16) -> None:
        self.capacity = capacity
        self.ms: dict[str, float] = {}
        self.launches: dict[str, int] = {}
        self.dropped = 0

    def __enter__(self) -> 'KernelTimes':
        check(load().tp_profile_start(self.capacity), 'tp_profile_start')
        return self

    def __exit__(self, *exc) -> None:
        n = len(_lib.TP_PROF_KINDS)
        ms = (ctypes.c_double * n)()
        cnt = (ctypes.c_int64 * n)()
        dropped = ctypes.c_int32(0)
        check(load().tp_profile_stop(ms, cnt, n, ctypes.byref(dropped)), 'tp_profile_stop')
        self.ms = {k: ms[i] for i, k in enumerate(_lib.TP_PROF_KINDS)}
        self.launches = {k: cnt[i] for i, k in enumerate(_lib.TP_PROF_KINDS)}
        self.dropped = dropped.value


def _ptr(t: Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _dtype_code(dt: torch.dtype) -> int:
    if dt == torch.bfloat16:
        return TP_DTYPE_BF16
    if dt == torch.float32:
        return TP_DTYPE_F32
    raise TypeError(f'unsupported activation dtype {dt} (bf16 or fp32)')


def _cuda(name: str, t: Tensor | None, dtype: torch.dtype | None = None) -> Tensor | None:
    if t is None:
        return None
    if not t.is_cuda:
        raise RuntimeError(f'{name} must be a CUDA tensor (tabpack_b200 has no CPU path)')
    if dtype is not None and t.dtype != dtype:
        raise TypeError(f'{name} must have dtype {dtype}, got {t.dtype}')
    return t.contiguous()


def _i32(name: str, t: Tensor | None) -> Tensor | None:
    if t is None:
        return None
    if not t.is_cuda:
        raise RuntimeError(f'{name} must be a CUDA tensor')
    return t.to(torch.int32).contiguous()


def _linear_args(x, weight, bias, in_features, out_features, n_blocks, block_index, relu,
                 dropout_p, seed, offset, member_base, y, row_index=None) -> _lib.LinearArgs:
    P, max_out, max_in = weight.shape
    shared = x.ndim == 2 and row_index is None
    B = row_index.shape[1] if row_index is not None else x.shape[0] if shared else x.shape[1]
    a = _lib.LinearArgs()
    a.P, a.B, a.max_in, a.max_out = P, B, max_in, max_out
    a.dtype = _dtype_code(x.dtype)
    a.x_shared = 1 if shared else 0
    if row_index is not None:
        a.row_index, a.x_rows = row_index.data_ptr(), x.shape[0]
    a.in_features = _ptr(in_features)
    a.out_features = _ptr(out_features)
    a.n_blocks = _ptr(n_blocks)
    a.block_index = int(block_index)
    a.relu = 1 if relu else 0
    a.dropout_p = _ptr(dropout_p)
    a.seed = int(seed) & 0xFFFFFFFFFFFFFFFF
    a.offset = int(offset) & 0xFFFFFFFF
    a.member_base = int(member_base) & 0xFFFFFFFF
    a.x = _ptr(x)
    a.w = _ptr(weight)
    a.bias = _ptr(bias)
    a.y = _ptr(y)
    return a


def _row_index(row_index: Tensor | None, P: int) -> Tensor | None:
    """(P, B) int32 CUDA row indices of a gathered input, or None."""
    if row_index is None:
        return None
    if row_index.ndim != 2 or row_index.shape[0] != P:
        raise ValueError(f'row_index must be (pack_size={P}, batch), got {tuple(row_index.shape)}')
    if not row_index.is_cuda:
        raise RuntimeError('row_index must be a CUDA tensor (tabpack_b200 has no CPU path)')
    return row_index.to(torch.int32).contiguous()


def linear_forward(
    x: Tensor,
    weight: Tensor,
    bias: Tensor | None,
    *,
    in_features: Tensor | None = None,
    out_features: Tensor | None = None,
    n_blocks: Tensor | None = None,
    block_index: int = 0,
    relu: bool = False,
    dropout_p: Tensor | None = None,
    seed: int = 0,
    offset: int = 0,
    member_base: int = 0,
    row_index: Tensor | None = None,
    y: Tensor | None = None,
) -> Tensor:
    """Packed linear (+ReLU +dropout +depth gating) forward; see `tp_linear_forward`.  With
    `row_index` (P, B), x is a (rows, in) table and member m's input row b is
    x[row_index[m, b]] (gathered by the GEMM's operand loads).  `y`: an output buffer whose
    padding columns already hold zeros (`y_pad_zero`: only the members' column tiles are
    written); by default a new one."""
    weight = _cuda('weight', weight)
    x = _cuda('x', x, weight.dtype)
    row_index = _row_index(row_index, weight.shape[0])
    bias = _cuda('bias', bias, torch.float32)
    dropout_p = _cuda('dropout_p', dropout_p, torch.float32)
    in_features, out_features, n_blocks = (_i32(n, t) for n, t in (
        ('in_features', in_features), ('out_features', out_features), ('n_blocks', n_blocks)))
    P, max_out, _ = weight.shape
    B = x.shape[-2] if row_index is None else row_index.shape[1]
    pad_zero = y is not None
    if y is None:
        y = torch.empty((P, B, max_out), dtype=x.dtype, device=x.device)
    elif tuple(y.shape) != (P, B, max_out) or y.dtype != x.dtype or not y.is_contiguous() or y.device != x.device:
        raise ValueError(f'y must be a contiguous ({P}, {B}, {max_out}) {x.dtype} tensor on {x.device}')
    a = _linear_args(x, weight, bias, in_features, out_features, n_blocks, block_index, relu,
                     dropout_p, seed, offset, member_base, y, row_index)
    a.y_pad_zero = 1 if pad_zero else 0
    check(load().tp_linear_forward(ctypes.byref(a), _stream()), 'tp_linear_forward')
    if pad_zero:
        increment_version([y])
    return y


def linear_backward(
    dy: Tensor,
    x: Tensor,
    weight: Tensor,
    y: Tensor | None,
    *,
    in_features: Tensor | None = None,
    out_features: Tensor | None = None,
    n_blocks: Tensor | None = None,
    block_index: int = 0,
    relu: bool = False,
    dropout_p: Tensor | None = None,
    seed: int = 0,
    offset: int = 0,
    member_base: int = 0,
    need_dx: bool = True,
    need_dw: bool = True,
    need_db: bool = True,
    dw_shape: tuple[int, int] | None = None,
    db_cols: int | None = None,
    dx_cols: int = 0,
    row_index: Tensor | None = None,
    dw_out: Tensor | None = None,
    dw_pad_zero: bool = False,
    dx_out: Tensor | None = None,
) -> tuple[Tensor | None, Tensor | None, Tensor | None]:
    """Backward of `linear_forward`: returns (dx, dw, db); dw/db are fp32.  With dx_cols > 0
    only dx's first dx_cols columns are computed (the rest are zeros).  With `row_index`, x is
    the forward's table (no dx).  `dw_out`: the weight gradient's buffer (else a new one);
    `dw_pad_zero`: it already holds zeros outside the active members' blocks (`tp_linear_grad_args`).
    `dx_out`: the input gradient's buffer, whose columns beyond each member's input column tiles
    already hold zeros (`dx_pad_zero`); by default a new one."""
    weight = _cuda('weight', weight)
    x = _cuda('x', x, weight.dtype)
    row_index = _row_index(row_index, weight.shape[0])
    if row_index is not None and need_dx:
        raise ValueError('a gathered input (a table) takes no input gradient')
    dy = _cuda('dy', dy, weight.dtype)
    y = _cuda('y', y, weight.dtype)
    dropout_p = _cuda('dropout_p', dropout_p, torch.float32)
    in_features, out_features, n_blocks = (_i32(n, t) for n, t in (
        ('in_features', in_features), ('out_features', out_features), ('n_blocks', n_blocks)))
    P, max_out, max_in = weight.shape
    B = x.shape[-2] if row_index is None else row_index.shape[1]
    need_g = relu or dropout_p is not None or out_features is not None or n_blocks is not None
    g = torch.empty_like(dy) if need_g else None
    dx = None
    if need_dx:
        if dx_out is not None:
            if (tuple(dx_out.shape) != (P, B, max_in) or dx_out.dtype != dy.dtype or not dx_out.is_contiguous()
                    or dx_out.device != dy.device):
                raise ValueError(f'dx_out must be a contiguous ({P}, {B}, {max_in}) {dy.dtype} tensor on {dy.device}')
            dx = dx_out
        else:
            dx = torch.empty((P, B, max_in), dtype=dy.dtype, device=dy.device)
    rows, cols = dw_shape if dw_shape is not None else (max_out, max_in)
    dw = None
    if need_dw:
        if dw_out is not None:
            if (tuple(dw_out.shape) != (P, rows, cols) or dw_out.dtype != torch.float32 or not dw_out.is_contiguous()
                    or dw_out.device != dy.device):
                raise ValueError('dw_out must be a contiguous fp32 (P, rows, cols) tensor on the gradient device')
            dw = dw_out
        else:
            dw = torch.empty((P, rows, cols), dtype=torch.float32, device=dy.device)
    dbc = db_cols if db_cols is not None else max_out
    db = torch.empty((P, dbc), dtype=torch.float32, device=dy.device) if need_db else None
    ga = _lib.LinearGradArgs()
    ga.fwd = _linear_args(x, weight, None, in_features, out_features, n_blocks, block_index, relu,
                          dropout_p, seed, offset, member_base, None, row_index)
    ga.dy, ga.y, ga.g = _ptr(dy), _ptr(y), _ptr(g)
    ga.dbias, ga.dx, ga.dw = _ptr(db), _ptr(dx), _ptr(dw)
    ga.dw_rows, ga.dw_cols, ga.db_cols = rows, cols, dbc
    ga.dx_cols = int(dx_cols)
    ga.dw_pad_zero = 1 if (dw_pad_zero and dw_out is not None) else 0
    ga.dx_pad_zero = 1 if (dx is not None and dx_out is not None) else 0
    check(load().tp_linear_backward(ctypes.byref(ga), _stream()), 'tp_linear_backward')
    if ga.dx_pad_zero:
        increment_version([dx])
    return dx, dw, db


def dropout_mask(*, seed: int, offset: int, member_base: int, p: Tensor, rows: int, cols: int) -> Tensor:
    """(P, rows, cols) uint8 Philox keep mask used by the fused dropout."""
    p = _cuda('p', p, torch.float32)
    P = p.shape[0]
    mask = torch.empty((P, rows, cols), dtype=torch.uint8, device=p.device)
    check(load().tp_dropout_mask(int(seed) & 0xFFFFFFFFFFFFFFFF, int(offset) & 0xFFFFFFFF,
                                 int(member_base) & 0xFFFFFFFF, p.data_ptr(), P, rows, cols,
                                 mask.data_ptr(), _stream()), 'tp_dropout_mask')
    return mask


def _hparam(v) -> _lib.HParam:
    h = _lib.HParam()
    if isinstance(v, Tensor):
        if not v.is_cuda or v.dtype != torch.float32 or v.ndim != 1:
            raise TypeError('per-member hyperparameters must be 1-D fp32 CUDA tensors')
        h.per_member = v.data_ptr()
        h.scalar = 0.0
    else:
        h.per_member = None
        h.scalar = float(v)
    return h


def adamw_step(params, grads, exp_avgs, exp_avg_sqs, *, steps=None, step: int = 0,
               lr, beta1, beta2, eps, weight_decay) -> None:
    """Grouped AdamW over parameter packs (each (P, ...) fp32, contiguous).

    `steps` (per-tensor (P,) int64 tensors, already incremented) or the scalar
    `step` give the bias-correction step.  Hyperparameters are floats or (P,)
    fp32 CUDA tensors.  Tensors are chunked into launches of at most 32.
    """
    hp = [lr, beta1, beta2, eps, weight_decay]
    hp = [v.contiguous() if isinstance(v, Tensor) else v for v in hp]
    n = len(params)
    for s in range(0, n, _lib.TP_MAX_OPT_TENSORS):
        a = _lib.AdamWArgs()
        chunk = range(s, min(n, s + _lib.TP_MAX_OPT_TENSORS))
        a.n_tensors = len(chunk)
        for j, i in enumerate(chunk):
            p = params[i]
            for name, t in (('param', p), ('grad', grads[i]), ('exp_avg', exp_avgs[i]),
                            ('exp_avg_sq', exp_avg_sqs[i])):
                if not t.is_cuda or t.dtype != torch.float32 or not t.is_contiguous():
                    raise TypeError(f'{name} must be a contiguous fp32 CUDA tensor')
            ot = a.t[j]
            ot.p, ot.grad = p.data_ptr(), grads[i].data_ptr()
            ot.exp_avg, ot.exp_avg_sq = exp_avgs[i].data_ptr(), exp_avg_sqs[i].data_ptr()
            ot.step = None if steps is None else steps[i].data_ptr()
            ot.numel = p.numel()
            ot.inner = max(1, p.numel() // p.shape[0])
        a.lr, a.beta1, a.beta2, a.eps, a.weight_decay = (_hparam(v) for v in hp)
        a.step = int(step)
        check(load().tp_adamw_step(ctypes.byref(a), _stream()), 'tp_adamw_step')
    # the kernel updated these in place: bump their version counters as torch's in-place ops do
    # (caches keyed on a parameter's version, e.g. its bf16 copy, see the new values)
    increment_version(list(params) + list(exp_avgs) + list(exp_avg_sqs))


def muon_workspace_size(P: int, max_out: int, max_in: int) -> int:
    """Bytes of scratch one `muon_step` call on a (P, max_out, max_in) pack needs."""
    return int(load().tp_muon_workspace_size(P, max_out, max_in))


def _muon_args(p: Tensor, grad: Tensor, momentum_buffer: Tensor, *, out_features=None, in_features=None, lr,
               momentum, weight_decay, update_scale=None, nesterov: bool = True, mutate_grad: bool = True,
               ns_steps: int = 5, p_bf16: Tensor | None = None, n_blocks: Tensor | None = None,
               block_index: int = 0, gated_momentum_zero: bool = False):
    """`tp_muon_args` of one group (workspace unset), the tensors that must stay alive until
    the launch is queued, and the tensors the step writes."""
    for name, t in (('p', p), ('grad', grad), ('momentum_buffer', momentum_buffer)):
        if not t.is_cuda or t.dtype != torch.float32 or not t.is_contiguous() or t.ndim != 3:
            raise TypeError(f'{name} must be a contiguous 3-D fp32 CUDA tensor')
    P, mo, mi = p.shape
    a = _lib.MuonArgs()
    a.P, a.max_out, a.max_in = P, mo, mi
    a.p, a.grad, a.momentum_buffer = p.data_ptr(), grad.data_ptr(), momentum_buffer.data_ptr()
    of, inf = _i32('out_features', out_features), _i32('in_features', in_features)
    a.out_features, a.in_features = _ptr(of), _ptr(inf)
    a.lr, a.momentum, a.weight_decay = _hparam(lr), _hparam(momentum), _hparam(weight_decay)
    us = _cuda('update_scale', update_scale, torch.float32)
    a.update_scale = _ptr(us)
    a.nesterov, a.mutate_grad, a.ns_steps = int(nesterov), int(mutate_grad), int(ns_steps)
    if p_bf16 is not None:
        if (not p_bf16.is_cuda or p_bf16.dtype != torch.bfloat16 or not p_bf16.is_contiguous() or p_bf16.ndim != 3
                or p_bf16.shape[0] != P):
            raise TypeError('p_bf16 must be a contiguous (P, rows, cols) bf16 CUDA tensor')
        a.p_bf16, a.p_bf16_rows, a.p_bf16_cols = p_bf16.data_ptr(), p_bf16.shape[1], p_bf16.shape[2]
    nb = _i32('n_blocks', n_blocks)
    if nb is not None:
        if nb.shape != (P,):
            raise ValueError(f'n_blocks must be ({P},), got {tuple(nb.shape)}')
        a.n_blocks, a.block_index = nb.data_ptr(), int(block_index)
        a.gated_momentum_zero = 1 if gated_momentum_zero else 0
    keep = (of, inf, us, nb, lr, momentum, weight_decay)
    written = [p, momentum_buffer] + ([grad] if mutate_grad else []) + ([p_bf16] if p_bf16 is not None else [])
    return a, keep, written


def muon_step(p: Tensor, grad: Tensor, momentum_buffer: Tensor, *, out_features=None, in_features=None, lr,
              momentum, weight_decay, update_scale=None, nesterov: bool = True, mutate_grad: bool = True,
              ns_steps: int = 5, workspace: Tensor | None = None, p_bf16: Tensor | None = None,
              n_blocks: Tensor | None = None, block_index: int = 0, gated_momentum_zero: bool = False) -> None:
    """One Muon group step on a packed (P, max_out, max_in) fp32 weight; see `tp_muon_step`.
    `p_bf16` (P, rows >= max_out, cols >= max_in) bf16, optional, receives bf16 of the updated
    weights of each member's out x in block in the same pass.  `n_blocks` / `block_index`: the
    weight's block is depth-gated for members with n_blocks <= block_index (their gradient is
    exactly zero and is not read); `gated_momentum_zero`: their momentum is zero as well (not
    read either)."""
    a, keep, written = _muon_args(p, grad, momentum_buffer, out_features=out_features, in_features=in_features,
                                  lr=lr, momentum=momentum, weight_decay=weight_decay, update_scale=update_scale,
                                  nesterov=nesterov, mutate_grad=mutate_grad, ns_steps=ns_steps, p_bf16=p_bf16,
                                  n_blocks=n_blocks, block_index=block_index,
                                  gated_momentum_zero=gated_momentum_zero)
    P, mo, mi = p.shape
    need = muon_workspace_size(P, mo, mi)
    if workspace is None or workspace.numel() * workspace.element_size() < need:
        workspace = torch.empty(need, dtype=torch.uint8, device=p.device)
    a.workspace, a.workspace_bytes = workspace.data_ptr(), workspace.numel() * workspace.element_size()
    check(load().tp_muon_step(ctypes.byref(a), _stream()), 'tp_muon_step')
    del keep
    increment_version(written)


def muon_grouped_workspace_size(shapes: list[tuple[int, int, int]]) -> int:
    """Bytes of the workspace of a grouped Muon call over weights of these (P, max_out, max_in)."""
    arr = (_lib.MuonArgs * len(shapes))()
    for a, (P, mo, mi) in zip(arr, shapes):
        a.P, a.max_out, a.max_in = P, mo, mi
    return int(load().tp_muon_grouped_workspace_size(arr, len(shapes)))


def muon_step_grouped(steps: list[dict], *, workspace: Tensor | None = None) -> None:
    """Several Muon groups of one device in one call (`tp_muon_step_grouped`): each entry of
    `steps` holds `muon_step`'s arguments for one group (`p`, `grad`, `momentum_buffer`, ...,
    without `workspace`).  Each group's result equals its own `muon_step` bit for bit; the
    Newton-Schulz GEMMs of all groups share launches."""
    if not steps:
        return
    built = [_muon_args(**kw) for kw in steps]
    arr = (_lib.MuonArgs * len(built))(*[b[0] for b in built])
    need = muon_grouped_workspace_size([tuple(kw['p'].shape) for kw in steps])
    dev = steps[0]['p'].device
    if workspace is None or workspace.numel() * workspace.element_size() < need:
        workspace = torch.empty(need, dtype=torch.uint8, device=dev)
    check(load().tp_muon_step_grouped(arr, len(built), workspace.data_ptr(),
                                      workspace.numel() * workspace.element_size(), _stream()),
          'tp_muon_step_grouped')
    del built
    increment_version([t for kw in steps for t in _muon_written(kw)])


def _muon_written(kw: dict) -> list:
    out = [kw['p'], kw['momentum_buffer']]
    if kw.get('mutate_grad', True):
        out.append(kw['grad'])
    if kw.get('p_bf16') is not None:
        out.append(kw['p_bf16'])
    return out


def metric_pack(metric: str, y_pred: Tensor, y_true: Tensor, classes: int = 1) -> Tensor:
    """(P,) metric values; y_pred (P, N[, classes]); see `tp_metric_pack`."""
    code = _lib.TP_METRIC[metric]
    y_pred = _cuda('y_pred', y_pred)
    y_true = _cuda('y_true', y_true)
    if code == _lib.TP_METRIC['accuracy']:
        y_pred, y_true = y_pred.to(torch.int64), y_true.to(torch.int64)
    elif code in (_lib.TP_METRIC['mse'], _lib.TP_METRIC['mae'], _lib.TP_METRIC['r2']):
        y_pred, y_true = y_pred.to(torch.float32), y_true.to(torch.float32)
    else:
        y_pred, y_true = y_pred.to(torch.float32), y_true.to(torch.int64)
    y_pred, y_true = y_pred.contiguous(), y_true.contiguous()
    P = y_pred.shape[0]
    N = y_true.numel()
    out = torch.empty(P, dtype=torch.float32, device=y_pred.device)
    a = _lib.MetricArgs(metric=code, P=P, N=N, C=classes, y_pred=y_pred.data_ptr(), y_true=y_true.data_ptr(),
                        out=out.data_ptr())
    check(load().tp_metric_pack(ctypes.byref(a), _stream()), 'tp_metric_pack')
    return out


def greedy_ensemble(predictions: Tensor, y_true: Tensor, *, metric: str, maximize: bool, classes: int = 1,
                    init_top_k: int = 1, max_ensemble_size: int | None = None,
                    with_replacement: bool = False) -> tuple[Tensor, Tensor]:
    """Fused greedy selection; returns (counts (n_pred,) int32, status (3,) int32) on the device."""
    code = _lib.TP_METRIC[metric]
    pred = _cuda('predictions', predictions).to(torch.float32).contiguous()
    yt = _cuda('y_true', y_true)
    yt = (yt.to(torch.float32) if metric in ('mse', 'mae') else yt.to(torch.int64)).contiguous()
    n_pred = pred.shape[0]
    N = yt.numel()
    ws = torch.empty(int(load().tp_greedy_workspace_size(n_pred, N, classes)), dtype=torch.uint8, device=pred.device)
    counts = torch.empty(n_pred, dtype=torch.int32, device=pred.device)
    status = torch.zeros(3, dtype=torch.int32, device=pred.device)
    a = _lib.GreedyArgs(metric=code, maximize=int(maximize), n_pred=n_pred, N=N, C=classes,
                        predictions=pred.data_ptr(), y_true=yt.data_ptr(), init_top_k=init_top_k,
                        max_ensemble_size=0 if max_ensemble_size is None else int(max_ensemble_size),
                        with_replacement=int(with_replacement), counts=counts.data_ptr(), workspace=ws.data_ptr(),
                        workspace_bytes=ws.numel(), status=status.data_ptr())
    check(load().tp_greedy_ensemble(ctypes.byref(a), _stream()), 'tp_greedy_ensemble')
    return counts, status


def ensemble_mean(pred: Tensor, idx: Tensor, weights: Tensor | None = None) -> Tensor:
    """(Weighted) mean of pred[idx] over the first dimension; see `tp_ensemble_mean`."""
    pred = _cuda('pred', pred, torch.float32)
    idx = _i32('idx', idx)
    weights = None if weights is None else _cuda('weights', weights).to(torch.float32).contiguous()
    out = torch.empty(pred.shape[1:], dtype=torch.float32, device=pred.device)
    n = out.numel()
    check(load().tp_ensemble_mean(pred.data_ptr(), idx.data_ptr(), _ptr(weights), idx.numel(), n, out.data_ptr(),
                                  _stream()), 'tp_ensemble_mean')
    return out


def softmax_rows(x: Tensor) -> Tensor:
    """Softmax over the last dimension (fp32); see `tp_softmax_rows`."""
    x = _cuda('x', x).to(torch.float32).contiguous()
    out = torch.empty_like(x)
    C = x.shape[-1]
    check(load().tp_softmax_rows(x.data_ptr(), x.numel() // C, C, out.data_ptr(), _stream()), 'tp_softmax_rows')
    return out


def permutation_keys(*, seed: int, epoch: int, member_base: int, P: int, N: int, device) -> Tensor:
    """(P, N) int32 Philox keys whose per-row stable argsort is each member's batch order."""
    keys = torch.empty((P, N), dtype=torch.int32, device=device)
    check(load().tp_permutation_keys(int(seed) & 0xFFFFFFFFFFFFFFFF, int(epoch) & 0xFFFFFFFF,
                                     int(member_base) & 0xFFFFFFFF, P, N, keys.data_ptr(), _stream()),
          'tp_permutation_keys')
    return keys


def _cos_emb_args(x, weight, bias, affine_weight, affine_bias, d_embedding):
    P, F, D = affine_weight.shape
    for name, t in (('weight', weight), ('bias', bias), ('affine_weight', affine_weight),
                    ('affine_bias', affine_bias)):
        if not t.is_cuda or t.dtype != torch.float32 or not t.is_contiguous():
            raise TypeError(f'{name} must be a contiguous fp32 CUDA tensor')
    x = _cuda('x', x, torch.float32)
    if x.ndim == 2:
        B, shared = x.shape[0], 1
    else:
        B, shared = x.shape[1], 0
    if x.shape[-1] != F:
        raise ValueError('The number of input features must match the number of features configured for the embeddings')
    d = _i32('d_embedding', d_embedding)
    a = _lib.CosEmbArgs(P=P, B=B, F=F, D=D, x_shared=shared, x=x.data_ptr(), weight=weight.data_ptr(),
                        bias=bias.data_ptr(), affine_weight=affine_weight.data_ptr(),
                        affine_bias=affine_bias.data_ptr(), d_embedding=_ptr(d))
    return a, (x, d)


def cos_emb_forward(x: Tensor, weight: Tensor, bias: Tensor, affine_weight: Tensor, affine_bias: Tensor,
                    d_embedding: Tensor | None = None, *, out: Tensor | None = None,
                    dtype: torch.dtype = torch.float32) -> Tensor:
    """Cosine embeddings of x (P, B, F) or shared (B, F) into the first F * D columns of `out`
    (P, B, >= F * D; allocated (P, B, F * D) of `dtype` when None); see `tp_cos_emb_forward`."""
    a, keep = _cos_emb_args(x, weight, bias, affine_weight, affine_bias, d_embedding)
    if out is None:
        out = torch.empty(a.P, a.B, a.F * a.D, dtype=dtype, device=weight.device)
    if out.stride(-1) != 1 or out.stride(0) != out.shape[1] * out.stride(1) or out.dtype not in (torch.float32,
                                                                                                   torch.bfloat16):
        raise TypeError('out must be a row-major fp32 or bf16 (P, B, width) tensor')
    a.out, a.out_ld = out.data_ptr(), out.stride(1)
    a.out_dtype = TP_DTYPE_BF16 if out.dtype == torch.bfloat16 else TP_DTYPE_F32
    check(load().tp_cos_emb_forward(ctypes.byref(a), _stream()), 'tp_cos_emb_forward')
    del keep
    return out


def cos_emb_backward(x: Tensor, weight: Tensor, bias: Tensor, affine_weight: Tensor, affine_bias: Tensor,
                     d_embedding: Tensor | None, grad_out: Tensor):
    """Parameter gradients (dweight, dbias, daffine_weight, daffine_bias) from the gradient of the
    flattened embedding (its first F * D columns); see `tp_cos_emb_backward`."""
    a, keep = _cos_emb_args(x, weight, bias, affine_weight, affine_bias, d_embedding)
    if grad_out.stride(-1) != 1 or grad_out.stride(0) != grad_out.shape[1] * grad_out.stride(1):
        grad_out = grad_out.contiguous()
    if grad_out.dtype not in (torch.float32, torch.bfloat16):
        grad_out = grad_out.float()
    a.grad_out, a.grad_ld = grad_out.data_ptr(), grad_out.stride(1)
    a.grad_dtype = TP_DTYPE_BF16 if grad_out.dtype == torch.bfloat16 else TP_DTYPE_F32
    dweight, dbias = torch.empty_like(weight), torch.empty_like(bias)
    daw, dab = torch.empty_like(affine_weight), torch.empty_like(affine_bias)
    a.dweight, a.dbias = dweight.data_ptr(), dbias.data_ptr()
    a.daffine_weight, a.daffine_bias = daw.data_ptr(), dab.data_ptr()
    need = int(load().tp_cos_emb_workspace_size(a.P, a.B, a.F, a.D))
    ws = torch.empty(max(need, 1), dtype=torch.uint8, device=weight.device)
    a.workspace, a.workspace_bytes = ws.data_ptr(), need
    check(load().tp_cos_emb_backward(ctypes.byref(a), _stream()), 'tp_cos_emb_backward')
    del keep
    return dweight, dbias, daw, dab


def tabpack_input(x_num: Tensor | None, x_cat: Tensor | None, cat_offsets: Tensor, width: int,
                  dtype: torch.dtype, row_index: Tensor | None = None, *, out: Tensor | None = None,
                  col0: int = 0) -> Tensor:
    """[x_num | one-hot(x_cat)] in `dtype`, zero-padded to `width` columns; leading dimensions
    of the inputs are kept, or with `row_index` (any shape, int64) output row r is built from
    dataset row row_index[r] and the output takes row_index's shape; see `tp_tabpack_input`.
    With `out` (contiguous, last dimension `width`) the columns from `col0` on are written into
    it and the columns before are left as they are."""
    ref = x_num if x_num is not None else x_cat
    ri = None if row_index is None else _cuda('row_index', row_index).to(torch.int64).contiguous()
    lead = ref.shape[:-1] if ri is None else ri.shape
    rows = ref[..., 0].numel() if ri is None else ri.numel()
    xn = None if x_num is None else _cuda('x_num', x_num).to(torch.float32).contiguous()
    xc = None if x_cat is None else _cuda('x_cat', x_cat).to(torch.int64).contiguous()
    if out is None:
        out = torch.empty(*lead, width, dtype=dtype, device=ref.device)
    elif (out.dtype != dtype or out.shape[-1] != width or not out.is_contiguous()
          or out.numel() != rows * width):
        raise ValueError('out must be a contiguous tensor of the rows x width output')
    a = _lib.InputArgs(rows=rows, n_num=0 if xn is None else xn.shape[-1], n_cat=0 if xc is None else xc.shape[-1],
                       x_num=_ptr(xn), x_cat=_ptr(xc), row_index=_ptr(ri), cat_offsets=cat_offsets.data_ptr(),
                       out=out.data_ptr(),
                       out_ld=width, out_dtype=TP_DTYPE_BF16 if dtype == torch.bfloat16 else TP_DTYPE_F32,
                       out_col0=int(col0))
    check(load().tp_tabpack_input(ctypes.byref(a), _stream()), 'tp_tabpack_input')
    return out


def weight_cast(src: Tensor, dst: Tensor, *, out_features: Tensor | None = None, in_features: Tensor | None = None,
                n_blocks: Tensor | None = None, block_index: int = 0, src_cols: int | None = None) -> Tensor:
    """Write bf16(src) into `dst` (P, dst_rows, dst_cols) over each active member's rows
    r < out_features[m], zero beyond in_features[m]; other rows of `dst` keep their contents
    (see `tp_weight_cast`).  `src_cols` takes only the first columns of each source row.
    Returns `dst`."""
    src = _cuda('src', src, torch.float32)
    dst = _cuda('dst', dst, torch.bfloat16)
    if not src.is_contiguous() or not dst.is_contiguous():
        raise ValueError('weight_cast needs contiguous tensors')
    P, R, ld = src.shape
    C = ld if src_cols is None else int(src_cols)
    if dst.shape[0] != P:
        raise ValueError('src and dst differ in their pack size')
    outf, inf, nb = (_i32(n, t) for n, t in (('out_features', out_features), ('in_features', in_features),
                                             ('n_blocks', n_blocks)))
    a = _lib.WeightCastArgs(P=P, src_rows=R, src_cols=C, src_ld=ld, dst_rows=dst.shape[1], dst_cols=dst.shape[2],
                            out_features=_ptr(outf), in_features=_ptr(inf), n_blocks=_ptr(nb),
                            block_index=block_index, src=src.data_ptr(), dst=dst.data_ptr())
    check(load().tp_weight_cast(ctypes.byref(a), _stream()), 'tp_weight_cast')
    increment_version(dst)
    return dst


def weight_cast_transposed(src: Tensor, dst: Tensor, *, col0: int, ncols: int,
                           out_features: Tensor | None = None) -> Tensor:
    """dst[m, j, n] = bf16(src[m, n, col0 + j]) over each member's rows n < out_features[m]
    (zeros up to the next multiple of 8); see `tp_weight_cast_transposed`.  Returns `dst`."""
    src = _cuda('src', src, torch.float32)
    dst = _cuda('dst', dst, torch.bfloat16)
    if not src.is_contiguous() or not dst.is_contiguous():
        raise ValueError('weight_cast_transposed needs contiguous tensors')
    P, R, ld = src.shape
    if tuple(dst.shape[:2]) != (P, ncols):
        raise ValueError('dst must be (P, ncols, dst_ld)')
    outf = _i32('out_features', out_features)
    a = _lib.WeightCastTArgs(P=P, src_rows=R, src_ld=ld, col0=int(col0), ncols=int(ncols), dst_ld=dst.shape[2],
                             out_features=_ptr(outf), src=src.data_ptr(), dst=dst.data_ptr())
    check(load().tp_weight_cast_transposed(ctypes.byref(a), _stream()), 'tp_weight_cast_transposed')
    increment_version(dst)
    return dst


def _round(n: int, k: int) -> int:
    return (n + k - 1) // k * k


def _onehot_args(oh: dict) -> _lib.OneHotArgs:
    a = _lib.OneHotArgs()
    a.n_dense, a.n_cat, a.n_onehot = oh['n_dense'], oh['n_cat'], oh['n_onehot']
    a.cat_offsets = oh['cat_offsets'].data_ptr()
    a.x_cat = oh['x_cat'].data_ptr()
    a.x_cat_member_stride = oh['x_cat_member_stride']
    a.row_index = _ptr(oh.get('row_index'))
    a.row_index_member_stride = oh.get('row_index_member_stride', 0)
    a.w_onehot_t = _ptr(oh.get('w_onehot_t'))
    a.wt_ld = 0 if oh.get('w_onehot_t') is None else oh['w_onehot_t'].shape[-1]
    a.sorted_keys = _ptr(oh.get('sorted_keys'))
    a.addend = _ptr(oh.get('addend'))
    a.addend_ld = 0 if oh.get('addend') is None else oh['addend'].shape[-1]
    return a


def onehot_linear_forward(x: Tensor, weight: Tensor, bias: Tensor | None, *, x_cat: Tensor, cat_offsets: Tensor,
                          n_dense: int, w_onehot_t: Tensor, row_index: Tensor | None = None,
                          out_features: Tensor | None = None, relu: bool = False, dropout_p: Tensor | None = None,
                          seed: int = 0, offset: int = 0, member_base: int = 0,
                          need_sort: bool = True) -> tuple[Tensor, dict]:
    """First layer over [dense | one-hot(x_cat)] with the one-hot columns gathered (bf16);
    see `tp_onehot_linear_forward`.  x: dense input (P or 1, B, max_in) bf16; weight: the bf16
    dense weight copy (P, max_out, max_in); w_onehot_t: (P, n_onehot, >= max_out) bf16.
    x_cat: (B, n_cat) shared, (P, B, n_cat) per member, or dataset rows with row_index (P, B).
    Returns (y, state) where state holds the category sort the backward needs (skipped with
    need_sort=False: a forward that no backward follows)."""
    weight = _cuda('weight', weight, torch.bfloat16)
    x = _cuda('x', x, torch.bfloat16)
    bias = _cuda('bias', bias, torch.float32)
    dropout_p = _cuda('dropout_p', dropout_p, torch.float32)
    outf = _i32('out_features', out_features)
    xc = _cuda('x_cat', x_cat, torch.int64).contiguous()
    P, max_out, _ = weight.shape
    B = x.shape[-2]
    n_cat = xc.shape[-1]
    ri = None
    if row_index is not None:
        ri = _cuda('row_index', row_index, torch.int64).contiguous()
        if ri.shape[-1] != B or (ri.ndim == 2 and ri.shape[0] not in (1, P)):
            raise ValueError('row_index must be (B,) or (P, B)')
        xcs, ris = 0, (B if ri.ndim == 2 and ri.shape[0] == P else 0)
    else:
        if xc.shape[-2] != B:
            raise ValueError('x_cat rows must match the batch')
        xcs, ris = (B if xc.ndim == 3 else 0), 0
    n_onehot = int(w_onehot_t.shape[1])
    dev = x.device
    state = {
        'n_dense': int(n_dense), 'n_cat': n_cat, 'n_onehot': n_onehot, 'cat_offsets': cat_offsets, 'x_cat': xc,
        'x_cat_member_stride': xcs, 'row_index': ri, 'row_index_member_stride': ris, 'w_onehot_t': w_onehot_t,
        'sorted_keys': torch.empty((P, n_cat, B), dtype=torch.int64, device=dev) if need_sort else None,
        'addend': torch.empty((P, B, _round(max_out, 16)), dtype=torch.float32, device=dev),
    }
    y = torch.empty((P, B, max_out), dtype=torch.bfloat16, device=dev)
    a = _linear_args(x, weight, bias, None, outf, None, 0, relu, dropout_p, seed, offset, member_base, y)
    oa = _onehot_args(state)
    check(load().tp_onehot_linear_forward(ctypes.byref(a), ctypes.byref(oa), _stream()), 'tp_onehot_linear_forward')
    state['addend'] = state['w_onehot_t'] = None  # used by the forward only
    return y, state


def onehot_linear_backward(dy: Tensor, x: Tensor, weight: Tensor, y: Tensor, state: dict, *,
                           out_features: Tensor | None = None, relu: bool = False, dropout_p: Tensor | None = None,
                           seed: int = 0, offset: int = 0, member_base: int = 0, need_dx: bool = False,
                           need_db: bool = True, dw_rows: int, db_cols: int) -> tuple[Tensor | None, Tensor, Tensor | None]:
    """Backward of `onehot_linear_forward`: (dx of the dense input or None, dw (P, dw_rows,
    n_dense + n_onehot) fp32, db fp32); see `tp_onehot_linear_backward`."""
    weight = _cuda('weight', weight, torch.bfloat16)
    dy = _cuda('dy', dy, torch.bfloat16)
    dropout_p = _cuda('dropout_p', dropout_p, torch.float32)
    outf = _i32('out_features', out_features)
    P, max_out, max_in = weight.shape
    B = x.shape[-2]
    g = torch.empty_like(dy)
    dx = torch.empty((P, B, max_in), dtype=torch.bfloat16, device=dy.device) if need_dx else None
    cols = state['n_dense'] + state['n_onehot']
    dw = torch.empty((P, dw_rows, cols), dtype=torch.float32, device=dy.device)
    db = torch.empty((P, db_cols), dtype=torch.float32, device=dy.device) if need_db else None
    ga = _lib.LinearGradArgs()
    ga.fwd = _linear_args(x, weight, None, None, outf, None, 0, relu, dropout_p, seed, offset, member_base, None)
    ga.dy, ga.y, ga.g = _ptr(dy), _ptr(y), _ptr(g)
    ga.dbias, ga.dx, ga.dw = _ptr(db), _ptr(dx), _ptr(dw)
    ga.dw_rows, ga.dw_cols, ga.db_cols = dw_rows, cols, db_cols
    oa = _onehot_args(state)
    check(load().tp_onehot_linear_backward(ctypes.byref(ga), ctypes.byref(oa), _stream()), 'tp_onehot_linear_backward')
    return dx, dw, db


def binary_roc_auc(scores: Tensor, labels: Tensor, workspace: Tensor | None = None) -> Tensor:
    """(P,) ROC AUC of each row of `scores` (P, N) fp32/fp64 against int64 labels (N,);
    see `tp_binary_roc_auc`.  The result has the scores' dtype."""
    scores = _cuda('scores', scores).contiguous()
    labels = _cuda('labels', labels, torch.int64).contiguous()
    if scores.dtype not in (torch.float32, torch.float64):
        raise TypeError('scores must be float32 or float64')
    P, N = scores.shape
    dtype = _lib.TP_DTYPE_F64 if scores.dtype == torch.float64 else _lib.TP_DTYPE_F32
    need = int(load().tp_roc_auc_workspace_size(P, N, dtype))
    if workspace is None or workspace.numel() * workspace.element_size() < need:
        workspace = torch.empty(need, dtype=torch.uint8, device=scores.device)
    out = torch.empty(P, dtype=scores.dtype, device=scores.device)
    check(load().tp_binary_roc_auc(scores.data_ptr(), labels.data_ptr(), P, N, dtype, out.data_ptr(),
                                   workspace.data_ptr(), workspace.numel() * workspace.element_size(), _stream()),
          'tp_binary_roc_auc')
    return out


def device_error() -> int:
    """Read and clear the device-side error flag (0 or TP_ETIMEOUT)."""
    return load().tp_device_error()
