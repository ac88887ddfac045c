"""Module packs whose forward and backward run on the sm_100a kernels.

Drop-in counterparts of the hot-path classes of `tabpackage.nn`
(`src/tabpackage/nn.py`): same constructors, same parameter/buffer names and
shapes (so state dicts interchange with the reference), same `pack_idx`,
`replace`, `remove`, `temporarily_select` and `load_state_dict_at` behaviour.
What changes is the arithmetic:

* `LinearPack.forward` and a whole `MLPBackbonePack.Block` (linear -> ReLU ->
  dropout) are one fused kernel launch, forward and backward, on tcgen05
  tensor cores under bf16 autocast and on CUDA cores in fp32 mode;
* ragged widths are never computed: each member's tiles stop at its own
  `in_features` / `out_features`, and padding is written as exact zeros;
* depth-varying members (`n_blocks`) are gated inside the same launch
  (inactive members pass their input through) instead of `torch.where` over a
  fully computed block;
* dropout draws a counter-based Philox4x32-10 mask keyed by
  (seed, call offset, member id, row, column) inside the epilogue, so masks are
  reproducible and independent of how members are sharded over GPUs.

There is no CPU path: calling a pack on CPU tensors raises.
"""

from __future__ import annotations

import contextlib
import enum
import itertools
import math
import weakref
from typing import Any, Final

import torch
import torch.nn as nn
from torch import Tensor

from tabpack_b200 import ops

PACK_DIM: Final = 0
BATCH_DIM: Final = 1

KWArgs = dict[str, Any]


# >>> tensor packs


class ParameterPack(nn.Parameter):
    """A trainable tensor with a leading pack dimension (`nn.py:159-163`)."""


def _mark_buffer(data) -> Tensor:
    t = data.detach() if isinstance(data, Tensor) else torch.as_tensor(data)
    t._is_buffer_pack = True  # type: ignore[attr-defined]
    return t


class _BufferPackMeta(type):
    def __instancecheck__(cls, instance):
        return isinstance(instance, Tensor) and getattr(instance, '_is_buffer_pack', False)


class BufferPack(metaclass=_BufferPackMeta):
    """Marker for non-trainable pack tensors (`nn.py:188-201`).

    `BufferPack(data)` returns `data` as a plain tensor tagged as a buffer pack, and
    `isinstance(t, BufferPack)` holds exactly for tagged tensors.
    """

    def __new__(cls, data):
        return _mark_buffer(data)


def _like(x: Tensor, data: Tensor) -> Tensor:
    if isinstance(x, nn.Parameter):
        return ParameterPack(data, requires_grad=x.requires_grad)
    return _mark_buffer(data)


def check_pack_idx(pack_idx: Tensor, pack_size: int | None) -> None:
    """`check_pack_idx` (`nn.py:116-122`)."""
    if pack_idx.dtype not in (torch.int32, torch.int64):
        raise TypeError('Indices must have the data type `torch.int32` or `torch.int64`')
    if pack_idx.ndim != 1:
        raise ValueError('Indices must be one-dimensional')
    if len(pack_idx) == 0:
        raise ValueError('Indices must not be empty')
    if pack_size is not None and len(pack_idx) > pack_size:
        raise ValueError('The number of pack indices must not exceed the pack size')


def make_complementary_pack_idx(pack_idx: Tensor, *, pack_size: int) -> Tensor:
    check_pack_idx(pack_idx, pack_size)
    mask = torch.ones(pack_size, dtype=torch.bool, device=pack_idx.device)
    mask[pack_idx] = False
    return torch.nonzero(mask)[:, 0]


def _select(x: Tensor | None, pack_idx: Tensor | None) -> Tensor | None:
    if x is None or pack_idx is None:
        return x
    return x.index_select(PACK_DIM, torch.where(pack_idx < 0, pack_idx + x.shape[PACK_DIM], pack_idx))


# >>> generic modules


class PackView(nn.Module):
    """`PackView` (`nn.py:39-99`): a 2-D input is shared by all members.

    The expansion is not materialised: packs below consume a 2-D input directly
    (the kernels read the shared rows once per member tile from L2).
    """

    def __init__(self, *, pack_size: int) -> None:
        super().__init__()
        self._pack_size = pack_size

    @property
    def pack_size(self) -> int:
        return self._pack_size

    def forward(self, x: Tensor, pack_idx: Tensor | None = None) -> Tensor:
        if pack_idx is not None:
            check_pack_idx(pack_idx, self.pack_size)
        pack_size = self.pack_size if pack_idx is None else len(pack_idx)
        if x.ndim == 2:
            return x.unsqueeze(PACK_DIM).expand(pack_size, -1, -1)
        if x.ndim != 3:
            raise ValueError('The input must have two or three dimensions')
        if not self.training:
            raise RuntimeError('Three-dimensional input requires training mode')
        if x.shape[PACK_DIM] != pack_size:
            raise ValueError('The pack dimension of the input must match the selected pack size')
        return x


class _PackBuffers(dict):
    """Buffer dict of module packs: a buffer pack stays a buffer pack when it is
    reassigned (e.g. by `Module.to`), like `_ModulePackBuffers` (`nn.py:259-279`)."""

    def __setitem__(self, key, value):
        cur = self.get(key)
        if value is not None and cur is not None and getattr(cur, '_is_buffer_pack', False):
            value._is_buffer_pack = True
        super().__setitem__(key, value)


class ModulePack(nn.Module):
    """Base class of module packs (`nn.py:282-531`)."""

    def __init__(self, *args, **kwargs) -> None:
        super().__init__(*args, **kwargs)
        self._buffers = _PackBuffers()

    @property
    def pack_size(self) -> int:  # pragma: no cover - abstract
        raise NotImplementedError

    def try_get_pack_size(self) -> int | None:
        try:
            return self.pack_size
        except RuntimeError:
            return None

    def _pack_tensors(self):
        for name, x in itertools.chain(self.named_parameters(), self.named_buffers()):
            if isinstance(x, ParameterPack) or getattr(x, '_is_buffer_pack', False):
                yield name, x

    def _owner(self, name: str):
        if '.' in name:
            sub, attr = name.rsplit('.', 1)
            return self.get_submodule(sub), attr
        return self, name

    def load_state_dict_at(self, state_dict: dict[str, Tensor], *, pack_idx: Tensor,
                           state_dict_idx: Tensor | None = None) -> None:
        """`ModulePack.load_state_dict_at` (`nn.py:334-397`)."""
        check_pack_idx(pack_idx, self.pack_size)
        if self.state_dict().keys() != state_dict.keys():
            raise ValueError('The state dictionary has missing or unexpected keys for this module')
        with torch.no_grad():
            for name, x in self._pack_tensors():
                if name not in state_dict:
                    continue
                v = state_dict[name]
                if v.ndim != x.ndim or v.shape[1:] != x.shape[1:]:
                    raise ValueError('The source and destination tensors have incompatible shapes')
                x[pack_idx] = (v if state_dict_idx is None else v[state_dict_idx]).to(x.device, x.dtype)
        for m in self.modules():
            if isinstance(m, MLPBackbonePack):
                m._invalidate()

    def remove(self, *, pack_idx: Tensor) -> dict:
        """`ModulePack.remove` (`nn.py:417-463`)."""
        check_pack_idx(pack_idx, self.pack_size)
        if len(pack_idx) != len(torch.unique(pack_idx)):
            raise ValueError('Pack indices to remove must be unique')
        keep = None
        mapping = {}
        for name, x in list(self._pack_tensors()):
            if keep is None:
                keep = make_complementary_pack_idx(pack_idx, pack_size=x.shape[PACK_DIM])
            owner, attr = self._owner(name)
            new_x = _like(x, x.data[keep])
            if isinstance(x, nn.Parameter):
                setattr(owner, attr, new_x)
                mapping[x] = new_x
            else:
                owner.register_buffer(attr, new_x, persistent=attr not in owner._non_persistent_buffers_set)
        for m in self.modules():
            if isinstance(m, PackView):
                m._pack_size -= len(pack_idx)
            if isinstance(m, MLPBackbonePack):
                m._invalidate()
        return mapping

    @contextlib.contextmanager
    def temporarily_select(self, *, pack_idx: Tensor):
        """`ModulePack.temporarily_select` (`nn.py:469-531`)."""
        check_pack_idx(pack_idx, None)
        if any(m.training for m in self.modules()):
            raise RuntimeError('The module and all its submodules must be in evaluation mode to use this method')
        saved, views = [], []
        try:
            for name, x in list(self._pack_tensors()):
                owner, attr = self._owner(name)
                setattr(owner, attr, _like(x, x.data[pack_idx]))
                saved.append((owner, attr, x))
            for m in self.modules():
                if isinstance(m, PackView):
                    views.append((m, m.pack_size))
                    m._pack_size = len(pack_idx)
                if isinstance(m, MLPBackbonePack):
                    m._invalidate()
            yield
        finally:
            for owner, attr, x in saved:
                setattr(owner, attr, x)
            for m, n in views:
                m._pack_size = n
            for m in self.modules():
                if isinstance(m, MLPBackbonePack):
                    m._invalidate()


def _positive_int_pack(value, max_value, *, pack_size):
    """`_prepare_positive_integer_pack` (`nn.py:554-587`)."""
    if isinstance(value, list):
        if len(value) != pack_size:
            raise ValueError('The number of per-member hyperparameter values does not match the pack size')
        if not all(v > 0 for v in value):
            raise ValueError('All values must be positive')
        if max_value is None:
            max_value = max(value)
        elif not all(v <= max_value for v in value):
            raise ValueError('Values must not exceed `max_value`')
        return _mark_buffer(torch.tensor(value)), max_value
    if value <= 0:
        raise ValueError('The value must be positive')
    if max_value is None:
        max_value = value
    elif max_value != value:
        raise ValueError('The configured maximum must equal the shared value')
    return None, max_value


# >>> compute plumbing shared by LinearPack and Block


class _DropoutStream:
    """Philox key and call counter of one module (masks are reproducible given
    the module's seed, its training-forward count and the member ids)."""

    def __init__(self) -> None:
        self.seed = int(torch.randint(0, 2**62, (1,), generator=None).item())
        self.calls = 0
        self.member_base = 0

    def next_offset(self, stride: int = 1) -> int:
        off = self.calls * stride
        self.calls += 1
        return off


def _reusable(buf: Tensor | None, shape, dtype: torch.dtype, device) -> bool:
    """True when `buf` has this geometry and nothing but its cache holds it (a pending
    backward that saved it would see an in-place refresh)."""
    if buf is None or tuple(buf.shape) != tuple(shape) or buf.dtype != dtype or buf.device != device:
        return False
    use_count = getattr(buf, '_use_count', None)
    return use_count is not None and use_count() == 1


class _WeightCache:
    """bf16 copy of an fp32 weight pack, refreshed when the weight changes (optimizer steps
    and in-place updates bump the parameter's version counter).

    With the layer's widths the copy comes from `tp_weight_cast`: one pass that reads only
    each active member's rows and columns; the other rows of the copy keep earlier (finite)
    contents, which the GEMMs only multiply by exact zeros.  The copy is refreshed in place
    unless something else (a pending backward) still holds it."""

    def __init__(self) -> None:
        self.key = None
        self.value = None

    @staticmethod
    def _tag(t):
        return None if t is None else (t.data_ptr(), t._version, tuple(t.shape))

    def get(self, w: Tensor, dtype: torch.dtype, cols: int, rows: int | None = None, widths=None) -> Tensor:
        rows = w.shape[-2] if rows is None else rows
        if w.dtype == dtype and w.shape[-1] == cols and w.shape[-2] == rows:
            return w.detach()
        out_f, in_f, nb, bi = widths if widths is not None else (None, None, None, 0)
        key = (w.data_ptr(), w._version, dtype, cols, rows, tuple(w.shape),
               self._tag(out_f), self._tag(in_f), self._tag(nb), bi)
        if self.key != key:
            self.key = None
            if dtype == torch.bfloat16 and w.dtype == torch.float32 and w.is_cuda and w.is_contiguous():
                shape = (w.shape[0], rows, cols)
                buf = self.value
                if not _reusable(buf, shape, dtype, w.device):
                    buf = torch.zeros(shape, dtype=dtype, device=w.device)
                self.value = None
                ops.weight_cast(w.detach(), buf, out_features=out_f, in_features=in_f, n_blocks=nb, block_index=bi)
                self.value = buf
            else:
                wd = w.detach().to(dtype)
                if cols != w.shape[-1] or rows != w.shape[-2]:
                    wd = nn.functional.pad(wd, (0, cols - w.shape[-1], 0, rows - w.shape[-2]))
                self.value = wd.contiguous()
            self.key = key
        return self.value

    def begin_update(self, w: Tensor) -> Tensor | None:
        """The bf16 copy for an optimizer step to refresh in the pass that updates `w`: the copy
        when it holds `w`'s current values (its key is at `w`'s present version) and nothing but
        this cache holds it; else None, and the next forward casts again."""
        key, buf = self.key, self.value
        if key is None or buf is None or key[0] != w.data_ptr() or key[1] != w._version or key[2] != torch.bfloat16:
            return None
        if buf is w or not _reusable(buf, tuple(buf.shape), torch.bfloat16, w.device):
            return None
        return buf

    def end_update(self, w: Tensor, buf: Tensor) -> None:
        """After a step that wrote bf16 of `w`'s new values into `buf` (`begin_update`): the copy
        is current at `w`'s new version."""
        if self.value is buf and self.key is not None:
            self.key = (self.key[0], w._version) + tuple(self.key[2:])


# id(parameter) -> (weak parameter, weak cache): the bf16 compute-copy cache of a LinearPack's
# weight, so that an optimizer step can write the refreshed copy in the same pass as the fp32
# weights.  Keyed by id (tensors do not hash by value); an entry leaves when its parameter dies.
_BF16_CACHES: dict[int, tuple] = {}


def _register_bf16_cache(w: Tensor, cache: _WeightCache) -> None:
    key = id(w)

    def gone(ref, key=key):
        entry = _BF16_CACHES.get(key)
        if entry is not None and entry[0] is ref:
            del _BF16_CACHES[key]

    _BF16_CACHES[key] = (weakref.ref(w, gone), weakref.ref(cache))


def bf16_copy_cache(w: Tensor) -> _WeightCache | None:
    """The bf16 compute-copy cache registered for parameter `w`, if any."""
    entry = _BF16_CACHES.get(id(w))
    if entry is None or entry[0]() is not w:
        return None
    return entry[1]()


class _OneHotWeightCache:
    """bf16 copies of a first-layer weight (P, max_out, n_dense + n_onehot) for the gathered
    one-hot path: the dense columns (tp_weight_cast, padded to `dense_cols`) and the one-hot
    columns transposed, (P, n_onehot, rows) (tp_weight_cast_transposed), refreshed when the
    weight or its widths change."""

    def __init__(self) -> None:
        self.key = None
        self.dense = None
        self.onehot_t = None

    def get(self, w: Tensor, out_f: Tensor | None, n_dense: int, rows: int, dense_cols: int) -> tuple[Tensor, Tensor]:
        key = (w.data_ptr(), w._version, tuple(w.shape), _WeightCache._tag(out_f), n_dense, rows, dense_cols)
        if self.key != key:
            self.key = None
            P, _, C = w.shape
            n_onehot = C - n_dense
            dense, wt = self.dense, self.onehot_t
            self.dense = self.onehot_t = None
            if not _reusable(dense, (P, rows, dense_cols), torch.bfloat16, w.device):
                dense = torch.zeros((P, rows, dense_cols), dtype=torch.bfloat16, device=w.device)
            if not _reusable(wt, (P, n_onehot, rows), torch.bfloat16, w.device):
                wt = torch.empty((P, n_onehot, rows), dtype=torch.bfloat16, device=w.device)
            src = w.detach()
            if n_dense > 0:
                ops.weight_cast(src, dense, out_features=out_f, src_cols=n_dense)
            ops.weight_cast_transposed(src, wt, col0=n_dense, ncols=n_onehot, out_features=out_f)
            self.dense, self.onehot_t = dense, wt
            self.key = key
        return self.dense, self.onehot_t


def _compute_dtype(x: Tensor) -> torch.dtype:
    if torch.is_autocast_enabled(x.device.type) and torch.get_autocast_dtype(x.device.type) == torch.bfloat16:
        return torch.bfloat16
    if x.dtype == torch.bfloat16:
        return torch.bfloat16
    return torch.float32


def _round8(n: int) -> int:
    return (n + 7) // 8 * 8


def _weight_gradient_buffer(slot: dict, shape: tuple, device, key) -> Tensor:
    """The weight gradient's buffer for a layer whose gradients the trainer owns: the previous
    step's storage again once nothing holds that step's gradient any more (its padding and the
    depth-inactive members' blocks are still zero, so the kernel writes the active blocks only),
    else a zeroed new one.  `key` (widths and depths) must match the previous step's."""
    st, ref = slot.get('storage'), slot.get('ref')
    if (st is not None and slot.get('shape') == shape and slot.get('key') == key and st.device == device
            and (ref is None or ref() is None)):
        return torch.empty(0, dtype=torch.float32, device=device).set_(st, 0, shape)
    t = torch.zeros(shape, dtype=torch.float32, device=device)
    slot.update(storage=t.untyped_storage(), shape=shape, key=key, ref=None)
    return t


def _activation_buffer(slot: dict, shape: tuple, dtype: torch.dtype, device, key) -> Tensor | None:
    """The output buffer of a layer whose activations the trainer owns: the previous call's
    storage again once nothing else holds it (a finished step's autograd graph has released
    it), else a zeroed new one.  Its padding columns stay zero (the kernels then write only
    the members' column tiles, `y_pad_zero`); `key` (widths and depths) must match the
    previous call's.  None (no reuse) where storage use counts are not available."""
    use_count = getattr(torch._C, '_storage_Use_Count', None)
    if use_count is None:
        return None
    st = slot.get('storage')
    if (st is not None and slot.get('shape') == shape and slot.get('dtype') == dtype and slot.get('key') == key
            and st.device == device and use_count(st._cdata) == 1):
        return torch.empty(0, dtype=dtype, device=device).set_(st, 0, shape)
    t = torch.zeros(shape, dtype=dtype, device=device)
    slot.update(storage=t.untyped_storage(), shape=shape, dtype=dtype, key=key)
    return t


class _PackedLinearFn(torch.autograd.Function):
    """One fused launch forward, three in backward (activation grad + bias grad,
    dgrad, wgrad); `cfg` carries the non-tensor configuration."""

    @staticmethod
    def forward(ctx, x, weight, bias, w_compute, b_compute, cfg):
        y_buf = None
        if cfg.get('y_slot') is not None:
            rows = cfg['kw']['row_index'].shape[1] if 'row_index' in cfg['kw'] else x.shape[-2]
            y_buf = _activation_buffer(cfg['y_slot'], (w_compute.shape[0], rows, w_compute.shape[1]), x.dtype,
                                       x.device, cfg['y_key'])
        y = ops.linear_forward(x, w_compute, b_compute, **cfg['kw'], y=y_buf)
        ctx.cfg = cfg
        ctx.x_shape = x.shape
        ctx.save_for_backward(x, w_compute, y if (cfg['kw']['relu'] or cfg['kw']['dropout_p'] is not None) else None)
        return y

    @staticmethod
    def backward(ctx, dy):
        x, w_compute, y = ctx.saved_tensors
        cfg = ctx.cfg
        need_dx, need_dw, need_db = ctx.needs_input_grad[0], ctx.needs_input_grad[1], ctx.needs_input_grad[2]
        slot = cfg.get('dw_slot')
        dw_out = None
        if slot is not None and need_dw:
            dw_out = _weight_gradient_buffer(slot, tuple(cfg['w_shape']), dy.device, cfg['dw_key'])
        dx_out = None
        if cfg.get('dx_slot') is not None and need_dx and len(ctx.x_shape) == 3 and x.shape == ctx.x_shape:
            dx_out = _activation_buffer(cfg['dx_slot'], tuple(x.shape), w_compute.dtype, dy.device, cfg['x_key'])
        dx, dw, db = ops.linear_backward(
            dy.contiguous().to(w_compute.dtype), x, w_compute, y, **cfg['kw'],
            need_dx=need_dx, need_dw=need_dw, need_db=need_db,
            dw_shape=cfg['w_shape'][1:], db_cols=cfg['w_shape'][1], dx_cols=cfg.get('dx_cols', 0),
            dw_out=dw_out, dw_pad_zero=dw_out is not None, dx_out=dx_out)
        if dw_out is not None:
            slot['ref'] = weakref.ref(dw)  # reusable once the optimizer has dropped this gradient
        if dx is not None:
            if len(ctx.x_shape) == 2:
                dx = dx.sum(PACK_DIM)
            if dx.shape[-1] != ctx.x_shape[-1]:  # the gradient of this function's (padded) input
                dx = dx[..., : ctx.x_shape[-1]]
        return dx, dw, db, None, None, None


def packed_linear(x: Tensor, weight: Tensor, bias: Tensor | None, *, in_features=None, out_features=None,
                  n_blocks=None, block_index=0, relu=False, dropout_p=None, seed=0, offset=0,
                  member_base=0, cache: _WeightCache | None = None, dx_cols: int = 0,
                  row_index: Tensor | None = None, dw_slot: dict | None = None,
                  y_slot: dict | None = None) -> Tensor:
    """Functional form of the fused packed linear layer (see module docstring).  `dx_cols` > 0:
    the input's gradient is needed in its first dx_cols columns only (zeros beyond).
    `row_index` (pack_size, batch): `x` is a (rows, in) table and member m's input row b is
    x[row_index[m, b]], gathered by the GEMMs' operand loads (the table takes no gradient).
    `dw_slot` / `y_slot`: storage that the weight gradient / the output reuse from the
    previous call (a trainer that owns them; the output only while autograd records)."""
    if not x.is_cuda:
        raise RuntimeError('tabpack_b200 packs run on CUDA devices only')
    dtype = _compute_dtype(x)
    in_cols = x.shape[-1]
    cols = _round8(in_cols) if dtype == torch.bfloat16 else in_cols
    # bf16 inputs may arrive already padded to the 8-column multiple the tensor-core path uses
    if weight.shape[-1] != in_cols and not (dtype == torch.bfloat16 and in_cols == _round8(weight.shape[-1])):
        raise ValueError('The number of input features must be equal to the maximum supported number of features')
    xc = x.to(dtype)
    if cols != in_cols:
        xc = nn.functional.pad(xc, (0, cols - in_cols))
    xc = xc.contiguous()
    # bf16 output widths that are not a multiple of 8 (e.g. a 1-wide output head) run on the
    # tensor cores over zero-padded weight rows and bias; the padded columns are sliced off
    max_out = weight.shape[-2]
    rows = _round8(max_out) if dtype == torch.bfloat16 else max_out
    wc = (cache or _WeightCache()).get(weight, dtype, cols, rows,
                                       widths=(out_features, in_features, n_blocks, block_index))
    bc = bias
    if bias is not None and rows != max_out:
        bc = nn.functional.pad(bias.detach(), (0, rows - max_out))
    kw = dict(in_features=in_features, out_features=out_features, n_blocks=n_blocks, block_index=block_index,
              relu=relu, dropout_p=dropout_p, seed=seed, offset=offset, member_base=member_base)
    if row_index is not None:
        if x.requires_grad:
            raise ValueError('a gathered input (a table) takes no gradient')
        kw['row_index'] = row_index
    cfg = {'kw': kw, 'w_shape': tuple(weight.shape), 'in_cols': in_cols, 'dx_cols': int(dx_cols)}
    if dw_slot is not None:
        tag = lambda t: None if t is None else (t.data_ptr(), t._version, tuple(t.shape))  # noqa: E731
        cfg['dw_slot'] = dw_slot
        cfg['dw_key'] = (tag(out_features), tag(in_features), tag(n_blocks), int(block_index))
    if y_slot is not None and dtype == torch.bfloat16 and torch.is_grad_enabled():
        tag = lambda t: None if t is None else (t.data_ptr(), t._version, tuple(t.shape))  # noqa: E731
        key = (tag(out_features), tag(in_features), tag(n_blocks), int(block_index))
        if rows == max_out:
            cfg['y_slot'], cfg['y_key'] = y_slot.setdefault('y', {}), key
        if x.ndim == 3 and cols == in_cols and row_index is None and not dx_cols:
            cfg['dx_slot'], cfg['x_key'] = y_slot.setdefault('dx', {}), key
    with torch.autocast(x.device.type, enabled=False):
        y = _PackedLinearFn.apply(xc, weight, bias, wc, bc, cfg)
    return y if rows == max_out else y[..., :max_out]


class _OneHotLinearFn(torch.autograd.Function):
    """First layer with gathered one-hot columns: one sort + gather + tensor-core launch
    forward (`tp_onehot_linear_forward`), activation grad + dense dgrad/wgrad + one-hot
    segmented sums backward (`tp_onehot_linear_backward`)."""

    @staticmethod
    def forward(ctx, x, weight, bias, w_dense, w_t, b_compute, cfg):
        kw = cfg['kw']
        y, state = ops.onehot_linear_forward(x, w_dense, b_compute, w_onehot_t=w_t, **cfg['onehot'], **kw,
                                             need_sort=cfg['need_sort'])
        ctx.cfg, ctx.state = cfg, state
        ctx.save_for_backward(x, w_dense, y)
        return y

    @staticmethod
    def backward(ctx, dy):
        x, w_dense, y = ctx.saved_tensors
        cfg = ctx.cfg
        need_dx, need_dw, need_db = ctx.needs_input_grad[0], ctx.needs_input_grad[1], ctx.needs_input_grad[2]
        dx, dw, db = ops.onehot_linear_backward(
            dy.contiguous().to(torch.bfloat16), x, w_dense, y, ctx.state, **cfg['kw'], need_dx=need_dx,
            need_db=need_db, dw_rows=cfg['w_shape'][1], db_cols=cfg['w_shape'][1])
        if dx is not None and x.ndim == 2:
            dx = dx.sum(PACK_DIM)
        return dx, (dw if need_dw else None), db, None, None, None, None


def _onehot_linear_call(linear: LinearPack, x: Tensor, onehot: dict, *, relu, dropout, stream,
                        offset_stride: int = 1, offset_add: int = 0) -> Tensor:
    """The first layer over [x | one-hot(categories)] with the one-hot columns gathered from
    the weight instead of multiplied (bf16 tensor-core path).  `x`: the dense columns (the
    numerical features or their embeddings), (B, n_dense) shared or (P, B, n_dense);
    `onehot`: x_cat / cat_offsets / n_dense / row_index as `ops.onehot_linear_forward` takes
    them."""
    w, b = linear.weight, linear.bias
    outf = _widths_cached(linear, 'out', linear.out_features)
    member_base = 0 if stream is None else stream.member_base
    seed = offset = 0
    if dropout is not None and stream is not None:
        seed = stream.seed
        offset = stream.next_offset(offset_stride) + offset_add
    max_out = w.shape[-2]
    rows = _round8(max_out)
    n_dense = int(onehot['n_dense'])
    dense_cols = _round8(max(n_dense, 1))
    xd = x.to(torch.bfloat16)
    if xd.shape[-1] != dense_cols:
        xd = nn.functional.pad(xd, (0, dense_cols - xd.shape[-1]))
    xd = xd.contiguous()
    cache = linear.__dict__.setdefault('_onehot_cache', _OneHotWeightCache())
    wd, wt = cache.get(w, outf, n_dense, rows, dense_cols)
    bc = b
    if b is not None and rows != max_out:
        bc = nn.functional.pad(b.detach(), (0, rows - max_out))
    kw = dict(out_features=outf, relu=relu, dropout_p=dropout, seed=seed, offset=offset, member_base=member_base)
    # the category sort serves the backward only
    need_sort = torch.is_grad_enabled() and any(t is not None and t.requires_grad for t in (xd, w, b))
    cfg = {'kw': kw, 'onehot': onehot, 'w_shape': tuple(w.shape), 'need_sort': need_sort}
    with torch.autocast(x.device.type, enabled=False):
        y = _OneHotLinearFn.apply(xd, w, b, wd, wt, bc, cfg)
    return y if rows == max_out else y[..., :max_out]


def _widths(buf: Tensor | None) -> Tensor | None:
    return None if buf is None else buf.to(torch.int32)


def _widths_cached(module: nn.Module, name: str, buf: Tensor | None) -> Tensor | None:
    """int32 copy of a width buffer, kept while the buffer is unchanged: one tensor per buffer
    state, so caches may key on its identity."""
    if buf is None:
        return None
    cache = module.__dict__.setdefault('_widths_i32', {})
    key = (buf.data_ptr(), buf._version, buf.dtype, tuple(buf.shape))
    hit = cache.get(name)
    if hit is None or hit[0] != key:
        hit = (key, buf.to(torch.int32))
        cache[name] = hit
    return hit[1]


# >>> module packs


class LinearPack(ModulePack):
    """`LinearPack` (`nn.py:598-816`) on the fused ragged grouped GEMM."""

    # Set by a training loop that owns the gradients (PackTrainer): each backward writes the
    # weight gradient into the previous step's storage once nothing holds that step's gradient
    # (the optimizer has stepped and the gradients were set to None); its padding and the
    # depth-inactive members' blocks are still zero there, so only the active blocks are
    # written.  Code that modifies a weight gradient's padding in place must leave it off.
    reuse_weight_gradient = False
    # When set (a trainer whose layer outputs feed only the next layer), a training-mode
    # forward writes its output into the previous step's storage once autograd has released it;
    # the padding columns stay zero there, so only the members' column tiles are written.
    reuse_activation_buffer = False

    def __init__(self, in_features, out_features, bias: bool = True, *, max_in_features=None,
                 max_out_features=None, pack_size: int, dtype=None, device=None) -> None:
        if pack_size <= 0:
            raise ValueError('The pack size must be positive')
        fk = {'dtype': dtype, 'device': device}
        inb, max_in = _positive_int_pack(in_features, max_in_features, pack_size=pack_size)
        outb, max_out = _positive_int_pack(out_features, max_out_features, pack_size=pack_size)
        super().__init__()
        self.register_buffer('in_features', None if inb is None else _mark_buffer(inb.to(device)))
        self.register_buffer('out_features', None if outb is None else _mark_buffer(outb.to(device)))
        self.weight = ParameterPack(torch.empty(pack_size, max_out, max_in, **fk))
        self.bias = ParameterPack(torch.empty(pack_size, max_out, **fk)) if bias else None
        self._cache = _WeightCache()
        _register_bf16_cache(self.weight, self._cache)
        self._dw_slot = {}
        self._y_slot = {}
        self.reset_parameters()

    @property
    def max_in_features(self) -> int:
        return self.weight.shape[-1]

    @property
    def max_out_features(self) -> int:
        return self.weight.shape[-2]

    @property
    def pack_size(self) -> int:
        return self.weight.shape[PACK_DIM]

    def reset_parameters(self, *, pack_idx: Tensor | None = None) -> None:
        """Per-member U(-1/sqrt(in_i), 1/sqrt(in_i)) (`nn.py:702-747`)."""
        if pack_idx is not None:
            check_pack_idx(pack_idx, self.pack_size)
        n = self.pack_size if pack_idx is None else len(pack_idx)
        if self.in_features is None:
            bound = torch.full((n,), self.max_in_features ** -0.5)
        else:
            bound = _select(self.in_features, pack_idx).float().rsqrt().cpu()
        for p in (self.weight, self.bias):
            if p is None:
                continue
            shape = (n, *p.shape[1:])
            bnd = bound.view(-1, *([1] * (p.ndim - 1))).to(p.device, p.dtype)
            u = torch.rand(shape, dtype=p.dtype, device=p.device)
            init = torch.lerp(-bnd.expand(shape), bnd.expand(shape), u)
            with torch.no_grad():
                if pack_idx is None:
                    p.copy_(init)
                else:
                    p[pack_idx] = init

    def replace(self, *, pack_idx: Tensor, in_features: list[int] | None = None,
                out_features: list[int] | None = None) -> None:
        """`LinearPack.replace` (`nn.py:749-790`)."""
        check_pack_idx(pack_idx, self.pack_size)
        updates = []
        for buf, mx, vals in ((self.in_features, self.max_in_features, in_features),
                              (self.out_features, self.max_out_features, out_features)):
            if vals is None:
                continue
            if len(vals) != len(pack_idx):
                raise ValueError('Each provided hyperparameter list must contain one value for each selected pack member')
            if buf is None:
                raise RuntimeError('Cannot replace feature counts that are shared by all pack members')
            if not all(0 < v <= mx for v in vals):
                raise ValueError('Feature counts must be positive and must not exceed the allocated maximum')
            updates.append((buf, torch.tensor(vals, dtype=buf.dtype, device=buf.device)))
        for buf, v in updates:
            buf[pack_idx] = v
        self.reset_parameters(pack_idx=pack_idx)

    def forward(self, x: Tensor, pack_idx: Tensor | None = None) -> Tensor:
        if x.ndim != 3:
            raise ValueError('The input must have three dimensions')
        if x.shape[-1] != self.max_in_features:
            raise ValueError('The number of input features must be equal to the maximum supported number of features')
        return _linear_call(self, x, pack_idx, relu=False, dropout=None, stream=None, n_blocks=None, block_index=0)


def _linear_call(linear: LinearPack, x: Tensor, pack_idx, *, relu, dropout, stream, n_blocks, block_index,
                 offset_stride: int = 1, offset_add: int = 0, dx_cols: int = 0, row_index: Tensor | None = None,
                 narrow: tuple[int | None, int | None] | None = None):
    """`narrow` = (out, in): with a member selection, the selected weights are cut to their
    first `out` rows / `in` columns (None: all), so the selected members' layer runs with
    those maximum widths (they must cover every selected member's widths)."""
    w, b = linear.weight, linear.bias
    if row_index is not None and pack_idx is not None:
        raise ValueError('a gathered input runs on the whole pack')
    inf, outf = linear.in_features, linear.out_features
    member_base = 0 if stream is None else stream.member_base
    if pack_idx is not None:
        check_pack_idx(pack_idx, linear.pack_size)
        # (n_blocks comes from the backbone already selected to the same members)
        w, b, inf, outf = (_select(t, pack_idx) for t in (w, b, inf, outf))
        if dropout is not None:
            raise NotImplementedError('pack_idx with training-mode dropout is not supported; '
                                      'use temporarily_select or remove')
        if narrow is not None:
            n_out, n_in = narrow
            if n_out is not None:
                w = w[:, :n_out]
                b = None if b is None else b[:, :n_out].contiguous()
            if n_in is not None:
                w = w[:, :, :n_in]
            w = w.contiguous()
    elif narrow is not None:
        raise ValueError('narrowed widths need a member selection')
    if row_index is not None:
        pass  # x is the gathered table
    elif x.ndim == 3 and x.shape[0] == 1 and w.shape[0] != 1:
        x = x[0]
    elif x.ndim == 3 and x.stride(0) == 0:
        x = x[0]
    seed = offset = 0
    if dropout is not None and stream is not None:
        seed = stream.seed
        offset = stream.next_offset(offset_stride) + offset_add
    if getattr(linear, 'full_width_input', False):
        inf = None  # the whole padded input width takes part (first layer of a TabPack with embeddings)
    if pack_idx is None:
        inf, outf = _widths_cached(linear, 'in', inf), _widths_cached(linear, 'out', outf)
    else:
        inf, outf = _widths(inf), _widths(outf)
    return packed_linear(x, w, b, in_features=inf, out_features=outf, n_blocks=n_blocks,
                         block_index=block_index, relu=relu, dropout_p=dropout, seed=seed, offset=offset,
                         member_base=member_base, cache=linear._cache if pack_idx is None else None,
                         dx_cols=dx_cols, row_index=row_index,
                         dw_slot=linear._dw_slot if (pack_idx is None and linear.reuse_weight_gradient) else None,
                         y_slot=linear._y_slot if (pack_idx is None and linear.reuse_activation_buffer) else None)


class DropoutPack(ModulePack):
    """`DropoutPack` (`nn.py:819-903`) with the Philox keep mask.

    Inside `MLPBackbonePack.Block` the mask is applied in the GEMM epilogue; a
    standalone `DropoutPack` applies the same mask to its input.
    """

    def __init__(self, p, *, pack_size: int) -> None:
        if isinstance(p, (int, float)):
            if not math.isfinite(p) or p < 0.0 or p >= 1.0:
                raise ValueError('The dropout probability must be finite and in [0, 1)')
        else:
            if len(p) != pack_size:
                raise ValueError('Provide one dropout probability per pack member')
            if any(not math.isfinite(v) or v < 0.0 or v >= 1.0 for v in p):
                raise ValueError('Dropout probabilities must be finite and in [0, 1)')
        super().__init__()
        if isinstance(p, (int, float)):
            self.p = float(p)
        else:
            self.register_buffer('p', _mark_buffer(torch.tensor([float(v) for v in p])))
        self._stream = _DropoutStream()

    @property
    def pack_size(self) -> int:
        if isinstance(self.p, (int, float)):
            raise RuntimeError('Cannot infer the pack size')
        return self.p.shape[PACK_DIM]

    def replace(self, *, pack_idx: Tensor, p: list[float] | None = None) -> None:
        if p is None:
            return
        if isinstance(self.p, (int, float)):
            raise RuntimeError('Cannot replace dropout probabilities when one probability is shared by all pack members')
        check_pack_idx(pack_idx, self.pack_size)
        if len(p) != len(pack_idx):
            raise ValueError('Each provided hyperparameter list must contain one value for each selected pack member')
        if any(not math.isfinite(v) or v < 0.0 or v >= 1.0 for v in p):
            raise ValueError('Dropout probabilities must be finite and in [0, 1)')
        self.p[pack_idx] = torch.tensor(p, dtype=self.p.dtype, device=self.p.device)

    def probabilities(self, pack_size: int, device) -> Tensor:
        if isinstance(self.p, (int, float)):
            return torch.full((pack_size,), float(self.p), device=device)
        return self.p.to(device=device, dtype=torch.float32)

    def forward(self, x: Tensor, pack_idx: Tensor | None = None) -> Tensor:
        if not self.training:
            return x
        if not x.is_cuda:
            raise RuntimeError('tabpack_b200 packs run on CUDA devices only')
        p = self.probabilities(x.shape[0], x.device) if pack_idx is None else _select(self.p, pack_idx).float()
        if x.ndim != 3:
            raise ValueError('DropoutPack expects (pack, batch, features) inputs')
        mask = ops.dropout_mask(seed=self._stream.seed, offset=self._stream.next_offset(),
                                member_base=self._stream.member_base, p=p.contiguous(),
                                rows=x.shape[1], cols=x.shape[2])
        scale = (1.0 / (1.0 - p)).to(x.dtype)
        return x * mask.to(x.dtype) * scale.view(-1, 1, 1)


class MLPBackbonePack(ModulePack):
    """`MLPBackbonePack` (`nn.py:996-1428`): each block is one fused launch."""

    class Block(ModulePack):
        """`MLPBackbonePack.Block` (`nn.py:1015-1079`): linear -> ReLU -> dropout, fused."""

        def __init__(self, *, activation: KWArgs, dropout, pack_size: int, **linear_kwargs) -> None:
            super().__init__()
            self.linear = LinearPack(pack_size=pack_size, **linear_kwargs)
            act = dict(activation)
            cls = act.pop('type')
            self.activation = cls(**act) if not issubclass(cls, ModulePack) else cls(pack_size=pack_size, **act)
            self.dropout = DropoutPack(dropout, pack_size=pack_size)

        @property
        def pack_size(self) -> int:
            return self.linear.pack_size

        def replace(self, *, pack_idx: Tensor, in_features=None, out_features=None, activation=None,
                    dropout=None) -> None:
            self.linear.replace(pack_idx=pack_idx, in_features=in_features, out_features=out_features)
            if activation is not None:
                raise RuntimeError('The activation module does not support member replacement')
            self.dropout.replace(pack_idx=pack_idx, p=dropout)

        def _fused_relu(self) -> bool:
            if isinstance(self.activation, nn.ReLU):
                return True
            if isinstance(self.activation, nn.Identity):
                return False
            raise NotImplementedError(f'fused blocks support ReLU or Identity, not {type(self.activation)}')

        def forward(self, x: Tensor, pack_idx: Tensor | None = None, *, n_blocks: Tensor | None = None,
                    block_index: int = 0, stream: _DropoutStream | None = None, offset_stride: int = 1,
                    onehot: dict | None = None, dx_cols: int = 0, row_index: Tensor | None = None,
                    narrow: tuple[int | None, int | None] | None = None) -> Tensor:
            drop = None
            if self.training:
                drop = self.dropout.probabilities(self.pack_size, x.device).contiguous()
                if isinstance(self.dropout.p, float) and self.dropout.p == 0.0:
                    drop = None
            if onehot is not None:
                return _onehot_linear_call(self.linear, x, onehot, relu=self._fused_relu(), dropout=drop,
                                           stream=stream or self.dropout._stream, offset_stride=offset_stride,
                                           offset_add=block_index)
            return _linear_call(self.linear, x, pack_idx, relu=self._fused_relu(), dropout=drop,
                                stream=stream or self.dropout._stream, n_blocks=n_blocks, block_index=block_index,
                                offset_stride=offset_stride, offset_add=block_index, dx_cols=dx_cols,
                                row_index=row_index, narrow=narrow)

    @enum.unique
    class ForwardImpl(enum.StrEnum):
        """Both reference implementations (`nn.py:1081-1116`) map to the same
        gated kernel; the value is kept for API compatibility."""

        DENSE = enum.auto()
        INDEXED = enum.auto()

    def __init__(self, *, d_in, max_d_in=None, n_blocks, d_block, activation: KWArgs | None = None, dropout,
                 max_n_blocks=None, max_d_block=None, forward_impl='dense', pack_size: int) -> None:
        nb, max_n_blocks = _positive_int_pack(n_blocks, max_n_blocks, pack_size=pack_size)
        super().__init__()
        self.blocks = nn.ModuleList([
            type(self).Block(
                in_features=d_in if i == 0 else d_block, out_features=d_block,
                max_in_features=max_d_in if i == 0 else max_d_block, max_out_features=max_d_block,
                activation={'type': nn.ReLU} if activation is None else activation,
                dropout=dropout, pack_size=pack_size)
            for i in range(max_n_blocks)
        ])
        self._max_n_blocks: Final = max_n_blocks
        self.register_buffer('n_blocks', nb)
        self._forward_impl = MLPBackbonePack.ForwardImpl(forward_impl)
        self._stream = _DropoutStream()
        self._nb_cache = None

    @property
    def pack_size(self) -> int:
        return self.blocks[0].pack_size

    @property
    def max_n_blocks(self) -> int:
        return self._max_n_blocks

    @property
    def forward_impl(self):
        return self._forward_impl

    def set_forward_impl(self, impl) -> None:
        self._forward_impl = MLPBackbonePack.ForwardImpl(impl)

    def set_member_base(self, base: int) -> None:
        """Global id of member 0 (for sharded packs: masks follow global ids)."""
        self._stream.member_base = int(base)
        for b in self.blocks:
            b.dropout._stream.member_base = int(base)

    def _invalidate(self) -> None:
        self._nb_cache = None

    def n_blocks_index_put_(self, indices, values) -> None:
        if self.n_blocks is None:
            raise RuntimeError('Cannot change block counts when all pack members share a fixed depth')
        self._invalidate()
        self.n_blocks.index_put_(indices, values)

    def replace(self, *, pack_idx: Tensor, d_in=None, n_blocks=None, d_block=None, **kwargs) -> None:
        check_pack_idx(pack_idx, self.pack_size)
        new_nb = None
        if n_blocks is not None:
            if self.n_blocks is None:
                raise RuntimeError('Cannot change block counts when all pack members share a fixed depth')
            if len(n_blocks) != len(pack_idx):
                raise ValueError('Each provided hyperparameter list must contain one value for each selected pack member')
            if not all(0 < v <= self.max_n_blocks for v in n_blocks):
                raise ValueError('Block counts must be positive and must not exceed `max_n_blocks`')
            new_nb = torch.tensor(n_blocks, dtype=self.n_blocks.dtype, device=self.n_blocks.device)
        for i, block in enumerate(self.blocks):
            block.replace(pack_idx=pack_idx, in_features=d_in if i == 0 else d_block, out_features=d_block, **kwargs)
        if new_nb is not None:
            self.n_blocks_index_put_((pack_idx,), new_nb)

    def _n_blocks_i32(self, pack_idx):
        if self.n_blocks is None:
            return None
        nb = _select(self.n_blocks, pack_idx)
        if pack_idx is not None:
            return nb.to(torch.int32)
        key = (self.n_blocks.data_ptr(), self.n_blocks._version if not self.n_blocks.is_inference() else -1)
        if self._nb_cache is None or self._nb_cache[0] != key:
            self._nb_cache = (key, nb.to(torch.int32))
        return self._nb_cache[1]

    def forward(self, x: Tensor, pack_idx: Tensor | None = None, *, onehot: dict | None = None,
                dx_cols: int = 0, row_index: Tensor | None = None, max_width: int | None = None) -> Tensor:
        """`onehot`: the first block's one-hot columns, gathered instead of multiplied (`x` then
        holds only the dense columns; see `_onehot_linear_call`).  `dx_cols`: the input's
        gradient is needed in its first dx_cols columns only.  `row_index` (pack_size, batch):
        `x` is a (rows, in) table whose rows the first block's GEMMs gather.  `max_width`
        (with `pack_idx`): the selected members' blocks run with this maximum width (at least
        every selected member's), so their activations are no wider."""
        if pack_idx is not None:
            check_pack_idx(pack_idx, self.pack_size)
            if onehot is not None:
                raise ValueError('the gathered one-hot first layer runs on the whole pack')
        nb = self._n_blocks_i32(pack_idx)
        stream = self._stream
        base_offset = None
        for i, block in enumerate(self.blocks):
            if block.training and base_offset is None:
                base_offset = stream.next_offset(self.max_n_blocks)
            sub = _OffsetView(stream, base_offset)
            first = {}
            if i == 0 and onehot is not None:
                first['onehot'] = onehot
            if i == 0 and dx_cols:
                first['dx_cols'] = dx_cols
            if i == 0 and row_index is not None:
                first['row_index'] = row_index
            if max_width is not None:
                first['narrow'] = (max_width, None if i == 0 else max_width)
            x = block(x, pack_idx, n_blocks=nb if i > 0 else None, block_index=i, stream=sub, **first)
        return x


class _OffsetView:
    """Per-forward Philox offsets of an MLP backbone: block i of the k-th
    training forward uses offset k * max_n_blocks + i."""

    def __init__(self, stream: _DropoutStream, base: int | None) -> None:
        self.seed = stream.seed
        self.member_base = stream.member_base
        self._base = base or 0

    def next_offset(self, stride: int = 1) -> int:
        return self._base


class _CosineEmbeddingFn(torch.autograd.Function):
    """One launch forward (`tp_cos_emb_forward`), one (or two) backward: parameter gradients
    from the gradient of the flattened embedding; the input takes no gradient."""

    @staticmethod
    def forward(ctx, x, weight, bias, affine_weight, affine_bias, d_embedding):
        y = ops.cos_emb_forward(x, weight, bias, affine_weight, affine_bias, d_embedding)
        ctx.save_for_backward(x, weight, bias, affine_weight, affine_bias)
        ctx.d_embedding = d_embedding
        return y

    @staticmethod
    def backward(ctx, gy):
        x, w, b, aw, ab = ctx.saved_tensors
        dw, db, daw, dab = ops.cos_emb_backward(x, w, b, aw, ab, ctx.d_embedding, gy)
        return None, dw, db, daw, dab, None


class _EmbeddedInputFn(torch.autograd.Function):
    """The first layer's bf16 input [cosine embeddings | one-hot | zeros] built in one buffer:
    `tp_cos_emb_forward` writes the embedding columns, `tp_tabpack_input` the one-hot block
    after them.  Backward: the parameter gradients from the embedding columns of the input's
    gradient, read in place."""

    @staticmethod
    def forward(ctx, x, weight, bias, affine_weight, affine_bias, d_embedding, cfg):
        P, F, D = affine_weight.shape
        B = x.shape[-2]
        out = torch.empty(P, B, cfg['width'], dtype=torch.bfloat16, device=x.device)
        ops.cos_emb_forward(x, weight, bias, affine_weight, affine_bias, d_embedding, out=out)
        ops.tabpack_input(None, cfg['x_cat'], cfg['cat_offsets'], cfg['width'], torch.bfloat16,
                          row_index=cfg['row_index'], out=out, col0=F * D)
        ctx.save_for_backward(x, weight, bias, affine_weight, affine_bias)
        ctx.d_embedding = d_embedding
        return out

    @staticmethod
    def backward(ctx, gx):
        x, w, b, aw, ab = ctx.saved_tensors
        dw, db, daw, dab = ops.cos_emb_backward(x, w, b, aw, ab, ctx.d_embedding, gx)
        return None, dw, db, daw, dab, None, None


class CosineEmbeddingsPack(ModulePack):
    """`CosineEmbeddingsPack` (`nn.py:1627-1833`): per feature the raw value and
    `cos(2 pi (w x + b))`, then an elementwise affine masked to each member's
    `d_embedding`, computed by `tp_cos_emb_forward` / `tp_cos_emb_backward`.

    Input `(pack_size, batch, n_features)` (or a shared `(batch, n_features)`), output
    `(pack_size, batch, n_features, max_d_embedding)`.
    """

    def __init__(self, n_features: int, d_embedding: int | list[int], *, max_d_embedding: int | None = None,
                 init_scale: float | list[float], pack_size: int) -> None:
        d_buf, max_d = _positive_int_pack(d_embedding, max_d_embedding, pack_size=pack_size)
        super().__init__()
        self.weight = ParameterPack(torch.empty(pack_size, n_features, max_d - 1))
        self.bias = ParameterPack(torch.empty(self.weight.shape))
        self.elementwise_affine_weight = ParameterPack(torch.empty(pack_size, n_features, max_d))
        self.elementwise_affine_bias = ParameterPack(torch.empty(self.elementwise_affine_weight.shape))
        self.register_buffer('d_embedding', d_buf)
        if isinstance(init_scale, (int, float)):
            self.init_scale = float(init_scale)
        else:
            self.register_buffer('init_scale', _mark_buffer(torch.tensor([float(v) for v in init_scale])))
        self._concat_input = True
        self.reset_parameters()

    @property
    def pack_size(self) -> int:
        return self.weight.shape[PACK_DIM]

    @property
    def max_d_embedding(self) -> int:
        return self.weight.shape[-1] + 1

    def get_output_shape(self) -> torch.Size:
        return torch.Size((self.weight.shape[1], self.weight.shape[2] + 1))

    def reset_parameters(self, *, pack_idx: Tensor | None = None) -> None:
        """Truncated N(0, 1) on [-3, 3] times the init scale for `weight`, zeros for the rest
        (`nn.py:1706-1753`)."""
        if pack_idx is not None:
            check_pack_idx(pack_idx, self.pack_size)
        n = self.pack_size if pack_idx is None else len(pack_idx)
        w = torch.empty(n, *self.weight.shape[1:], dtype=self.weight.dtype, device=self.weight.device)
        nn.init.trunc_normal_(w, a=-3.0, b=3.0)
        with torch.no_grad():
            if isinstance(self.init_scale, float):
                w *= self.init_scale
            else:
                w *= _select(self.init_scale, pack_idx).to(w)[:, None, None]
            if pack_idx is None:
                self.weight.copy_(w)
            else:
                self.weight[pack_idx] = w
            for p in (self.bias, self.elementwise_affine_weight, self.elementwise_affine_bias):
                if pack_idx is None:
                    p.zero_()
                else:
                    p[pack_idx] = 0.0

    def replace(self, *, pack_idx: Tensor, d_embedding: list[int] | None = None,
                init_scale: list[float] | None = None) -> None:
        """`CosineEmbeddingsPack.replace` (`nn.py:1755-1781`)."""
        check_pack_idx(pack_idx, self.pack_size)
        updates = []
        for vals in (d_embedding, init_scale):
            if vals is not None and len(vals) != len(pack_idx):
                raise ValueError('Each provided hyperparameter list must contain one value for each selected pack member')
        if d_embedding is not None:
            if self.d_embedding is None:
                raise RuntimeError('Cannot replace embedding sizes that are shared by all pack members')
            if not all(0 < v <= self.max_d_embedding for v in d_embedding):
                raise ValueError('Embedding sizes must be positive and must not exceed `max_d_embedding`')
            updates.append((self.d_embedding, d_embedding))
        if init_scale is not None:
            if isinstance(self.init_scale, float):
                raise RuntimeError('Cannot replace initialization scales that are shared by all pack members')
            updates.append((self.init_scale, init_scale))
        for buf, vals in updates:
            buf[pack_idx] = torch.tensor(vals, dtype=buf.dtype, device=buf.device)
        self.reset_parameters(pack_idx=pack_idx)

    def _flat(self, x: Tensor, pack_idx: Tensor | None) -> Tensor:
        """(P, B, n_features * max_d_embedding) embedding, the layout the first layer reads."""
        if x.ndim not in (2, 3):
            raise ValueError('The input must have three dimensions')
        if x.shape[-1] != self.weight.shape[-2]:
            raise ValueError('The number of input features must match the number of features configured for the '
                             'embeddings')
        if not x.is_cuda:
            raise RuntimeError('tabpack_b200 packs run on CUDA devices only')
        prm = [self.weight, self.bias, self.elementwise_affine_weight, self.elementwise_affine_bias]
        d = self.d_embedding
        if pack_idx is not None:
            check_pack_idx(pack_idx, self.pack_size)
            prm = [p[pack_idx] for p in prm]
            d = _select(d, pack_idx)
        if x.ndim == 3 and x.stride(0) == 0:
            x = x[0]
        xf = x.float().contiguous()
        d32 = None if d is None else d.to(torch.int32)
        with torch.autocast(x.device.type, enabled=False):
            return _CosineEmbeddingFn.apply(xf, *[p.contiguous() for p in prm], d32)

    def forward(self, x: Tensor, pack_idx: Tensor | None = None) -> Tensor:
        if x.ndim != 3:
            raise ValueError('The input must have three dimensions')
        y = self._flat(x, pack_idx)
        return y.view(y.shape[0], y.shape[1], *self.get_output_shape())


class _OneHotEncoding(nn.Module):
    """`_OneHotEncoding` (`nn.py:1836-1871`); the value `card` encodes as zeros."""

    def __init__(self, cardinalities: list[int]) -> None:
        super().__init__()
        self._cardinalities = cardinalities

    def forward(self, x: Tensor) -> Tensor:
        if x.shape[-1] != len(self._cardinalities):
            raise ValueError('The input must contain one categorical feature for each entry in `cardinalities`')
        return torch.cat([nn.functional.one_hot(x[..., i], c + 1)[..., :-1]
                          for i, c in enumerate(self._cardinalities)], -1)


def _embedding_class(kind):
    """The embedding class of `numerical_embeddings['type']`: this package's class, or the
    reference's class of the same name (configurations written for the reference work)."""
    name = kind if isinstance(kind, str) else getattr(kind, '__name__', '')
    if name == 'CosineEmbeddingsPack':
        return CosineEmbeddingsPack
    raise NotImplementedError(f'numerical embeddings of type {name!r} are not implemented on the B200 path '
                              '(CosineEmbeddingsPack is)')


class TabPack(ModulePack):
    """`TabPack` (`nn.py:1883-2110`); numerical embeddings: `CosineEmbeddingsPack`."""

    def __init__(self, *, n_numerical_features: int, categorical_cardinalities: list[int], d_out: int,
                 n_blocks, d_block, dropout, pack_size: int, numerical_embeddings: KWArgs | None = None,
                 **backbone_kwargs) -> None:
        super().__init__()
        max_d_in = None
        if numerical_embeddings is None:
            self.num_module = None
            d_in_num = n_numerical_features
        else:
            kw = dict(numerical_embeddings)
            cls = _embedding_class(kw.pop('type'))
            self.num_module = cls(n_numerical_features, pack_size=pack_size, **kw)
            d_emb = numerical_embeddings['d_embedding']
            if isinstance(d_emb, int):
                d_in_num = d_emb * n_numerical_features
            else:
                if not isinstance(d_emb, list):
                    raise TypeError('The `d_embedding` setting in `numerical_embeddings` must be an integer or a list')
                max_d_emb = numerical_embeddings.get('max_d_embedding') or max(d_emb)
                d_in_num = [v * n_numerical_features for v in d_emb]
                max_d_in = max_d_emb * n_numerical_features
        self.cat_module = _OneHotEncoding(categorical_cardinalities) if categorical_cardinalities else None
        d_in_cat = sum(categorical_cardinalities)
        d_in = d_in_num + d_in_cat if isinstance(d_in_num, int) else [v + d_in_cat for v in d_in_num]
        self.pack_view = PackView(pack_size=pack_size)
        self.backbone = MLPBackbonePack(d_in=d_in, max_d_in=None if max_d_in is None else max_d_in + d_in_cat,
                                        n_blocks=n_blocks, d_block=d_block, dropout=dropout,
                                        pack_size=pack_size, **backbone_kwargs)
        # With per-member embedding sizes the first layer's input is not a prefix of valid
        # columns (member m's embedding slots sit at f * max_d + k, the one-hot block after
        # all of them); the reference's first layer multiplies the whole padded width
        # (`nn.py:792-816` uses in_features only for initialisation), so this one does too.
        # (with embeddings of one size for all members the input widths all equal the maximum,
        # so the whole width is the same computation)
        self.backbone.blocks[0].linear.full_width_input = isinstance(d_in, list) or self.num_module is not None
        self.output = LinearPack(d_block, d_out, max_in_features=backbone_kwargs.get('max_d_block'),
                                 pack_size=pack_size)
        self._n_numerical_features = n_numerical_features
        self._categorical_cardinalities = categorical_cardinalities
        # prefix sums of the cardinalities: the one-hot block of each feature (tp_tabpack_input)
        offs = [0]
        for c in categorical_cardinalities:
            offs.append(offs[-1] + c)
        self.register_buffer('_cat_offsets', torch.tensor(offs, dtype=torch.int32), persistent=False)

    @property
    def pack_size(self) -> int:
        return self.backbone.pack_size

    def _fused_input(self, x_num: Tensor | None, x_cat: Tensor, row_index: Tensor | None = None) -> Tensor | None:
        """[x_num | one-hot(x_cat)] built by one kernel in the first layer's dtype (already
        padded to the tensor-core width), or None when the generic path has to run (input
        gradients, numerical embeddings, CPU tensors, an fp32 width the kernel cannot pad).
        With `row_index`, x_num / x_cat are whole datasets and the rows are gathered too."""
        if self.num_module is not None or self.cat_module is None or not x_cat.is_cuda:
            return None
        if row_index is not None and (not row_index.is_cuda or x_cat.ndim != 2
                                      or (x_num is not None and (x_num.ndim != 2 or x_num.shape[0] != x_cat.shape[0]))):
            return None
        lead_ok = row_index is not None or x_num is None or x_num.shape[:-1] == x_cat.shape[:-1]
        if x_num is not None and (x_num.requires_grad or not x_num.is_cuda or not lead_ok
                                  or x_num.shape[-1] != self._n_numerical_features):
            return None
        if x_cat.shape[-1] != len(self._categorical_cardinalities):
            return None
        if torch.is_autocast_enabled('cuda') and torch.get_autocast_dtype('cuda') == torch.bfloat16:
            dtype = torch.bfloat16
        else:
            dtype = x_num.dtype if x_num is not None else torch.get_default_dtype()
        d_in = self._n_numerical_features + sum(self._categorical_cardinalities)
        if dtype == torch.bfloat16:
            width = _round8(d_in)
        elif dtype == torch.float32 and d_in % 4 == 0:
            width = d_in
        else:
            return None
        return ops.tabpack_input(x_num, x_cat, self._cat_offsets, width, dtype, row_index=row_index)

    # The per-step batch gather (`_training.py:2667-2669`) inside the first block's GEMM operand
    # loads: the dataset's first-layer input ([x_num | one-hot(x_cat)], bf16, padded width) is
    # built once and kept, and every step's rows are gathered from it by the forward and weight-
    # gradient GEMMs (TMA gather4, 4 table rows per load) instead of being copied into a
    # (pack, batch, width) tensor.  Off by default: on a B200 the gathered GEMMs (single CTAs,
    # 32 gather loads per 16 KB operand stage) measured 2.7 ms (forward) and 3.7 ms (weight
    # gradient) slower per step of the 512-member training configuration than the copied batch
    # on CTA pairs, against 0.47 ms saved by not building the copy.
    gather_batch_in_gemm = False

    def _input_table(self, x_num: Tensor | None, x_cat: Tensor | None, row_index: Tensor,
                     pack_idx: Tensor | None) -> Tensor | None:
        """The dataset's encoded first-layer input for `forward_rows` to gather from, or None when
        the other paths apply (no one-hot features, numerical embeddings, a member subset,
        fp32 compute, per-member input datasets)."""
        if not self.gather_batch_in_gemm or pack_idx is not None or x_cat is None or row_index.ndim != 2:
            return None
        if not (torch.is_autocast_enabled('cuda') and torch.get_autocast_dtype('cuda') == torch.bfloat16):
            return None
        # the cache holds the datasets weakly and keys on their identity and version counters, so
        # a new or modified dataset (even one at a freed dataset's address) builds a new table
        versions = tuple(None if t is None else t._version for t in (x_num, x_cat))
        cached = self.__dict__.get('_table_cache')
        if cached is not None:
            refs, vers, offsets, table = cached
            same = all((r is None and t is None) or (r is not None and r() is t) for r, t in zip(refs, (x_num, x_cat)))
            if same and vers == versions and offsets is self._cat_offsets:
                return table
        table = self._fused_input(x_num, x_cat)  # every dataset row, no gather
        if table is None or table.dtype != torch.bfloat16 or table.ndim != 2:
            return None
        refs = tuple(None if t is None else weakref.ref(t) for t in (x_num, x_cat))
        self.__dict__['_table_cache'] = (refs, versions, self._cat_offsets, table)
        return table

    # batch rows one gathered first-layer call sorts in shared memory (tp_onehot_linear_forward)
    _GATHER_MAX_ROWS = 16384

    # The gathered first layer in training too.  Off by default: its backward forms the one-hot
    # columns' weight gradient as segmented sums on the CUDA cores, which measured slower on a
    # B200 than the dense tensor-core weight gradient over the one-hot input (both write the
    # same dW); forwards without a backward (evaluation, prediction) always gather.
    gather_one_hot_in_training = False

    def _gathered(self, x_num: Tensor | None, x_cat: Tensor | None, row_index: Tensor | None,
                  pack_idx: Tensor | None) -> Tensor | None:
        """The model output with the first layer's one-hot columns gathered from the weight
        (one W column per feature and row) instead of multiplied, or None when this path does
        not apply: it needs bf16 autocast on a CUDA device (the tensor-core path), categorical
        features, the whole pack, inputs whose gradient is not requested, and no backward
        (unless `gather_one_hot_in_training`)."""
        if pack_idx is not None or self.cat_module is None or x_cat is None or not x_cat.is_cuda:
            return None
        if (torch.is_grad_enabled() and not self.gather_one_hot_in_training
                and any(p.requires_grad for p in self.parameters())):
            return None
        if not (torch.is_autocast_enabled('cuda') and torch.get_autocast_dtype('cuda') == torch.bfloat16):
            return None
        if x_cat.shape[-1] != len(self._categorical_cardinalities) or x_cat.ndim not in (2, 3):
            return None
        if x_num is not None and (x_num.requires_grad or not x_num.is_cuda
                                  or x_num.shape[-1] != self._n_numerical_features):
            return None
        P = self.pack_size
        if row_index is not None:
            if (not row_index.is_cuda or row_index.ndim != 2 or row_index.shape[0] != P or x_cat.ndim != 2
                    or (x_num is not None and (x_num.ndim != 2 or x_num.shape[0] != x_cat.shape[0]))):
                return None
            B = row_index.shape[1]
        else:
            if x_num is not None and x_num.shape[:-1] != x_cat.shape[:-1]:
                return None
            if x_cat.ndim == 3 and x_cat.shape[0] != P:
                return None
            B = x_cat.shape[-2]
        if B > self._GATHER_MAX_ROWS or B == 0:
            return None
        if (row_index is not None or x_cat.ndim == 3) and not self.training:
            raise RuntimeError('Three-dimensional input requires training mode')
        linear = self.backbone.blocks[0].linear
        n_dense = linear.max_in_features - sum(self._categorical_cardinalities)
        if self.num_module is None:
            lead = (B,) if row_index is None and x_cat.ndim == 2 else (P, B)
            if x_num is None:
                dense = torch.zeros(*lead, 8, dtype=torch.bfloat16, device=x_cat.device)
            else:
                dense = ops.tabpack_input(x_num, None, self._cat_offsets, _round8(max(n_dense, 1)), torch.bfloat16,
                                          row_index=row_index)
        else:
            if x_num is None:
                raise ValueError('`x_num` is required when numerical embeddings are configured')
            xn = x_num[row_index] if row_index is not None else x_num
            if xn.ndim == 2:
                xn = xn.expand(P, *xn.shape)
            dense = self.num_module._flat(xn, None)
        onehot = {'x_cat': x_cat, 'cat_offsets': self._cat_offsets, 'n_dense': n_dense, 'row_index': row_index}
        return self.output(self.backbone(dense, None, onehot=onehot), None)

    def _embedded_input(self, x_num: Tensor | None, x_cat: Tensor | None, row_index: Tensor | None,
                        pack_idx: Tensor | None) -> tuple[Tensor, int] | None:
        """(bf16 first-layer input [cosine embeddings | one-hot], embedding columns) built in one
        buffer (`_EmbeddedInputFn`), or None when the generic path has to run: it needs cosine
        numerical embeddings, categorical features, bf16 autocast on a CUDA device, the whole
        pack and an embedding width that keeps the one-hot block 16-byte aligned."""
        if (not isinstance(self.num_module, CosineEmbeddingsPack) or self.cat_module is None or x_num is None
                or x_cat is None or pack_idx is not None or not x_cat.is_cuda or not x_num.is_cuda):
            return None
        if not (torch.is_autocast_enabled('cuda') and torch.get_autocast_dtype('cuda') == torch.bfloat16):
            return None
        emb = self.num_module
        P, F, D = emb.elementwise_affine_weight.shape
        if (F * D) % 8 != 0 or x_cat.shape[-1] != len(self._categorical_cardinalities) or x_num.shape[-1] != F:
            return None
        if row_index is not None:
            if row_index.ndim != 2 or row_index.shape[0] != P or x_cat.ndim != 2 or x_num.ndim != 2:
                return None
            x = x_num[row_index]
            ri = row_index
        else:
            if x_num.shape[:-1] != x_cat.shape[:-1] or (x_cat.ndim == 3 and x_cat.shape[0] != P):
                return None
            x = x_num
            B = x_cat.shape[-2]
            # one-hot rows per member: the shared batch's rows for every member
            ri = None if x_cat.ndim == 3 else torch.arange(B, device=x_cat.device).expand(P, B)
        if x.ndim == 3 and x.stride(0) == 0:
            x = x[0]
        width = self.backbone.blocks[0].linear.max_in_features
        width = _round8(width)
        cfg = {'x_cat': x_cat, 'cat_offsets': self._cat_offsets, 'row_index': ri, 'width': width}
        prm = [emb.weight, emb.bias, emb.elementwise_affine_weight, emb.elementwise_affine_bias]
        d32 = None if emb.d_embedding is None else emb.d_embedding.to(torch.int32)
        with torch.autocast(x.device.type, enabled=False):
            buf = _EmbeddedInputFn.apply(x.float().contiguous(), *[p.contiguous() for p in prm], d32, cfg)
        return buf, F * D

    def forward_rows(self, x_num: Tensor | None, x_cat: Tensor | None, row_index: Tensor,
                     pack_idx: Tensor | None = None) -> Tensor:
        """`forward(x_num[row_index], x_cat[row_index])`: the per-step batch gather of the
        training loop (`_training.py:2667-2669`), fused into the first-layer input build when
        the model has one-hot features and no numerical embeddings (otherwise gathered first).
        `row_index`: (pack_size, batch) dataset rows of every member."""
        y = self._gathered(x_num, x_cat, row_index, pack_idx)
        if y is not None:
            return y
        emb = self._embedded_input(x_num, x_cat, row_index, pack_idx)
        if emb is not None:
            return self.output(self.backbone(emb[0], pack_idx, dx_cols=emb[1]), pack_idx)
        table = self._input_table(x_num, x_cat, row_index, pack_idx)
        if table is not None:
            return self.output(self.backbone(table, pack_idx, row_index=row_index), pack_idx)
        fused = None if x_cat is None else self._fused_input(x_num, x_cat, row_index)
        if fused is None:
            return self(None if x_num is None else x_num[row_index], None if x_cat is None else x_cat[row_index],
                        pack_idx)
        return self.output(self.backbone(fused, pack_idx), pack_idx)

    def replace(self, *, pack_idx: Tensor, numerical_embeddings=None, d_block=None, **kwargs) -> None:
        """`TabPack.replace` (`nn.py:1986-2024`)."""
        if numerical_embeddings is not None and self.num_module is None:
            raise RuntimeError('Cannot replace numerical embeddings because this model has none')
        if self.num_module is not None:
            self.num_module.replace(pack_idx=pack_idx, **({} if numerical_embeddings is None else numerical_embeddings))
        d_emb = None if numerical_embeddings is None else numerical_embeddings.get('d_embedding')
        d_in = None if d_emb is None else [v * self._n_numerical_features + sum(self._categorical_cardinalities)
                                           for v in d_emb]
        self.backbone.replace(pack_idx=pack_idx, d_in=d_in, d_block=d_block, **kwargs)
        self.output.replace(pack_idx=pack_idx, in_features=d_block)

    def _head(self, h: Tensor, pack_idx: Tensor | None, max_width: int | None) -> Tensor:
        if max_width is None:
            return self.output(h, pack_idx)
        return _linear_call(self.output, h, pack_idx, relu=False, dropout=None, stream=None, n_blocks=None,
                            block_index=0, narrow=(None, max_width))

    def forward(self, x_num: Tensor | None, x_cat: Tensor | None, pack_idx: Tensor | None = None, *,
                max_width: int | None = None) -> Tensor:
        """`max_width` (evaluation with `pack_idx`): the selected members' hidden width bound; the
        backbone and the head then run with that maximum width instead of `max_d_block`, which
        leaves every member's output unchanged and its activations narrower."""
        if x_num is None and x_cat is None:
            raise ValueError('Provide at least one of `x_num` and `x_cat`')
        if max_width is not None:
            if pack_idx is None or self.training:
                raise ValueError('max_width applies to an evaluation-mode forward of selected members')
            max_width = min(int(max_width), self.backbone.blocks[0].linear.max_out_features)
        # per-member batches are a training-time input (PackView, `nn.py:88-131`); a shared batch
        # may still become per-member inside (numerical embeddings)
        if not self.training and any(t is not None and t.ndim == 3 for t in (x_num, x_cat)):
            raise RuntimeError('Three-dimensional input requires training mode')
        y = self._gathered(x_num, x_cat, None, pack_idx)
        if y is not None:
            return y
        emb = self._embedded_input(x_num, x_cat, None, pack_idx)
        if emb is not None:
            return self._head(self.backbone(emb[0], pack_idx, dx_cols=emb[1], max_width=max_width), pack_idx,
                              max_width)
        fused = None if x_cat is None else self._fused_input(x_num, x_cat)
        if fused is not None:
            return self._head(self.backbone(fused, pack_idx, max_width=max_width), pack_idx, max_width)
        parts = []
        if x_num is not None:
            if self.num_module is None:
                parts.append(x_num)
            else:
                if x_num.ndim == 2:
                    x_num = x_num.expand(self.pack_size, *x_num.shape)
                parts.append(self.num_module._flat(x_num, pack_idx))
        elif self.num_module is not None:
            raise ValueError('`x_num` is required when numerical embeddings are configured')
        if x_cat is not None:
            if self.cat_module is None:
                raise ValueError('`x_cat` can only be provided when categorical features are configured')
            dt = parts[0].dtype if parts else torch.get_default_dtype()
            oh = self.cat_module(x_cat).to(dt)
            if parts and parts[0].ndim == 3 and oh.ndim == 2:
                oh = oh.expand(parts[0].shape[0], *oh.shape)
            parts.append(oh)
        x = torch.cat(parts, -1) if len(parts) > 1 else parts[0]
        x = self.backbone(x, pack_idx, max_width=max_width)
        return self._head(x, pack_idx, max_width)
