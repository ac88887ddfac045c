"""ctypes binding of `libtabpack_b200.so` (the C ABI in `include/tabpack_b200.h`).

The library is loaded lazily on first use.  There is no fallback: if the
library is missing or fails to load, every op raises.
"""

from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, 'libtabpack_b200.so')

TP_DTYPE_F32 = 0
TP_DTYPE_BF16 = 1
TP_DTYPE_F64 = 2
TP_MAX_OPT_TENSORS = 32
TP_NOALLOC_SCRATCH_BYTES = 16 << 20

_c_int32_p = ctypes.POINTER(ctypes.c_int32)
_c_float_p = ctypes.POINTER(ctypes.c_float)


class LinearArgs(ctypes.Structure):
    _fields_ = [
        ('P', ctypes.c_int32), ('B', ctypes.c_int32), ('max_in', ctypes.c_int32),
        ('max_out', ctypes.c_int32), ('dtype', ctypes.c_int32), ('x_shared', ctypes.c_int32),
        ('in_features', ctypes.c_void_p), ('out_features', ctypes.c_void_p),
        ('n_blocks', ctypes.c_void_p), ('block_index', ctypes.c_int32), ('relu', ctypes.c_int32),
        ('dropout_p', ctypes.c_void_p), ('seed', ctypes.c_uint64), ('offset', ctypes.c_uint32),
        ('member_base', ctypes.c_uint32), ('x', ctypes.c_void_p), ('w', ctypes.c_void_p),
        ('bias', ctypes.c_void_p), ('y', ctypes.c_void_p), ('y_pad_zero', ctypes.c_int32),
        ('row_index', ctypes.c_void_p), ('x_rows', ctypes.c_int32),
    ]


class LinearGradArgs(ctypes.Structure):
    _fields_ = [
        ('fwd', LinearArgs), ('dy', ctypes.c_void_p), ('y', ctypes.c_void_p), ('g', ctypes.c_void_p),
        ('dbias', ctypes.c_void_p), ('dx', ctypes.c_void_p), ('dw', ctypes.c_void_p),
        ('dw_rows', ctypes.c_int32), ('dw_cols', ctypes.c_int32), ('db_cols', ctypes.c_int32),
        ('g_ready', ctypes.c_int32), ('dx_cols', ctypes.c_int32), ('dw_pad_zero', ctypes.c_int32),
        ('dx_pad_zero', ctypes.c_int32),
    ]


class OptTensor(ctypes.Structure):
    _fields_ = [
        ('p', ctypes.c_void_p), ('grad', ctypes.c_void_p), ('exp_avg', ctypes.c_void_p),
        ('exp_avg_sq', ctypes.c_void_p), ('step', ctypes.c_void_p), ('numel', ctypes.c_int64),
        ('inner', ctypes.c_int64),
    ]


class HParam(ctypes.Structure):
    _fields_ = [('per_member', ctypes.c_void_p), ('scalar', ctypes.c_double)]


class AdamWArgs(ctypes.Structure):
    _fields_ = [
        ('n_tensors', ctypes.c_int32), ('t', OptTensor * TP_MAX_OPT_TENSORS),
        ('lr', HParam), ('beta1', HParam), ('beta2', HParam), ('eps', HParam),
        ('weight_decay', HParam), ('step', ctypes.c_int64),
    ]


class MuonArgs(ctypes.Structure):
    _fields_ = [
        ('P', ctypes.c_int32), ('max_out', ctypes.c_int32), ('max_in', ctypes.c_int32),
        ('p', ctypes.c_void_p), ('grad', ctypes.c_void_p), ('momentum_buffer', ctypes.c_void_p),
        ('out_features', ctypes.c_void_p), ('in_features', ctypes.c_void_p),
        ('lr', HParam), ('momentum', HParam), ('weight_decay', HParam),
        ('update_scale', ctypes.c_void_p), ('nesterov', ctypes.c_int32), ('mutate_grad', ctypes.c_int32),
        ('ns_steps', ctypes.c_int32), ('workspace', ctypes.c_void_p), ('workspace_bytes', ctypes.c_size_t),
        ('p_bf16', ctypes.c_void_p), ('p_bf16_rows', ctypes.c_int32), ('p_bf16_cols', ctypes.c_int32),
        ('n_blocks', ctypes.c_void_p), ('block_index', ctypes.c_int32), ('gated_momentum_zero', ctypes.c_int32),
    ]


class MetricArgs(ctypes.Structure):
    _fields_ = [
        ('metric', ctypes.c_int32), ('P', ctypes.c_int32), ('N', ctypes.c_int64), ('C', ctypes.c_int32),
        ('y_pred', ctypes.c_void_p), ('y_true', ctypes.c_void_p), ('out', ctypes.c_void_p),
    ]


class CosEmbArgs(ctypes.Structure):
    _fields_ = [
        ('P', ctypes.c_int32), ('B', ctypes.c_int32), ('F', ctypes.c_int32), ('D', ctypes.c_int32),
        ('x_shared', ctypes.c_int32), ('x', ctypes.c_void_p), ('weight', ctypes.c_void_p), ('bias', ctypes.c_void_p),
        ('affine_weight', ctypes.c_void_p), ('affine_bias', ctypes.c_void_p), ('d_embedding', ctypes.c_void_p),
        ('out', ctypes.c_void_p), ('out_ld', ctypes.c_int32), ('out_dtype', ctypes.c_int32),
        ('grad_out', ctypes.c_void_p), ('grad_ld', ctypes.c_int32), ('grad_dtype', ctypes.c_int32),
        ('dweight', ctypes.c_void_p), ('dbias', ctypes.c_void_p), ('daffine_weight', ctypes.c_void_p),
        ('daffine_bias', ctypes.c_void_p), ('workspace', ctypes.c_void_p), ('workspace_bytes', ctypes.c_size_t),
    ]


class InputArgs(ctypes.Structure):
    _fields_ = [
        ('rows', ctypes.c_int64), ('n_num', ctypes.c_int32), ('n_cat', ctypes.c_int32), ('x_num', ctypes.c_void_p),
        ('x_cat', ctypes.c_void_p), ('row_index', ctypes.c_void_p), ('cat_offsets', ctypes.c_void_p),
        ('out', ctypes.c_void_p),
        ('out_ld', ctypes.c_int32), ('out_dtype', ctypes.c_int32), ('out_col0', ctypes.c_int32),
    ]


class WeightCastArgs(ctypes.Structure):
    _fields_ = [
        ('P', ctypes.c_int32), ('src_rows', ctypes.c_int32), ('src_cols', ctypes.c_int32),
        ('src_ld', ctypes.c_int32), ('dst_rows', ctypes.c_int32), ('dst_cols', ctypes.c_int32), ('out_features', ctypes.c_void_p),
        ('in_features', ctypes.c_void_p), ('n_blocks', ctypes.c_void_p), ('block_index', ctypes.c_int32),
        ('src', ctypes.c_void_p), ('dst', ctypes.c_void_p),
    ]


class WeightCastTArgs(ctypes.Structure):
    _fields_ = [
        ('P', ctypes.c_int32), ('src_rows', ctypes.c_int32), ('src_ld', ctypes.c_int32), ('col0', ctypes.c_int32),
        ('ncols', ctypes.c_int32), ('dst_ld', ctypes.c_int32), ('out_features', ctypes.c_void_p),
        ('src', ctypes.c_void_p), ('dst', ctypes.c_void_p),
    ]


class OneHotArgs(ctypes.Structure):
    _fields_ = [
        ('n_dense', ctypes.c_int32), ('n_cat', ctypes.c_int32), ('n_onehot', ctypes.c_int32),
        ('cat_offsets', ctypes.c_void_p), ('x_cat', ctypes.c_void_p), ('x_cat_member_stride', ctypes.c_int64),
        ('row_index', ctypes.c_void_p), ('row_index_member_stride', ctypes.c_int64),
        ('w_onehot_t', ctypes.c_void_p), ('wt_ld', ctypes.c_int32), ('sorted_keys', ctypes.c_void_p),
        ('addend', ctypes.c_void_p), ('addend_ld', ctypes.c_int32),
    ]


class GreedyArgs(ctypes.Structure):
    _fields_ = [
        ('metric', ctypes.c_int32), ('maximize', ctypes.c_int32), ('n_pred', ctypes.c_int32),
        ('N', ctypes.c_int64), ('C', ctypes.c_int32), ('predictions', ctypes.c_void_p), ('y_true', ctypes.c_void_p),
        ('init_top_k', ctypes.c_int32), ('max_ensemble_size', ctypes.c_int32), ('with_replacement', ctypes.c_int32),
        ('counts', ctypes.c_void_p), ('workspace', ctypes.c_void_p), ('workspace_bytes', ctypes.c_size_t),
        ('status', ctypes.c_void_p),
    ]


# kernel families of tp_profile_stop, in TP_PROF_* order
TP_PROF_KINDS = ('fwd', 'dgrad', 'wgrad', 'newton_schulz_gram', 'newton_schulz_update', 'gemm_f32', 'act_backward',
                 'muon_elementwise', 'adamw', 'weight_cast', 'input', 'embedding', 'onehot', 'metric', 'greedy',
                 'roc_auc', 'other')
TP_METRIC = {'mse': 0, 'mae': 1, 'accuracy': 2, 'bce': 3, 'ce': 4, 'accuracy_argmax': 5, 'r2': 6}


# name -> (restype, argtypes); every symbol here is declared in include/tabpack_b200.h
SIGNATURES = {
    'tp_linear_forward': (ctypes.c_int, [ctypes.POINTER(LinearArgs), ctypes.c_void_p]),
    'tp_linear_backward': (ctypes.c_int, [ctypes.POINTER(LinearGradArgs), ctypes.c_void_p]),
    'tp_linear_backward_noalloc': (ctypes.c_int, [ctypes.POINTER(LinearGradArgs), ctypes.c_void_p]),
    'tp_profile_start': (ctypes.c_int, [ctypes.c_int32]),
    'tp_profile_stop': (ctypes.c_int, [ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_int64), ctypes.c_int32,
                                       ctypes.POINTER(ctypes.c_int32)]),
    'tp_quotient_check': (ctypes.c_int, [ctypes.c_int32, ctypes.c_int32, ctypes.c_void_p, ctypes.c_void_p]),
    'tp_dropout_mask': (ctypes.c_int, [ctypes.c_uint64, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_void_p,
                                       ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_void_p,
                                       ctypes.c_void_p]),
    'tp_adamw_step': (ctypes.c_int, [ctypes.POINTER(AdamWArgs), ctypes.c_void_p]),
    'tp_muon_workspace_size': (ctypes.c_size_t, [ctypes.c_int32, ctypes.c_int32, ctypes.c_int32]),
    'tp_muon_step': (ctypes.c_int, [ctypes.POINTER(MuonArgs), ctypes.c_void_p]),
    'tp_muon_grouped_workspace_size': (ctypes.c_size_t, [ctypes.POINTER(MuonArgs), ctypes.c_int32]),
    'tp_muon_step_grouped': (ctypes.c_int, [ctypes.POINTER(MuonArgs), ctypes.c_int32, ctypes.c_void_p,
                                            ctypes.c_size_t, ctypes.c_void_p]),
    'tp_metric_pack': (ctypes.c_int, [ctypes.POINTER(MetricArgs), ctypes.c_void_p]),
    'tp_greedy_workspace_size': (ctypes.c_size_t, [ctypes.c_int32, ctypes.c_int64, ctypes.c_int32]),
    'tp_greedy_ensemble': (ctypes.c_int, [ctypes.POINTER(GreedyArgs), ctypes.c_void_p]),
    'tp_ensemble_mean': (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int32,
                                        ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p]),
    'tp_softmax_rows': (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32, ctypes.c_void_p,
                                       ctypes.c_void_p]),
    'tp_permutation_keys': (ctypes.c_int, [ctypes.c_uint64, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_int32,
                                           ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p]),
    'tp_cos_emb_workspace_size': (ctypes.c_size_t, [ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32]),
    'tp_cos_emb_forward': (ctypes.c_int, [ctypes.POINTER(CosEmbArgs), ctypes.c_void_p]),
    'tp_cos_emb_backward': (ctypes.c_int, [ctypes.POINTER(CosEmbArgs), ctypes.c_void_p]),
    'tp_tabpack_input': (ctypes.c_int, [ctypes.POINTER(InputArgs), ctypes.c_void_p]),
    'tp_weight_cast': (ctypes.c_int, [ctypes.POINTER(WeightCastArgs), ctypes.c_void_p]),
    'tp_weight_cast_transposed': (ctypes.c_int, [ctypes.POINTER(WeightCastTArgs), ctypes.c_void_p]),
    'tp_onehot_linear_forward': (ctypes.c_int, [ctypes.POINTER(LinearArgs), ctypes.POINTER(OneHotArgs),
                                                ctypes.c_void_p]),
    'tp_onehot_linear_backward': (ctypes.c_int, [ctypes.POINTER(LinearGradArgs), ctypes.POINTER(OneHotArgs),
                                                 ctypes.c_void_p]),
    'tp_roc_auc_workspace_size': (ctypes.c_size_t, [ctypes.c_int32, ctypes.c_int64, ctypes.c_int32]),
    'tp_binary_roc_auc': (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64,
                                         ctypes.c_int32, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t,
                                         ctypes.c_void_p]),
    'tp_device_error': (ctypes.c_int, []),
    'tp_last_error_string': (ctypes.c_char_p, []),
    'tp_version': (ctypes.c_char_p, []),
}

_lock = threading.Lock()
_lib = None


class TabPackError(RuntimeError):
    """A tabpack_b200 C-ABI call returned an error code."""


def load(path: str | None = None) -> ctypes.CDLL:
    """Load the library (once) and bind every declared symbol."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        p = path or LIB_PATH
        if not os.path.exists(p):
            raise TabPackError(
                f'{p} is missing: build it with `python -m tabpack_b200.csrc.build` '
                '(this package has no CPU fallback)'
            )
        lib = ctypes.CDLL(p)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def check(rc: int, what: str) -> None:
    if rc != 0:
        msg = load().tp_last_error_string().decode(errors='replace')
        raise TabPackError(f'{what} failed ({rc}): {msg}')
