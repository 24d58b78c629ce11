"""ctypes binding of the C ABI in include/sq325.h (libsq325.so, built in-tree for sm_100a).

There is no fallback: if the shared library is missing or a GPU call fails, the
error surfaces as an exception with the library's own message.  Status codes map to
the exception classes the reference raises for the same conditions
(ValueError / RuntimeError / FloatingPointError).
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / 'libsq325.so'

SQ_OK, SQ_EINVAL, SQ_ESTATE, SQ_ENONFINITE, SQ_ECUDA, SQ_ETIMEOUT, SQ_ENOMEM = range(7)
ABI_VERSION = 1


class DeviceTimeout(RuntimeError):
    """A bounded device-side wait expired (SQ_ETIMEOUT); the CUDA context stays usable."""


_EXC = {SQ_EINVAL: ValueError, SQ_ESTATE: RuntimeError, SQ_ENONFINITE: FloatingPointError,
        SQ_ECUDA: RuntimeError, SQ_ETIMEOUT: DeviceTimeout, SQ_ENOMEM: MemoryError}

p = C.c_void_p
i32 = C.c_int32
i64 = C.c_int64


class ScanArgs(C.Structure):
    _fields_ = [('batch', i32), ('length', i32), ('heads', i32), ('dim', i32), ('groups', i32), ('layout', i32),
                ('x', p), ('x_batch_stride', i64), ('x_token_stride', i64),
                ('dt', p), ('dt_batch_stride', i64), ('dt_token_stride', i64),
                ('A', p),
                ('B', p), ('b_batch_stride', i64), ('b_token_stride', i64),
                ('C', p), ('c_batch_stride', i64), ('c_token_stride', i64),
                ('D', p), ('d_is_f32', i32), ('dt_bias', p), ('dt_bias_is_f32', i32),
                ('permutation', p), ('basis', p), ('latent_scale', p), ('predictor', p),
                ('lo', p), ('hi', p), ('q4', p), ('latent', p), ('s8', p), ('s4', p),
                ('y', p), ('y_batch_stride', i64), ('y_token_stride', i64),
                ('workspace', p), ('workspace_bytes', i64)]


class S16Args(C.Structure):
    _fields_ = [('batch', i32), ('length', i32), ('heads', i32), ('dim', i32), ('groups', i32),
                ('x', p), ('x_batch_stride', i64), ('x_token_stride', i64),
                ('dt', p), ('dt_batch_stride', i64), ('dt_token_stride', i64),
                ('A', p),
                ('B', p), ('b_batch_stride', i64), ('b_token_stride', i64),
                ('C', p), ('c_batch_stride', i64), ('c_token_stride', i64),
                ('D', p), ('d_is_f32', i32), ('dt_bias', p), ('dt_bias_is_f32', i32),
                ('state', p), ('y', p), ('y_batch_stride', i64), ('y_token_stride', i64), ('stats', p)]


class Sq3p25Args(C.Structure):
    _fields_ = [('batch', i32), ('length', i32), ('heads', i32), ('dim', i32), ('groups', i32),
                ('x', p), ('x_batch_stride', i64), ('x_token_stride', i64),
                ('dt', p), ('dt_batch_stride', i64), ('dt_token_stride', i64),
                ('A', p),
                ('B', p), ('b_batch_stride', i64), ('b_token_stride', i64),
                ('C', p), ('c_batch_stride', i64), ('c_token_stride', i64),
                ('D', p), ('d_is_f32', i32), ('dt_bias', p), ('dt_bias_is_f32', i32),
                ('permutation', p),
                ('lo', p), ('hi', p), ('q4', p), ('s8', p), ('s4', p),
                ('y', p), ('y_batch_stride', i64), ('y_token_stride', i64)]


class ConvArgs(C.Structure):
    _fields_ = [('weight', p), ('bias', p), ('ring', p), ('ring_batch_stride', i64), ('position', i32)]


class ModelConfig(C.Structure):
    _fields_ = [('n_layer', i32), ('vocab', i32), ('eps', C.c_float)]


class Fp4Matrix(C.Structure):
    _fields_ = [('codes', p), ('block_scales', p), ('global_scale', p), ('rows', i32), ('cols', i32)]


class LayerDesc(C.Structure):
    _fields_ = [('in_proj', Fp4Matrix), ('out_proj', Fp4Matrix), ('norm_weight', p), ('conv_weight', p),
                ('conv_bias', p), ('A', p), ('D', p), ('dt_bias', p), ('gated_norm_weight', p), ('layout', i32),
                ('permutation', p), ('basis', p), ('latent_scale', p), ('predictor', p)]


# name -> (restype, argtypes)
_PROTOS = {
    'sq_abi_version': (C.c_int, []),
    'sq_last_error': (C.c_char_p, []),
    'sq_layout_index': (C.c_int, [C.c_char_p]),
    'sq_layout_counts': (C.c_int, [C.c_int, C.POINTER(C.c_int), C.POINTER(C.c_int), C.POINTER(C.c_int)]),
    'sq_state_bytes': (i64, [C.c_int, C.c_int, C.c_int]),
    'sq_scan': (C.c_int, [C.POINTER(ScanArgs), p]),
    'sq_scan_conv': (C.c_int, [C.POINTER(ScanArgs), C.POINTER(ConvArgs), p]),
    'sq_s16_scan': (C.c_int, [C.POINTER(S16Args), p]),
    'sq_sq3p25_scan': (C.c_int, [C.POINTER(Sq3p25Args), p]),
    'sq_ste_workspace': (i64, [C.c_int, C.c_int, C.c_int, C.c_int, C.c_int]),
    'sq_ste_backward': (C.c_int, [C.POINTER(Sq3p25Args), C.c_int, p, p, p, p, p, p, i64, p]),
    'sq_state_decode': (C.c_int, [C.c_int] * 5 + [p] * 9 + [p]),
    'sq_state_encode': (C.c_int, [C.c_int] * 6 + [p] * 9 + [p]),
    'sq_fp4_decode': (C.c_int, [p, p, p, C.c_int, C.c_int, p, i64, p]),
    'sq_fp4_validate': (C.c_int, [p, p, p, C.c_int, C.c_int, p]),
    'sq_scan_workspace': (i64, [C.c_int, C.c_int, C.c_int, C.c_int, C.c_int]),
    'sq_model_set_exact_skinny': (C.c_int, [p, C.c_int]),
    'sq_model_time_gemm': (C.c_int, [p, C.c_int]),
    'sq_model_gemm_time': (C.c_int, [p, C.POINTER(C.c_double), C.POINTER(i64)]),
    'sq_model_set_capture': (C.c_int, [p, p, i64]),
    'sq_model_decode': (C.c_int, [p, p, C.c_int, C.c_int, p, p]),
    'sq_fp4_linear_workspace': (i64, [C.c_int, C.c_int, C.c_int]),
    'sq_fp4_linear': (C.c_int, [p, p, p, C.c_int, C.c_int, p, i64, C.c_int, p, i64, p, i64, p]),
    'sq_fp4_linear_static_max_k': (i64, []),
    'sq_fp4_linear_static': (C.c_int, [p, p, p, C.c_int, C.c_int, p, i64, C.c_int, p, i64, p]),
    'sq_gemm_f16': (C.c_int, [p, i64, p, i64, p, i64, C.c_int, C.c_int, C.c_int, p]),
    'sq_device_check': (C.c_int, [p]),
    'sq_set_wait_limit_ns': (C.c_int, [C.c_uint64]),
    'sq_model_create': (C.c_int, [C.POINTER(ModelConfig), C.POINTER(p)]),
    'sq_model_destroy': (C.c_int, [p]),
    'sq_model_set_layer': (C.c_int, [p, C.c_int, C.POINTER(LayerDesc)]),
    'sq_model_set_globals': (C.c_int, [p, C.POINTER(Fp4Matrix), C.POINTER(Fp4Matrix), p]),
    'sq_model_set_adapter': (C.c_int, [p, C.c_int, p, p, p, p, C.c_int]),
    'sq_model_bind_state': (C.c_int, [p, C.c_int, C.c_int, p, p, p, p, p, p, p]),
    'sq_model_reserve': (C.c_int, [p, C.c_int]),
    'sq_model_forward': (C.c_int, [p, p, C.c_int, C.c_int, C.c_int, p, p]),
    'sq_model_mixer_forward': (C.c_int, [p, C.c_int, p, C.c_int, C.c_int, C.c_int, p, p]),
    'sq_model_score': (C.c_int, [p, p, C.c_int, p, p, p]),
    'sq_model_greedy': (C.c_int, [p, p, C.c_int, p, p, p]),
    'sq_model_check': (C.c_int, [p, p]),
}

_lib = None


def load():
    """Load libsq325.so once; raise ImportError if it is absent (no fallback path exists)."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise ImportError(f'{LIB_PATH} is missing: build it with '
                          f'`python mamb2_8b_fp4_recall_sq3.25_b200/build.py` (nvcc, sm_100a)')
    lib = C.CDLL(str(LIB_PATH))
    for name, (res, args) in _PROTOS.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if lib.sq_abi_version() != ABI_VERSION:
        raise ImportError('libsq325.so ABI version differs from the Python binding')
    _lib = lib
    return lib


def exported_symbols():
    return tuple(_PROTOS)


def call(name, *args):
    """Call an entry point; map a non-zero status to the reference's exception class."""
    lib = load()
    status = getattr(lib, name)(*args)
    if status != SQ_OK:
        msg = lib.sq_last_error().decode(errors='replace')
        raise _EXC.get(status, RuntimeError)(f'{name}: {msg}')
    return status


def stream_ptr(stream=None):
    import torch
    s = stream if stream is not None else torch.cuda.current_stream()
    return C.c_void_p(s.cuda_stream)


def ptr(t):
    return C.c_void_p(t.data_ptr()) if t is not None else C.c_void_p(0)
