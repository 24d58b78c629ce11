"""The FP16-state control arm of mamba2_recall/state_codec.py (mode 's16').

Same names, checks and results as the reference module for the s16 mode: `allocate_state`
(:50-62), `scan` (:203-262, with `collect_stats`), `decode_state` / `encode_state_`
(s16 branches of :269-331) and `validate_permutation` (:179-184).  The scan runs in
libsq325.so (sq_s16_scan): fp32 arithmetic, the carry rounded to fp16 after every token,
the readout summed in the reference kernel's order.  The reference's other mode, the fixed
16/64/48 'sq3p25' codec (:105-176), is superseded by the latent codec that the released
model runs (sq325.codec, scripts/fp4_zero_predictor_codec_v1.py) and is not provided here.
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _lib
from .codec import PackedState

MODES = ('s16', 'sq3p25')
RP = 16
S16_TILE = 4
N = 128


def allocate_state(batch, heads, dim, dstate, mode, device):
    if mode not in MODES or dstate != N or min(batch, heads, dim) <= 0:
        raise ValueError('Require s16/sq3p25, dstate=128, and positive geometry')
    if mode != 's16':
        raise ValueError('sq3p25 (the fixed 16/64/48 codec) is superseded by the latent codec: use sq325.codec')
    shape = (batch, heads, dim, dstate)
    return PackedState(mode, {'state': torch.zeros(shape, dtype=torch.float16, device=device)}, shape)


def validate_permutation(permutation, groups):
    if permutation is None or permutation.dtype != torch.uint8 or tuple(permutation.shape) != (groups, N):
        raise ValueError('Permutation must be uint8[groups,128]')
    expected = torch.arange(N, device=permutation.device).expand(groups, N)
    if not torch.equal(permutation.long().sort(-1).values, expected):
        raise ValueError('Each permutation row must contain 0..127 exactly once')


def _validate_state(state, device):
    if not isinstance(state, PackedState) or state.mode not in MODES:
        raise ValueError('Invalid packed state')
    if state.mode != 's16':
        raise ValueError('Only the s16 control state is provided here')
    b, h, p, n = state.shape
    t = state.tensors.get('state')
    if n != N or set(state.tensors) != {'state'}:
        raise ValueError('State keys or geometry differ')
    if tuple(t.shape) != (b, h, p, n) or t.dtype != torch.float16 or t.device != device or not t.is_contiguous():
        raise ValueError('Invalid state buffer state')


@torch.no_grad()
def scan(x, dt, A, B, C_, D, dt_bias, state, permutation=None, collect_stats=False):
    """Mutate the FP16 carry for every token; return (FP16 readouts, statistics or None).

    Inputs: x[B,L,H,P], dt[B,L,H], B/C[B,L,G,128] in FP16; A[H] FP32 negative, D[H] and
    dt_bias[H] FP16/FP32.  collect_stats returns fp32 [B,H,ceil(P/16),128]: per 16-row block
    the sum over tokens and rows of |FP16 carry| (the calibration statistics)."""
    if x.ndim != 4 or x.dtype != torch.float16 or not x.is_cuda:
        raise ValueError('x must be CUDA FP16[batch,tokens,heads,dim]')
    b, length, h, p = x.shape
    if length < 1 or state.shape != (b, h, p, N):
        raise ValueError('Positive sequence length and matching state required')
    _validate_state(state, x.device)
    if B.ndim != 4:
        raise ValueError('B must have four axes')
    g = B.shape[2]
    if g < 1 or h % g:
        raise ValueError('heads must be divisible by B/C groups')
    shapes = ((dt, (b, length, h)), (A, (h,)), (B, (b, length, g, N)), (C_, (b, length, g, N)), (D, (h,)),
              (dt_bias, (h,)))
    for t, shape in shapes:
        if tuple(t.shape) != shape or t.device != x.device:
            raise ValueError('Input device/geometry mismatch')
    if A.dtype != torch.float32 or any(t.dtype != torch.float16 for t in (dt, B, C_)):
        raise ValueError('A must be FP32; dt/B/C must be FP16')
    if any(t.dtype not in (torch.float16, torch.float32) for t in (D, dt_bias)):
        raise ValueError('D and dt_bias must be FP16 or FP32')
    if permutation is not None:
        raise ValueError('s16 does not accept a permutation')
    x, dt, A, B, C_, D, dt_bias = (v.contiguous() for v in (x, dt, A, B, C_, D, dt_bias))
    out = torch.empty_like(x)
    stats = (torch.empty((b, h, (p + RP - 1) // RP, N), device=x.device, dtype=torch.float32)
             if collect_stats else None)
    a = _lib.S16Args()
    a.batch, a.length, a.heads, a.dim, a.groups = b, length, h, p, g
    a.x, a.x_batch_stride, a.x_token_stride = x.data_ptr(), length * h * p, h * p
    a.dt, a.dt_batch_stride, a.dt_token_stride = dt.data_ptr(), length * h, h
    a.A = A.data_ptr()
    a.B, a.b_batch_stride, a.b_token_stride = B.data_ptr(), length * g * N, g * N
    a.C, a.c_batch_stride, a.c_token_stride = C_.data_ptr(), length * g * N, g * N
    a.D, a.d_is_f32 = D.data_ptr(), int(D.dtype == torch.float32)
    a.dt_bias, a.dt_bias_is_f32 = dt_bias.data_ptr(), int(dt_bias.dtype == torch.float32)
    a.state = state.tensors['state'].data_ptr()
    a.y, a.y_batch_stride, a.y_token_stride = out.data_ptr(), length * h * p, h * p
    a.stats = stats.data_ptr() if stats is not None else None
    with torch.cuda.device(x.device):
        _lib.call('sq_s16_scan', C.byref(a), _lib.stream_ptr())
    return out, stats


@torch.no_grad()
def decode_state(state, permutation=None):
    """s16: the carry in original coordinates as fp32."""
    if state.mode != 's16':
        raise ValueError('Unsupported mode')
    return state.tensors['state'].float()


@torch.no_grad()
def encode_state_(state, dense_permuted):
    """s16: copy a finite dense carry of the state's shape into it (fp16)."""
    if tuple(dense_permuted.shape) != state.shape or not bool(torch.isfinite(dense_permuted).all()):
        raise ValueError('Diagnostic input must be finite and match state shape')
    if state.mode != 's16':
        raise ValueError('Unsupported mode')
    state.tensors['state'].copy_(dense_permuted)
    return state
