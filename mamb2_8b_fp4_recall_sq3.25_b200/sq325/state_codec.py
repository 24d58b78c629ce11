"""The two state modes of mamba2_recall/state_codec.py: the FP16-state control arm 's16'
and the fixed-split packed codec 'sq3p25'.

Same names, checks and results as the reference module: `allocate_state` (:50-62), `scan`
(:203-262, with `collect_stats` for s16), `decode_state` / `encode_state_` (:265-331) and
`validate_permutation` (:179-184).
  s16     sq_s16_scan: fp32 arithmetic, the carry rounded to fp16 after every token, the
          readout summed in the reference kernel's order.
  sq3p25  sq_sq3p25_scan: per row 16 INT8 + 64 INT4 stored coordinates (the group's
          permutation orders them) and 48 pruned ones that read out only the current token,
          52 bytes (lo / hi u8[8], q4 u8[32], s8 / s4 fp16); the codec the training scan
          (sq325.state_training, mamba2_recall/state_training_scan.py) runs.  The released
          model runs the latent codec instead (sq325.codec).
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
    shape = (batch, heads, dim, dstate)
    if mode == 's16':
        return PackedState(mode, {'state': torch.zeros(shape, dtype=torch.float16, device=device)}, shape)
    tensors = {key: torch.zeros((batch, heads, dim, size), dtype=torch.uint8, device=device)
               for key, size in (('lo', 8), ('hi', 8), ('q4', 32))}
    tensors.update({key: torch.zeros((batch, heads, dim), dtype=torch.float16, device=device) for key in ('s8', 's4')})
    return PackedState(mode, tensors, shape)


def validate_permutation(permutation, groups):
    if permutation is None or permutation.dtype != torch.uint8 or tuple(permutation.shape) != (groups, N):
        raise ValueError('Permutation must be uint8[groups,128]')
    expected = torch.arange(N, device=permutation.device).expand(groups, N)
    if not torch.equal(permutation.long().sort(-1).values, expected):
        raise ValueError('Each permutation row must contain 0..127 exactly once')


def _validate_state(state, device):
    if not isinstance(state, PackedState) or state.mode not in MODES:
        raise ValueError('Invalid packed state')
    b, h, p, n = state.shape
    spec = ({'state': (state.shape, torch.float16)} if state.mode == 's16' else {
        'lo': ((b, h, p, 8), torch.uint8), 'hi': ((b, h, p, 8), torch.uint8),
        'q4': ((b, h, p, 32), torch.uint8), 's8': ((b, h, p), torch.float16),
        's4': ((b, h, p), torch.float16)})
    if n != N or set(state.tensors) != set(spec):
        raise ValueError('State keys or geometry differ')
    for key, (shape, dtype) in spec.items():
        t = state.tensors[key]
        if tuple(t.shape) != tuple(shape) or t.dtype != dtype or t.device != device or not t.is_contiguous():
            raise ValueError(f'Invalid state buffer {key}')


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
    if collect_stats and state.mode != 's16':
        raise ValueError('Calibration statistics require s16')
    if state.mode == 'sq3p25':
        if permutation is None or permutation.dtype != torch.uint8 or tuple(permutation.shape) != (g, N) or \
                permutation.device != x.device:
            raise ValueError('SQ requires CUDA uint8[groups,128] permutation')
        return _sq3p25_scan(x, dt, A, B, C_, D, dt_bias, state, permutation.contiguous()), None
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


def sq3p25_args(x, dt, A, B, C_, D, dt_bias, permutation, state=None, y=None):
    """ctypes argument block of sq_sq3p25_scan / sq_ste_backward over contiguous inputs."""
    b, length, h, p = x.shape
    g = B.shape[2]
    a = _lib.Sq3p25Args()
    a.batch, a.length, a.heads, a.dim, a.groups = b, length, h, p, g
    a.x, a.x_batch_stride, a.x_token_stride = x.data_ptr(), length * h * p, h * p
    a.dt, a.dt_batch_stride, a.dt_token_stride = dt.data_ptr(), length * h, h
    a.A = A.data_ptr()
    a.B, a.b_batch_stride, a.b_token_stride = B.data_ptr(), length * g * N, g * N
    a.C, a.c_batch_stride, a.c_token_stride = C_.data_ptr(), length * g * N, g * N
    a.D, a.d_is_f32 = D.data_ptr(), int(D.dtype == torch.float32)
    a.dt_bias, a.dt_bias_is_f32 = dt_bias.data_ptr(), int(dt_bias.dtype == torch.float32)
    a.permutation = permutation.data_ptr()
    if state is not None:
        t = state.tensors
        a.lo, a.hi, a.q4, a.s8, a.s4 = (t[k].data_ptr() for k in ('lo', 'hi', 'q4', 's8', 's4'))
    if y is not None:
        a.y, a.y_batch_stride, a.y_token_stride = y.data_ptr(), length * h * p, h * p
    return a


def _sq3p25_scan(x, dt, A, B, C_, D, dt_bias, state, permutation):
    x, dt, A, B, C_, D, dt_bias = (v.contiguous() for v in (x, dt, A, B, C_, D, dt_bias))
    if x.shape[3] > 128:
        raise ValueError('sq3p25 supports head dims up to 128')
    out = torch.empty_like(x)
    a = sq3p25_args(x, dt, A, B, C_, D, dt_bias, permutation, state, out)
    with torch.cuda.device(x.device):
        _lib.call('sq_sq3p25_scan', C.byref(a), _lib.stream_ptr())
    return out


def _unpack_nibbles(value):
    return torch.stack((value & 15, (value >> 4) & 15), -1).flatten(-2).to(torch.int32)


@torch.no_grad()
def decode_state(state, permutation=None):
    """Diagnostic full FP32 decode.  s16: the carry.  sq3p25: the permuted coordinates (16 INT8,
    64 INT4, 48 zeros), or the original coordinates when a [G,128] permutation is given."""
    if state.mode == 's16':
        return state.tensors['state'].float()
    if state.mode != 'sq3p25':
        raise ValueError('Unsupported mode')
    t = state.tensors
    ub = (_unpack_nibbles(t['hi']) << 4) | _unpack_nibbles(t['lo'])
    q8 = ub - (ub > 127).to(torch.int32) * 256
    q4 = _unpack_nibbles(t['q4'])
    q4 = q4 - (q4 > 7).to(torch.int32) * 16
    values = torch.cat((q8.float() * t['s8'].float()[..., None], q4.float() * t['s4'].float()[..., None],
                        torch.zeros((*state.shape[:-1], 48), device=q8.device)), -1)
    if permutation is None:
        return values
    g = permutation.shape[0]
    validate_permutation(permutation, g)
    b, h, p, _ = state.shape
    if h % g:
        raise ValueError('Invalid grouping')
    indices = permutation.long().repeat_interleave(h // g, 0)[None, :, None, :].expand(b, h, p, N)
    return torch.zeros_like(values).scatter_(-1, indices, values)


@torch.no_grad()
def encode_state_(state, dense_permuted):
    """Diagnostic initializer.  s16: copy a finite dense carry (fp16).  sq3p25: coordinates
    already in permuted order; INT8 / INT4 codes with fp32 denominators max(|v|max / limit,
    1e-8), round half away, clip; scales stored as fp16 (not the runtime rule)."""
    if tuple(dense_permuted.shape) != state.shape or not bool(torch.isfinite(dense_permuted).all()):
        raise ValueError('Diagnostic input must be finite and match state shape')
    if state.mode == 's16':
        state.tensors['state'].copy_(dense_permuted)
        return state
    if state.mode != 'sq3p25':
        raise ValueError('Unsupported mode')

    v = dense_permuted.float()
    parts = []
    for block, limit in ((v[..., :16], 127), (v[..., 16:80], 7)):
        den = torch.clamp_min(block.abs().amax(-1) / limit, 1e-8)
        parts.append((block, den, limit))
    if not all(bool(torch.isfinite(den.half()).all()) for _, den, _ in parts):
        raise ValueError('Scale exceeds FP16 range')
    codes = []
    for block, den, limit in parts:
        z = block / den[..., None]
        codes.append(torch.clamp(torch.sign(z) * torch.floor(z.abs() + 0.5), -limit, limit).to(torch.int32))

    def nibbles(q):
        q = (q & 15).to(torch.uint8)
        return q[..., 0::2] | (q[..., 1::2] << 4)

    (q8, q4), (s8, s4) = codes, (parts[0][1], parts[1][1])
    t = state.tensors
    t['lo'].copy_(nibbles(q8))
    t['hi'].copy_(nibbles(q8 >> 4))
    t['q4'].copy_(nibbles(q4))
    t['s8'].copy_(s8)
    t['s4'].copy_(s4)
    return state
