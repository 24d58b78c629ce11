"""SQ3.25 latent-codec host API: reference-shaped wrappers over the C ABI.

Mirrors scripts/fp4_zero_predictor_codec_v1.py (layout_descriptor :28, allocate_state
:39, validate_state :52, scan :184) and the PackedState container of
mamba2_recall/state_codec.py:29-48.  Buffers are the reference's six per-layer
tensors (lo, hi, q4, latent, s8, s4) with identical shapes and dtypes, so a state
produced here can be read by the reference and vice versa.  All arithmetic runs in
libsq325.so on the GPU.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import torch

from . import _lib

# The seven released layouts; base counts from scripts/w4_state_repair_codec_v2.py:22-28.
BASE_COUNTS = {
    '32_32_64': (32, 32, 64), '16_64_48': (16, 64, 48), '8_80_40': (8, 80, 40),
    '24_48_56': (24, 48, 56), '36_24_68': (36, 24, 68), '40_16_72': (40, 16, 72),
    '44_8_76': (44, 8, 76),
}
LAYOUTS = tuple(BASE_COUNTS)
ROW_BYTES = 52
CACHE_BYTES = 28499968
TABLE_BYTES = 57344
RP = 16


def layout_index(layout):
    if layout not in BASE_COUNTS:
        raise ValueError('Unknown fixed W4 state repair tier layout')
    return LAYOUTS.index(layout)


def layout_descriptor(layout):
    """Tier counts after the latent shift: 4 INT4 coordinates join the zero tier (:28-36)."""
    n8, n4, nz = BASE_COUNTS[layout] if layout in BASE_COUNTS else (None, None, None)
    if n8 is None:
        raise ValueError('Unknown fixed W4 state repair tier layout')
    n4, nz = n4 - 4, nz + 4
    if n4 < 4 or n8 + n4 + nz != 128 or n8 + n4 // 2 + 2 + 4 != 52:
        raise ValueError('Latent tier layout violates same-byte geometry')
    return dict(layout=layout, n8=n8, n4=n4, nzero=nz, payload_bytes=48, scale_bytes=4, row_bytes=52,
                latent_coefficients=2, latent_dtype='torch.float8_e4m3fn',
                tensor_widths=dict(lo=n8 // 2, hi=n8 // 2, q4=n4 // 2, latent=2))


@dataclass
class PackedState:
    """Same container as mamba2_recall/state_codec.py:29-48."""
    mode: str
    tensors: dict
    shape: tuple

    @property
    def nbytes(self):
        storages = {(t.device, t.untyped_storage().data_ptr()): t.untyped_storage().nbytes()
                    for t in self.tensors.values()}
        return sum(storages.values())

    def clone(self):
        return PackedState(self.mode, {k: v.clone() for k, v in self.tensors.items()}, self.shape)

    def zero_(self):
        for v in self.tensors.values():
            v.zero_()
        return self


def allocate_state(batch, heads, dim, dstate, device, *, layout):
    spec = layout_descriptor(layout)
    if dstate != 128 or any(type(v) is not int or v <= 0 for v in (batch, heads, dim)):
        raise ValueError('Positive state geometry and dstate=128 required')
    base = (batch, heads, dim)
    tensors = {name: torch.zeros((*base, width), device=device,
                                 dtype=torch.float8_e4m3fn if name == 'latent' else torch.uint8)
               for name, width in spec['tensor_widths'].items()}
    tensors.update({name: torch.zeros(base, device=device, dtype=torch.float16) for name in ('s8', 's4')})
    return PackedState('latent_fp8_' + layout, tensors, (*base, 128))


def validate_state(state, device, layout):
    """Exact inventory, shapes, dtypes, contiguity, no aliasing, 52 B/row (:52-73)."""
    spec = layout_descriptor(layout)
    if (state.mode != 'latent_fp8_' + layout or len(state.shape) != 4 or state.shape[-1] != 128 or
            set(state.tensors) != {'lo', 'hi', 'q4', 'latent', 's8', 's4'}):
        raise ValueError('Latent packed state mode/inventory differs')
    base = tuple(state.shape[:3])
    if min(base) <= 0:
        raise ValueError('Invalid latent state geometry')
    storages = set()
    for name, value in state.tensors.items():
        shape = base + ((spec['tensor_widths'][name],) if name in spec['tensor_widths'] else ())
        dtype = (torch.float16 if name in ('s8', 's4') else
                 torch.float8_e4m3fn if name == 'latent' else torch.uint8)
        if (tuple(value.shape) != shape or value.dtype != dtype or value.device != torch.device(device) or
                not value.is_contiguous() or value.storage_offset() != 0 or
                value.untyped_storage().nbytes() != value.numel() * value.element_size()):
            raise ValueError('Latent packed state backing allocation differs: ' + name)
        storages.add(value.untyped_storage().data_ptr())
    if len(storages) != 6 or state.nbytes != base[0] * base[1] * base[2] * 52:
        raise ValueError('Latent state aliases or exceeds 52-byte row')
    return True


def _state_ptrs(state):
    t = state.tensors
    return [_lib.ptr(t[k]) for k in ('lo', 'hi', 'q4', 'latent', 's8', 's4')]


@torch.no_grad()
def scan(x, dt, A, B, C_, D, dt_bias, state, permutation, basis, latent_scale, predictor, *, layout,
         fused=False):
    """Mutate `state` for every token and return (y fp16 [batch,L,H,P], None).

    Same contract and checks as the reference scan (:184-236); the predictor readout
    correction is computed on the device.  By default a workspace from the torch allocator
    selects the two-kernel path (group-level dots once per group); fused=True runs the single
    fused kernel instead.  Both give identical bytes.
    """
    spec = layout_descriptor(layout)
    if x.ndim != 4 or x.dtype != torch.float16 or not x.is_cuda:
        raise ValueError('x must be CUDA FP16 [batch,tokens,heads,dim]')
    batch, length, heads, dim = x.shape
    if length < 1 or dim % RP or state.shape != (batch, heads, dim, 128):
        raise ValueError('Positive sequence and matching latent state required')
    validate_state(state, x.device, layout)
    groups = B.shape[2]
    expected = ((dt, (batch, length, heads)), (A, (heads,)), (B, (batch, length, groups, 128)),
                (C_, (batch, length, groups, 128)), (D, (heads,)), (dt_bias, (heads,)))
    for value, shape in expected:
        if tuple(value.shape) != shape or value.device != x.device:
            raise ValueError('Latent scan input geometry/device differs')
    if (heads % groups or A.dtype != torch.float32 or
            any(v.dtype != torch.float16 for v in (dt, B, C_)) or
            any(v.dtype not in (torch.float16, torch.float32) for v in (D, dt_bias))):
        raise ValueError('Latent scan dtype/grouping differs')
    if (permutation.dtype != torch.uint8 or tuple(permutation.shape) != (groups, 128) or
            permutation.device != x.device or
            basis.dtype != torch.float16 or tuple(basis.shape) != (groups, spec['nzero'], 2) or
            basis.device != x.device or
            latent_scale.dtype != torch.float16 or tuple(latent_scale.shape) != (groups, 2) or
            latent_scale.device != x.device or not bool(torch.isfinite(basis).all()) or
            not bool(torch.isfinite(latent_scale).all()) or not bool((latent_scale > 0).all())):
        raise ValueError('Latent static basis/scales differ')
    features = spec['n8'] + spec['n4'] + 2
    if (predictor.dtype != torch.float16 or tuple(predictor.shape) != (groups, features, spec['nzero']) or
            predictor.device != x.device or not predictor.is_contiguous() or
            not bool(torch.isfinite(predictor).all())):
        raise ValueError('Static zero-tier predictor differs')
    x, dt, A, B, C_, D, dt_bias, permutation, basis, latent_scale = (
        v.contiguous() for v in (x, dt, A, B, C_, D, dt_bias, permutation, basis, latent_scale))
    y = torch.empty_like(x)
    a = _lib.ScanArgs()
    a.batch, a.length, a.heads, a.dim, a.groups, a.layout = batch, length, heads, dim, groups, layout_index(layout)
    a.x, a.x_batch_stride, a.x_token_stride = x.data_ptr(), length * heads * dim, heads * dim
    a.dt, a.dt_batch_stride, a.dt_token_stride = dt.data_ptr(), length * heads, heads
    a.A = A.data_ptr()
    a.B, a.b_batch_stride, a.b_token_stride = B.data_ptr(), length * groups * 128, groups * 128
    a.C, a.c_batch_stride, a.c_token_stride = C_.data_ptr(), length * groups * 128, groups * 128
    a.D, a.d_is_f32 = D.data_ptr(), int(D.dtype == torch.float32)
    a.dt_bias, a.dt_bias_is_f32 = dt_bias.data_ptr(), int(dt_bias.dtype == torch.float32)
    a.permutation, a.basis, a.latent_scale, a.predictor = (permutation.data_ptr(), basis.data_ptr(),
                                                           latent_scale.data_ptr(), predictor.data_ptr())
    t = state.tensors
    a.lo, a.hi, a.q4, a.latent, a.s8, a.s4 = (t[k].data_ptr() for k in ('lo', 'hi', 'q4', 'latent', 's8', 's4'))
    a.y, a.y_batch_stride, a.y_token_stride = y.data_ptr(), length * heads * dim, heads * dim
    ws = None
    if not fused:
        need = _lib.load().sq_scan_workspace(batch, length, heads, groups, layout_index(layout))
        if need > 0:
            ws = torch.empty(need, device=x.device, dtype=torch.uint8)
            a.workspace, a.workspace_bytes = ws.data_ptr(), need
    with torch.cuda.device(x.device):
        _lib.call('sq_scan', C.byref(a), _lib.stream_ptr())
    return y, None


@torch.no_grad()
def scan_with_conv(xbc, dt, A, D, dt_bias, state, permutation, basis, latent_scale, predictor, conv_weight,
                   conv_bias, conv_ring, position, *, layout, fused=False):
    """Causal conv + codec scan in one pass (the conv of mamba2_recall/state_quant.py:283-317
    followed by `scan`, as PredictorState._forward runs them, :341-352).

    xbc fp16 [batch, L, 10240] holds the RAW in_proj xBC columns (x | B | C); dt fp16
    [batch, L, 128].  conv_ring fp16 [batch, 4, 10240] is the conv cache in ring order (slot
    = absolute position % 4).  position == 0 runs a prefill from a reset ring (conv1d
    numerics); position > 0 with L == 1 runs the one-token step numerics.  Mutates `state`
    and `conv_ring`; returns (y fp16 [batch, L, 128, 64], None)."""
    spec = layout_descriptor(layout)
    if xbc.ndim != 3 or xbc.dtype != torch.float16 or not xbc.is_cuda or xbc.shape[2] != 10240 or \
            xbc.stride(2) != 1:
        raise ValueError('xbc must be CUDA FP16 [batch,tokens,10240] with unit channel stride')
    batch, length, _ = xbc.shape
    heads, dim, groups = 128, 64, 8
    if state.shape != (batch, heads, dim, 128):
        raise ValueError('Positive sequence and matching latent state required')
    validate_state(state, xbc.device, layout)
    if tuple(conv_ring.shape) != (batch, 4, 10240) or conv_ring.dtype != torch.float16 or \
            not conv_ring.is_contiguous() or conv_ring.device != xbc.device:
        raise ValueError('conv_ring must be contiguous CUDA FP16 [batch,4,10240]')
    if tuple(conv_weight.shape) != (10240, 4) or tuple(conv_bias.shape) != (10240,) or \
            conv_weight.dtype != torch.float16 or conv_bias.dtype != torch.float16:
        raise ValueError('conv weight [10240,4] and bias [10240] must be FP16')
    if type(position) is not int or position < 0 or (position > 0 and length != 1):
        raise ValueError('position 0 (prefill from a reset ring) or a one-token step required')
    if tuple(dt.shape) != (batch, length, heads) or dt.dtype != torch.float16:
        raise ValueError('dt must be FP16 [batch,tokens,128]')
    dt, A, D, dt_bias, permutation, basis, latent_scale, predictor, conv_weight, conv_bias = (
        v.contiguous() for v in (dt, A, D, dt_bias, permutation, basis, latent_scale, predictor, conv_weight,
                                 conv_bias))
    y = torch.empty((batch, length, heads, dim), device=xbc.device, dtype=torch.float16)
    a = _lib.ScanArgs()
    a.batch, a.length, a.heads, a.dim, a.groups, a.layout = batch, length, heads, dim, groups, layout_index(layout)
    sb, st = xbc.stride(0), xbc.stride(1)
    base = xbc.data_ptr()
    a.x, a.x_batch_stride, a.x_token_stride = base, sb, st
    a.B, a.b_batch_stride, a.b_token_stride = base + 8192 * 2, sb, st
    a.C, a.c_batch_stride, a.c_token_stride = base + 9216 * 2, sb, st
    a.dt, a.dt_batch_stride, a.dt_token_stride = dt.data_ptr(), length * heads, heads
    a.A = A.data_ptr()
    a.D, a.d_is_f32 = D.data_ptr(), int(D.dtype == torch.float32)
    a.dt_bias, a.dt_bias_is_f32 = dt_bias.data_ptr(), int(dt_bias.dtype == torch.float32)
    a.permutation, a.basis, a.latent_scale, a.predictor = (permutation.data_ptr(), basis.data_ptr(),
                                                           latent_scale.data_ptr(), predictor.data_ptr())
    t = state.tensors
    a.lo, a.hi, a.q4, a.latent, a.s8, a.s4 = (t[k].data_ptr() for k in ('lo', 'hi', 'q4', 'latent', 's8', 's4'))
    a.y, a.y_batch_stride, a.y_token_stride = y.data_ptr(), length * heads * dim, heads * dim
    ws = None
    if not fused:          # the two-kernel path (prefill or one-token step); fused: one kernel
        need = _lib.load().sq_scan_workspace(batch, length, heads, groups, layout_index(layout))
        ws = torch.empty(need, device=xbc.device, dtype=torch.uint8)
        a.workspace, a.workspace_bytes = ws.data_ptr(), need
    c = _lib.ConvArgs(conv_weight.data_ptr(), conv_bias.data_ptr(), conv_ring.data_ptr(), 4 * 10240, position)
    with torch.cuda.device(xbc.device):
        _lib.call('sq_scan_conv', C.byref(a), C.byref(c), _lib.stream_ptr())
    return y, None


@torch.no_grad()
def decode_state(state, latent_scale, *, layout):
    """Packed rows -> (tiers fp32 [B,H,P,n8+n4] in tier order, z fp32 [B,H,P,2])."""
    spec = layout_descriptor(layout)
    validate_state(state, state.tensors['lo'].device, layout)
    b, h, pdim, _ = state.shape
    groups = latent_scale.shape[0]
    dev = state.tensors['lo'].device
    tiers = torch.empty((b, h, pdim, spec['n8'] + spec['n4']), device=dev, dtype=torch.float32)
    z = torch.empty((b, h, pdim, 2), device=dev, dtype=torch.float32)
    ls = latent_scale.to(device=dev, dtype=torch.float16).contiguous()
    with torch.cuda.device(dev):
        _lib.call('sq_state_decode', layout_index(layout), b, h, pdim, groups, *_state_ptrs(state),
                  _lib.ptr(ls), _lib.ptr(tiers), _lib.ptr(z), _lib.stream_ptr())
    return tiers, z


@torch.no_grad()
def encode_state_(state, tiers, z=None, latent_scale=None, *, layout, mode='kernel'):
    """Write tier values (+ latent z) into `state`.

    mode='kernel': the production requant (fp16 scale from max/L, exact division,
    round half away, clip; latent e4m3(clamp(z/ls))).  mode='diagnostic': the
    reference's encode_state_ initializer (fp32 denominators, latent bytes 0).
    """
    spec = layout_descriptor(layout)
    validate_state(state, state.tensors['lo'].device, layout)
    b, h, pdim, _ = state.shape
    dev = state.tensors['lo'].device
    tiers = tiers.to(device=dev, dtype=torch.float32).contiguous()
    if tuple(tiers.shape) != (b, h, pdim, spec['n8'] + spec['n4']) or not bool(torch.isfinite(tiers).all()):
        raise ValueError('Tier values must be finite [batch,heads,dim,n8+n4]')
    m = {'kernel': 0, 'diagnostic': 1}[mode]
    if m == 0:
        z = z.to(device=dev, dtype=torch.float32).contiguous()
        ls = latent_scale.to(device=dev, dtype=torch.float16).contiguous()
        groups = ls.shape[0]
    else:
        z = ls = None
        groups = 1 if latent_scale is None else latent_scale.shape[0]
    with torch.cuda.device(dev):
        _lib.call('sq_state_encode', layout_index(layout), b, h, pdim, groups, m, _lib.ptr(tiers), _lib.ptr(z),
                  _lib.ptr(ls), *_state_ptrs(state), _lib.stream_ptr())
    return state
