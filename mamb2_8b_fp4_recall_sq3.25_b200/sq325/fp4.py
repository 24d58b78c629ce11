"""Packed-resident FP4-E2M1 G16 weights (host side).

Format as mamba2_recall/fp4.py and fp4_checkpoint.py store it: `codes` u8[rows, cols/2]
(low nibble = even column), `block_scale_bytes` u8[rows, cols/16] (E4M3FN bytes) and one
fp32 `global_scale`.  The bytes stay resident on the GPU; decode happens inside the
kernels (libsq325.so), bit-exact with FP16(FP32(FP32(code*block)*global))
(mamba2_recall/fp4.py:151-154).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib

FORMAT = 'fp4_g16_e4m3'
GROUP_SIZE = 16
E2M1_MAGNITUDES = (0., .5, 1., 1.5, 2., 3., 4., 6.)


@dataclass
class Fp4Tensor:
    codes: torch.Tensor              # u8 [rows, cols/2] (device)
    block_scale_bytes: torch.Tensor  # u8 [rows, cols/16] (device)
    global_scale: torch.Tensor       # f32 [1] (device)
    shape: tuple

    @property
    def rows(self):
        return self.shape[0]

    @property
    def cols(self):
        return self.shape[1]

    @property
    def nbytes(self):
        return self.codes.numel() + self.block_scale_bytes.numel() + 4

    def cabi(self):
        return _lib.Fp4Matrix(self.codes.data_ptr(), self.block_scale_bytes.data_ptr(),
                              self.global_scale.data_ptr(), self.rows, self.cols)

    def to_numpy(self):
        return (self.codes.cpu().numpy(), self.block_scale_bytes.cpu().numpy(),
                np.float32(self.global_scale.cpu().item()))


def from_packet(packet, device='cuda'):
    """Accept the reference's packet dict (fp4.quantize_chunk / load path) or raw arrays."""
    if packet.get('format', FORMAT) != FORMAT or packet.get('group_size', 16) != 16:
        raise ValueError('Only the fp4_g16_e4m3 format is supported')
    rows, cols = packet['shape']
    if cols % 16:
        raise ValueError('Production FP4 width is not divisible by 16')
    codes = torch.as_tensor(packet['packed']).to(device=device, dtype=torch.uint8).contiguous()
    scales = packet['scales']
    scales = scales.view(torch.uint8) if isinstance(scales, torch.Tensor) and scales.dtype == torch.float8_e4m3fn \
        else torch.as_tensor(scales)
    scales = scales.to(device=device, dtype=torch.uint8).contiguous()
    g = torch.as_tensor(packet['global_scale'], dtype=torch.float32).reshape(1).to(device)
    if tuple(codes.shape) != (rows, cols // 2) or tuple(scales.shape) != (rows, cols // 16):
        raise ValueError('Packed geometry differs')
    if not bool(torch.isfinite(g).all()) or not bool((g > 0).all()):
        raise ValueError('Global scale must be finite and positive')
    return Fp4Tensor(codes, scales, g, (rows, cols))


def validate(w):
    """decode_packet's content checks (mamba2_recall/fp4.py:235-249) on the device: ValueError
    for a negative / NaN block scale, a nonzero code in a zero-scale group, or a weight that
    decodes to a nonfinite fp16 value (the reference's messages)."""
    with torch.cuda.device(w.codes.device):
        _lib.call('sq_fp4_validate', _lib.ptr(w.codes), _lib.ptr(w.block_scale_bytes), _lib.ptr(w.global_scale),
                  w.rows, w.cols, _lib.stream_ptr())
    return w


@torch.no_grad()
def decode_packet(w):
    """Bit-exact FP16 decode of a packed matrix (replaces fp4.decode_packet), with the
    reference's checks first."""
    if isinstance(w, dict):
        w = from_packet(w)
    validate(w)
    out = torch.empty(w.shape, device=w.codes.device, dtype=torch.float16)
    with torch.cuda.device(w.codes.device):
        _lib.call('sq_fp4_decode', _lib.ptr(w.codes), _lib.ptr(w.block_scale_bytes), _lib.ptr(w.global_scale),
                  w.rows, w.cols, _lib.ptr(out), w.cols, _lib.stream_ptr())
    return out


_workspace = {}


@torch.no_grad()
def linear(w, x):
    """y = x @ decode(w).T with fp32 accumulation and fp16 output (the nn.Linear the reference runs)."""
    if x.dtype != torch.float16 or x.shape[-1] != w.cols or not x.is_cuda:
        raise ValueError('Input must be CUDA FP16 [..., cols]')
    lead = x.shape[:-1]
    x2 = x.reshape(-1, w.cols).contiguous()
    m = x2.shape[0]
    y = torch.empty((m, w.rows), device=x.device, dtype=torch.float16)
    need = _lib.load().sq_fp4_linear_workspace(m, w.rows, w.cols)
    ws = None
    if need:
        key = x.device
        ws = _workspace.get(key)
        if ws is None or ws.numel() < need:
            ws = torch.empty(need, device=x.device, dtype=torch.uint8)
            _workspace[key] = ws
    with torch.cuda.device(x.device):
        _lib.call('sq_fp4_linear', _lib.ptr(w.codes), _lib.ptr(w.block_scale_bytes), _lib.ptr(w.global_scale),
                  w.rows, w.cols, _lib.ptr(x2), w.cols, m, _lib.ptr(y), w.rows,
                  _lib.ptr(ws) if ws is not None else C.c_void_p(0), int(ws.numel()) if ws is not None else 0,
                  _lib.stream_ptr())
    return y.reshape(*lead, w.rows)


def synthetic_arrays(rows, cols, rng, mu=-4.0, sigma=0.5):
    """Config-2 weights on the host: codes uniform over 16 values, effective scales
    logNormal(mu, sigma) realised as global = max_eff/448, block = E4M3(eff/global)."""
    codes = rng.integers(0, 256, size=(rows, cols // 2), dtype=np.uint8)
    eff = np.exp(rng.normal(mu, sigma, size=(rows, cols // 16))).astype(np.float32)
    g = np.float32(eff.max() / 448.0)
    blocks = torch.from_numpy(eff / g).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    return codes, blocks, g


@torch.no_grad()
def synthetic(rows, cols, generator, device='cuda', mu=-4.0, sigma=0.5, row_mu=None):
    """Config-2 weights generated on the device from a seeded torch.Generator; `row_mu`
    (optional tensor [rows]) overrides the log-normal mean per output row."""
    codes = torch.randint(0, 256, (rows, cols // 2), generator=generator, device=device, dtype=torch.uint8)
    n = torch.empty((rows, cols // 16), device=device, dtype=torch.float32).normal_(0.0, 1.0, generator=generator)
    mus = mu if row_mu is None else row_mu.to(device=device, dtype=torch.float32)[:, None]
    eff = torch.exp(mus + sigma * n)
    g = (eff.max() / 448.0).reshape(1).float()
    blocks = (eff / g).to(torch.float8_e4m3fn).view(torch.uint8).contiguous()
    return Fp4Tensor(codes, blocks, g, (rows, cols))


def from_arrays(codes, blocks, g, device='cuda'):
    rows = codes.shape[0]
    cols = codes.shape[1] * 2
    return Fp4Tensor(torch.from_numpy(np.ascontiguousarray(codes)).to(device),
                     torch.from_numpy(np.ascontiguousarray(blocks)).to(device),
                     torch.tensor([float(g)], dtype=torch.float32, device=device), (rows, cols))
