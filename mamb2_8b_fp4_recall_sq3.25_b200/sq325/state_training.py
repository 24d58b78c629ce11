"""Differentiable training scan over the packed 'sq3p25' state (mamba2_recall/state_training_scan.py).

`scan_training` runs the exact packed forward (sq_sq3p25_scan, bit for bit the deployment
codec's readout) and, in backward, the straight-through derivative of the reference
(:1-12, :175-211): identity on the 80 stored coordinates, zero through the 48 pruned carry
coordinates, scales and rounding detached, current-token readout through all 128.  The
backward (sq_ste_backward) recomputes the dequantized carries, checkpoints the stored
coordinates every `chunk_size` tokens, rebuilds one chunk of history at a time and walks
the adjoint carry backwards; dx / ddt / dB / dC are summed in fp32 in the reference's order
(no atomics: deterministic) and returned in the inputs' dtype.  A, D and dt_bias are
frozen: they receive no gradient.
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _lib
from .state_codec import allocate_state, scan, sq3p25_args

__all__ = ['scan_training', 'training_workspace_bytes']


def _cdiv(a, b):
    return (a + b - 1) // b


class _StateQuantSTE(torch.autograd.Function):
    """Forward: packed sq3p25 scan from a zero state.  Backward: sq_ste_backward
    (state_training_scan.py:175-211)."""

    @staticmethod
    def forward(ctx, x, dt, A, B, C_, D, dt_bias, permutation, chunk_size):
        tensors = tuple(v.contiguous() for v in (x, dt, A, B, C_, D, dt_bias, permutation))
        x, dt, A, B, C_, D, dt_bias, permutation = tensors
        batch, length, heads, dim = x.shape
        state = allocate_state(batch, heads, dim, 128, 'sq3p25', x.device)
        y, _ = scan(x, dt, A, B, C_, D, dt_bias, state, permutation=permutation)
        ctx.save_for_backward(*tensors)
        ctx.chunk_size = chunk_size
        return y

    @staticmethod
    def backward(ctx, grad_y):
        x, dt, A, B, C_, D, dt_bias, permutation = ctx.saved_tensors
        batch, length, heads, dim = x.shape
        k = ctx.chunk_size
        dy = grad_y.to(torch.float16).contiguous()
        dx = torch.empty(x.shape, device=x.device, dtype=torch.float32)
        ddt = torch.empty(dt.shape, device=x.device, dtype=torch.float32)
        db = torch.empty(B.shape, device=x.device, dtype=torch.float32)
        dc = torch.empty(C_.shape, device=x.device, dtype=torch.float32)
        nbytes = int(_lib.load().sq_ste_workspace(batch, length, heads, dim, k))
        work = torch.empty(nbytes, device=x.device, dtype=torch.uint8)
        a = sq3p25_args(x, dt, A, B, C_, D, dt_bias, permutation)
        with torch.cuda.device(x.device):
            _lib.call('sq_ste_backward', C.byref(a), k, dy.data_ptr(), dx.data_ptr(), ddt.data_ptr(),
                      db.data_ptr(), dc.data_ptr(), work.data_ptr(), nbytes, _lib.stream_ptr())
        return dx.to(x.dtype), ddt.to(dt.dtype), None, db.to(B.dtype), dc.to(C_.dtype), None, None, None, None


def scan_training(x, dt, A, B, C_, D, dt_bias, permutation, mode='sq3p25', chunk_size=32):
    """Exact SQ3.25 forward with the approximate straight-through backward
    (state_training_scan.py:224-239).  Whole sequence from a zero state; A, D and dt_bias
    must be frozen; the permutation's contents are the caller's to validate."""
    if mode != 'sq3p25':
        raise ValueError('Training scan supports sq3p25 only; Q8 is excluded')
    if not isinstance(chunk_size, int) or chunk_size < 1 or chunk_size > 256:
        raise ValueError('chunk_size must be an integer in [1,256]')
    if any(v.requires_grad for v in (A, D, dt_bias)):
        raise ValueError('A, D, and dt_bias must be frozen')
    return _StateQuantSTE.apply(x, dt, A, B, C_, D, dt_bias, permutation, chunk_size)


def training_workspace_bytes(batch, length, heads=128, dim=64, groups=8, chunk_size=32):
    """Scratch bytes of one backward, inputs / outputs and the allocator excluded
    (state_training_scan.py:214-221): the checkpoints, one chunk of history and the adjoint
    carry (80 fp32 per row each), plus the fp32 gradient buffers."""
    nc = _cdiv(length, chunk_size)
    carries = batch * (nc + chunk_size + 1) * heads * dim * 80 * 4
    gradients = batch * length * (heads * dim + heads + 2 * groups * 128) * 4
    return {'carry_scratch_bytes': carries, 'gradient_scratch_bytes': gradients,
            'total_scratch_bytes': carries + gradients}
