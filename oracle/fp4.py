"""numpy restatement of the FP4-E2M1 G16 weight format (CPU, test only).

  e2m1 values          mamba2_recall/fp4.py:100-103 (levels [0,.5,1,1.5,2,3,4,6], bit 3 = sign)
  encode_e2m1          mamba2_recall/fp4.py:85-91 (bucketize on .25,.75,1.25,1.75,2.5,3.5,5;
                       exact ties go to the even code; zero is never negative)
  pack / unpack        mamba2_recall/fp4.py:118-130 (low nibble = even column)
  decode               mamba2_recall/fp4.py:151-154:
                       FP16(FP32(FP32(code*block)*global))
  synthetic_matrix     the build's config-2 generator: codes uniform over the 16 values,
                       effective per-16 scale ~ logNormal(mu, sigma) realised as
                       global = max_eff / 448, block = E4M3(eff / global).
"""
from __future__ import annotations

import numpy as np

from .codec import E4M3_VALUES, f32_to_e4m3

E2M1 = np.array([0., .5, 1., 1.5, 2., 3., 4., 6.], np.float32)
BOUNDS = np.array([.25, .75, 1.25, 1.75, 2.5, 3.5, 5.], np.float32)


def e2m1_values(codes):
    c = np.asarray(codes).astype(np.int64)
    v = E2M1[c & 7]
    return np.where(c & 8, -v, v).astype(np.float32)


def encode_e2m1(values):
    v = np.asarray(values, np.float32)
    mag = np.abs(v)
    code = np.searchsorted(BOUNDS, mag, side='left')          # bucketize(right=False)
    tie = (code < 7) & (mag == BOUNDS[np.minimum(code, 6)]) & ((code & 1) != 0)
    code = (code + tie).astype(np.uint8)
    return code | (((v < 0) & (code != 0)).astype(np.uint8) << 3)


def unpack(codes_packed, cols):
    p = np.asarray(codes_packed, np.uint8)
    out = np.stack((p & 15, p >> 4), -1).reshape(p.shape[0], -1)
    return out[:, :cols]


def pack(codes):
    c = np.asarray(codes, np.uint8)
    return (c[:, 0::2] | (c[:, 1::2] << 4)).astype(np.uint8)


# value pair of every code byte: (low nibble = even column, high nibble = odd column)
_PAIR_VALUES = np.stack((np.where(np.arange(256) & 8, -1, 1) * E2M1[np.arange(256) & 7],
                         np.where((np.arange(256) >> 4) & 8, -1, 1) * E2M1[(np.arange(256) >> 4) & 7]),
                        -1).astype(np.float32)


def decode(codes_packed, block_scale_bytes, global_scale, cols=None):
    """-> fp16 [rows, cols], bit-exact with the reference decode.

    Same three roundings as the reference (fp4.py:151-154): code * block is exact in
    fp32, the product with the fp32 global rounds once to fp32, then once to fp16.  Runs
    as torch CPU table lookups and elementwise products (multi-threaded)."""
    import torch
    p = torch.from_numpy(np.ascontiguousarray(codes_packed, np.uint8))
    rows = p.shape[0]
    cols = cols or p.shape[1] * 2
    pairs = torch.from_numpy(_PAIR_VALUES)[p.long()].reshape(rows, -1)[:, :cols]        # [rows, cols] fp32
    blocks = torch.from_numpy(E4M3_VALUES)[torch.from_numpy(np.ascontiguousarray(block_scale_bytes, np.uint8)).long()]
    vals = (pairs.reshape(rows, -1, 16) * blocks[:, :, None]).reshape(rows, cols)
    vals = vals * torch.tensor(np.float32(global_scale), dtype=torch.float32)
    return vals.half().numpy()


def synthetic_matrix(rows, cols, rng, mu=-4.0, sigma=0.5, row_mu=None):
    """(codes u8[rows,cols/2], block bytes u8[rows,cols/16], global f32) for config 2.
    `row_mu` (optional, [rows]) overrides mu per output row."""
    codes = rng.integers(0, 256, size=(rows, cols // 2), dtype=np.uint8)
    mus = mu if row_mu is None else np.asarray(row_mu, np.float64)[:, None]
    import torch
    eff = torch.from_numpy(mus + sigma * rng.standard_normal(size=(rows, cols // 16))).exp().float().numpy()
    g = np.float32(eff.max() / 448.0)
    # torch's RNE + saturating float8_e4m3fn cast (equal to f32_to_e4m3 on this range)
    blocks = torch.from_numpy((eff / g).astype(np.float32)).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    return codes, blocks, g
