"""ctypes front end of oracle/csrc/latent_scan.c (CPU, test only).

TEST INFRASTRUCTURE ONLY, like the rest of oracle/.  `latent_scan` has the signature and
result of oracle.codec.latent_scan: the per-token scalars that need exp / log (softplus of
dt, exp(A dt)) and the predictor correction einsum are computed here with the same numpy /
torch expressions as oracle/codec.py, per token, and the per-row recurrence, readout and
requant run in C (one IEEE fp32 operation per numpy operation, numpy's pairwise summation
order, OpenMP over rows).  tests/test_oracle_golden.py pins it bit-exact to the numpy
restatement and to the reference's golden vectors.

build() compiles the library into oracle/_build/ with gcc (-O2 -fopenmp -ffp-contract=off).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

from . import codec as oc

HERE = Path(__file__).resolve().parent
SRC = HERE / 'csrc' / 'latent_scan.c'
LIB = HERE / '_build' / 'liblatent_scan.so'
_lib = None


def build(force=False):
    if not force and LIB.exists() and LIB.stat().st_mtime >= SRC.stat().st_mtime:
        return LIB
    LIB.parent.mkdir(exist_ok=True)
    tmp = LIB.with_suffix('.so.tmp')
    cmd = ['gcc', '-O2', '-fopenmp', '-ffp-contract=off', '-fno-fast-math', '-shared', '-fPIC', '-o', str(tmp),
           str(SRC), '-lm']
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f'gcc failed:\n{r.stderr}')
    os.replace(tmp, LIB)
    return LIB


def load():
    global _lib
    if _lib is None:
        build()
        lib = C.CDLL(str(LIB))
        lib.latent_scan_rows.restype = None
        lib.latent_scan_rows.argtypes = [C.c_int] * 7 + [C.c_void_p] * 18
        _lib = lib
    return _lib


def _p(a):
    return C.c_void_p(a.ctypes.data)


def per_token_scalars(dt, A, dt_bias):
    """(dt after softplus, exp(A dt)) fp32 [Bt,L,H], token by token with the expressions of
    oracle.codec.latent_scan (so that every exp / log sees the same array shapes)."""
    dt = np.asarray(dt, np.float16)
    Bt, L, H = dt.shape
    av = np.asarray(A, np.float32)[None, :]
    bias = np.asarray(dt_bias).astype(np.float32)[None, :]
    dtv_all = np.empty((Bt, L, H), np.float32)
    dec_all = np.empty((Bt, L, H), np.float32)
    F32 = np.float32
    for t in range(L):
        dtv = dt[:, t].astype(np.float32) + bias
        with np.errstate(over='ignore'):
            dtv = np.where(dtv <= F32(20.0), np.log(np.exp(dtv) + F32(1.0)), dtv).astype(np.float32)
        dtv_all[:, t] = dtv
        dec_all[:, t] = np.exp(av * dtv).astype(np.float32)
    return dtv_all, dec_all


def latent_scan(x, dt, A, B, C_, D, dt_bias, state, permutation, basis, latent_scale, predictor, layout,
                corr=None, head_groups=None):
    """Same contract and bits as oracle.codec.latent_scan (state mutated, y fp16 returned)."""
    lib = load()
    n8, n4, nz = oc.layout_counts(layout)
    x = np.ascontiguousarray(x, np.float16)
    Bt, L, H, P = x.shape
    G = np.asarray(B).shape[2]
    groups = (np.arange(H) // (H // G) if head_groups is None else np.asarray(head_groups)).astype(np.int32)
    if corr is None:
        corr = oc.predictor_correction(C_, permutation, predictor, layout)
    corr = np.ascontiguousarray(corr, np.float32)
    dtv, dec = per_token_scalars(dt, A, dt_bias)
    Bh = np.ascontiguousarray(B, np.float16)
    Ch = np.ascontiguousarray(C_, np.float16)
    Dv = np.ascontiguousarray(np.asarray(D).astype(np.float32))
    perm = np.ascontiguousarray(permutation, np.uint8)
    bas = np.ascontiguousarray(basis, np.float16)
    ls = np.ascontiguousarray(np.asarray(latent_scale, np.float16).astype(np.float32))
    for k in ('lo', 'hi', 'q4', 'latent', 's8', 's4'):
        if not state[k].flags['C_CONTIGUOUS']:
            raise ValueError('state arrays must be C-contiguous')
    y = np.zeros((Bt, L, H, P), np.float16)
    lib.latent_scan_rows(Bt, L, H, P, G, n8, n4, _p(x), _p(dtv), _p(dec), _p(Bh), _p(Ch), _p(Dv), _p(corr), _p(perm),
                         _p(bas), _p(ls), _p(groups), _p(state['lo']), _p(state['hi']), _p(state['q4']),
                         _p(state['latent']), _p(state['s8']), _p(state['s4']), _p(y))
    return y
