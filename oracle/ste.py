"""CPU oracle (test infrastructure only) for the legacy sq3p25 scan and its straight-through
training backward.

Restates, op for op in numpy float32 without fused multiply-adds:
  sq3p25_scan   the packed 16 INT8 + 64 INT4 (+ 48 pruned) scan `_sq_scan`,
                mamba2_recall/state_codec.py:105-176, as launched by `scan` (:204-262);
  ste_backward  the straight-through backward of mamba2_recall/state_training_scan.py:
                `_carry_checkpoints` (:24-57), `_chunk_history` (:60-98),
                `_chunk_backward` (:101-179) and the driver loop of
                `_StateQuantSTE.backward` (:195-221).
Reductions run over the kernels' tile widths (16 / 64 / 64 lanes, rows in tiles of 16) with
np.sum / np.max, which is what the Triton interpreter executes; atomic additions are applied
in the interpreter's program order (batch, head, row tile).  Pinned bit-exact to the
reference kernels run by the interpreter (tests/golden/ste.npz, tests/golden/make_golden.py).
Nothing in the product path imports this module.
"""
from __future__ import annotations

import numpy as np

F32 = np.float32
TILE = 16


def round_half_away(q):
    """C round() (ties away from zero); a negative q that rounds to zero gives +0, as the
    interpreter's negation (0 - r) does."""
    a = np.abs(q)
    r = np.floor(a)
    r = np.where(a - r >= F32(0.5), r + F32(1.0), r).astype(np.float32)
    return np.where(q < 0, F32(0.0) - r, r).astype(np.float32)


def _unpack(v):
    v = v.astype(np.int32)
    return np.stack((v & 15, (v >> 4) & 15), -1).reshape(*v.shape[:-1], v.shape[-1] * 2)


def _positions(perm, group):
    p = perm[group].astype(np.int64)
    posd = np.zeros(64, np.int64)
    posd[:48] = p[80:]
    return p[:16], p[16:80], posd


def _softplus(dt):
    return np.where(dt <= F32(20.0), np.log(np.exp(dt) + F32(1.0)), dt).astype(np.float32)


def _requant(s8, s4):
    den8 = np.maximum((np.max(np.abs(s8), 1) / F32(127.0)).astype(np.float32), F32(1e-8))
    den4 = np.maximum((np.max(np.abs(s4), 1) / F32(7.0)).astype(np.float32), F32(1e-8))
    q8 = np.minimum(np.maximum(round_half_away((s8 / den8[:, None]).astype(np.float32)), F32(-127)), F32(127))
    q4 = np.minimum(np.maximum(round_half_away((s4 / den4[:, None]).astype(np.float32)), F32(-7)), F32(7))
    sc8 = den8.astype(np.float16).astype(np.float32)
    sc4 = den4.astype(np.float16).astype(np.float32)
    return q8, q4, (q8 * sc8[:, None]).astype(np.float32), (q4 * sc4[:, None]).astype(np.float32), sc8, sc4


def _transcendentals(device_math, b, t, h, raw, av):
    """softplus(raw), exp(A * softplus) and sigmoid(raw) of one (batch, token, head): numpy's,
    or the device's own values when `device_math` (float32 [B,L,H] arrays 'softplus', 'decay',
    'sigmoid') is given.  exp / log are the only operations whose last bit differs between
    libraries; substituting the device's results lets a device run be checked bit for bit."""
    if device_math is not None:
        return (F32(device_math['softplus'][b, t, h]), F32(device_math['decay'][b, t, h]),
                F32(device_math['sigmoid'][b, t, h]) if 'sigmoid' in device_math else None)
    d = _softplus(raw)
    decay = np.exp((av * d).astype(np.float32)).astype(np.float32)
    sig = np.where(raw <= F32(20.0), (F32(1.0) / (F32(1.0) + np.exp(-raw))).astype(np.float32),
                   F32(1.0)).astype(np.float32)
    return d, decay, sig


def sq3p25_scan(x, dt, A, B, C, D, dt_bias, state, perm, device_math=None):
    """Mutates `state` (dict of numpy lo/hi/q4 u8, s8/s4 f16); returns y fp16 [B,L,H,P]."""
    Bn, L, H, P = x.shape
    G = B.shape[2]
    y = np.zeros(x.shape, np.float16)
    for b in range(Bn):
        for h in range(H):
            g = h // (H // G)
            pos8, pos4, posd = _positions(perm, g)
            dmask = np.arange(64) < 48
            av, dv, bias = F32(A[h]), F32(np.float32(D[h])), F32(np.float32(dt_bias[h]))
            for t0 in range(0, P, TILE):
                rows = slice(t0, min(P, t0 + TILE))
                nr = rows.stop - rows.start
                ub = (_unpack(state['hi'][b, h, rows]) << 4) | _unpack(state['lo'][b, h, rows])
                q8 = (ub - 256 * (ub > 127)).astype(np.int32)
                nib = _unpack(state['q4'][b, h, rows])
                q4 = (nib - 16 * (nib > 7)).astype(np.int32)
                s8 = (q8.astype(np.float32) * state['s8'][b, h, rows].astype(np.float32)[:, None]).astype(np.float32)
                s4 = (q4.astype(np.float32) * state['s4'][b, h, rows].astype(np.float32)[:, None]).astype(np.float32)
                # padded to the kernel's 16-row tile (masked rows carry zeros)
                if nr < TILE:
                    s8 = np.vstack([s8, np.zeros((TILE - nr, 16), np.float32)])
                    s4 = np.vstack([s4, np.zeros((TILE - nr, 64), np.float32)])
                sc8 = sc4 = None
                qa8 = qa4 = None
                for t in range(L):
                    xv = np.zeros(TILE, np.float32)
                    xv[:nr] = x[b, t, h, rows].astype(np.float32)
                    d, decay, _ = _transcendentals(device_math, b, t, h,
                                                   (np.float32(dt[b, t, h]) + bias).astype(np.float32), av)
                    bv, cv = B[b, t, g].astype(np.float32), C[b, t, g].astype(np.float32)
                    bv8, cv8, bv4, cv4 = bv[pos8], cv[pos8], bv[pos4], cv[pos4]
                    bvd = np.where(dmask, bv[posd], F32(0)).astype(np.float32)
                    cvd = np.where(dmask, cv[posd], F32(0)).astype(np.float32)
                    s8 = (s8 * decay + ((bv8[None, :] * d).astype(np.float32) * xv[:, None])).astype(np.float32)
                    s4 = (s4 * decay + ((bv4[None, :] * d).astype(np.float32) * xv[:, None])).astype(np.float32)
                    sd = ((bvd[None, :] * d).astype(np.float32) * xv[:, None]).astype(np.float32)
                    out = np.sum((s8 * cv8[None, :]).astype(np.float32), 1)
                    out = (out + np.sum((s4 * cv4[None, :]).astype(np.float32), 1)).astype(np.float32)
                    out = (out + (np.sum((sd * cvd[None, :]).astype(np.float32), 1) + (xv * dv).astype(np.float32))
                           ).astype(np.float32)
                    y[b, t, h, rows] = out[:nr].astype(np.float16)
                    qa8, qa4, s8, s4, sc8, sc4 = _requant(s8, s4)
                q8i = qa8[:nr].astype(np.int32)
                q4i = qa4[:nr].astype(np.int32)
                lo, hi = q8i & 15, (q8i >> 4) & 15
                state['lo'][b, h, rows] = (lo[:, 0::2] | (lo[:, 1::2] << 4)).astype(np.uint8)
                state['hi'][b, h, rows] = (hi[:, 0::2] | (hi[:, 1::2] << 4)).astype(np.uint8)
                qn = q4i & 15
                state['q4'][b, h, rows] = (qn[:, 0::2] | (qn[:, 1::2] << 4)).astype(np.uint8)
                state['s8'][b, h, rows] = sc8[:nr].astype(np.float16)
                state['s4'][b, h, rows] = sc4[:nr].astype(np.float16)
    return y


def _tile_step(s8, s4, xv, d, decay, bv8, bv4):
    s8 = (s8 * decay + ((bv8[None, :] * d).astype(np.float32) * xv[:, None])).astype(np.float32)
    s4 = (s4 * decay + ((bv4[None, :] * d).astype(np.float32) * xv[:, None])).astype(np.float32)
    _, _, s8, s4, _, _ = _requant(s8, s4)
    return s8, s4


def ste_backward(x, dt, A, B, C, D, dt_bias, perm, dy, chunk, device_math=None):
    """Returns (dx, ddt, dB, dC, checkpoints) in float32, the reference's backward with a fresh
    zero state: carries replayed exactly, identity derivative through the 80 live lanes, zero
    through the 48 pruned ones, current-token readout through all 128."""
    Bn, L, H, P = x.shape
    G = B.shape[2]
    K = chunk
    NC = -(-L // K)
    ntile = -(-P // TILE)
    cp = np.zeros((Bn, NC, H, ntile * TILE, 80), np.float32)
    dx = np.zeros(x.shape, np.float32)
    ddt = np.zeros(dt.shape, np.float32)
    dB = np.zeros(B.shape, np.float32)
    dC = np.zeros(C.shape, np.float32)
    dmask = np.arange(64) < 48

    def token(b, t, h, g, rows_idx, nr):
        pos8, pos4, posd = _positions(perm, g)
        xv = np.zeros(TILE, np.float32)
        xv[:nr] = x[b, t, h, rows_idx].astype(np.float32)
        bias = F32(np.float32(dt_bias[h]))
        raw = (np.float32(dt[b, t, h]) + bias).astype(np.float32)
        d, decay, sig = _transcendentals(device_math, b, t, h, raw, F32(A[h]))
        return pos8, pos4, posd, xv, sig, d, decay

    # carry checkpoints: the carry entering each chunk
    for b in range(Bn):
        for h in range(H):
            g = h // (H // G)
            for tile in range(ntile):
                rows_idx = slice(tile * TILE, min(P, tile * TILE + TILE))
                nr = rows_idx.stop - rows_idx.start
                s8 = np.zeros((TILE, 16), np.float32)
                s4 = np.zeros((TILE, 64), np.float32)
                for c in range(NC):
                    cp[b, c, h, tile * TILE:tile * TILE + TILE, :16] = s8
                    cp[b, c, h, tile * TILE:tile * TILE + TILE, 16:] = s4
                    for j in range(K):
                        t = c * K + j
                        if t < L:
                            pos8, pos4, _, xv, _, d, decay = token(b, t, h, g, rows_idx, nr)
                            bv = B[b, t, g].astype(np.float32)
                            s8, s4 = _tile_step(s8, s4, xv, d, decay, bv[pos8], bv[pos4])
    adj = np.zeros((Bn, H, ntile * TILE, 80), np.float32)
    for c in reversed(range(NC)):
        # history of the chunk: the carry entering each of its tokens
        hist = np.zeros((Bn, K, H, ntile * TILE, 80), np.float32)
        for b in range(Bn):
            for h in range(H):
                g = h // (H // G)
                for tile in range(ntile):
                    rows_idx = slice(tile * TILE, min(P, tile * TILE + TILE))
                    nr = rows_idx.stop - rows_idx.start
                    r0 = tile * TILE
                    s8 = cp[b, c, h, r0:r0 + TILE, :16].copy()
                    s4 = cp[b, c, h, r0:r0 + TILE, 16:].copy()
                    for j in range(K):
                        t = c * K + j
                        if t < L:
                            hist[b, j, h, r0:r0 + TILE, :16] = s8
                            hist[b, j, h, r0:r0 + TILE, 16:] = s4
                            pos8, pos4, _, xv, _, d, decay = token(b, t, h, g, rows_idx, nr)
                            bv = B[b, t, g].astype(np.float32)
                            s8, s4 = _tile_step(s8, s4, xv, d, decay, bv[pos8], bv[pos4])
        # reverse sweep over the chunk's tokens, programs in (batch, head, tile) order
        for b in range(Bn):
            for h in range(H):
                g = h // (H // G)
                av, dv = F32(A[h]), F32(np.float32(D[h]))
                for tile in range(ntile):
                    rows_idx = slice(tile * TILE, min(P, tile * TILE + TILE))
                    nr = rows_idx.stop - rows_idx.start
                    r0 = tile * TILE
                    rmask = np.arange(TILE) < nr
                    adj8 = adj[b, h, r0:r0 + TILE, :16].copy()
                    adj4 = adj[b, h, r0:r0 + TILE, 16:].copy()
                    for rev in range(K):
                        j = K - 1 - rev
                        t = c * K + j
                        if t >= L:
                            continue
                        pos8, pos4, posd, xv, sig, d, decay = token(b, t, h, g, rows_idx, nr)
                        gy = np.zeros(TILE, np.float32)
                        gy[:nr] = dy[b, t, h, rows_idx].astype(np.float32)
                        prev8 = hist[b, j, h, r0:r0 + TILE, :16]
                        prev4 = hist[b, j, h, r0:r0 + TILE, 16:]
                        bv, cv = B[b, t, g].astype(np.float32), C[b, t, g].astype(np.float32)
                        b8, b4, c8, c4 = bv[pos8], bv[pos4], cv[pos8], cv[pos4]
                        bd = np.where(dmask, bv[posd], F32(0)).astype(np.float32)
                        cd = np.where(dmask, cv[posd], F32(0)).astype(np.float32)
                        v8 = ((gy[:, None] * c8[None, :]).astype(np.float32) + adj8).astype(np.float32)
                        v4 = ((gy[:, None] * c4[None, :]).astype(np.float32) + adj4).astype(np.float32)
                        vd = (gy[:, None] * cd[None, :]).astype(np.float32)
                        h8 = ((prev8 * decay).astype(np.float32) + ((b8[None, :] * d).astype(np.float32) * xv[:, None])
                              ).astype(np.float32)
                        h4 = ((prev4 * decay).astype(np.float32) + ((b4[None, :] * d).astype(np.float32) * xv[:, None])
                              ).astype(np.float32)
                        hd = ((bd[None, :] * d).astype(np.float32) * xv[:, None]).astype(np.float32)
                        dxv = np.sum((v8 * (b8[None, :] * d).astype(np.float32)).astype(np.float32), 1)
                        dxv = (dxv + np.sum((v4 * (b4[None, :] * d).astype(np.float32)).astype(np.float32), 1)
                               ).astype(np.float32)
                        dxv = (dxv + (np.sum((vd * (bd[None, :] * d).astype(np.float32)).astype(np.float32), 1)
                                      + (gy * dv).astype(np.float32))).astype(np.float32)
                        dx[b, t, h, rows_idx] = dxv[:nr]
                        ad = (av * decay).astype(np.float32)
                        e8 = ((prev8 * ad).astype(np.float32) + (b8[None, :] * xv[:, None]).astype(np.float32)
                              ).astype(np.float32)
                        e4 = ((prev4 * ad).astype(np.float32) + (b4[None, :] * xv[:, None]).astype(np.float32)
                              ).astype(np.float32)
                        dl = np.sum((v8 * e8).astype(np.float32), 1)
                        dl = (dl + np.sum((v4 * e4).astype(np.float32), 1)).astype(np.float32)
                        dl = (dl + np.sum((vd * (bd[None, :] * xv[:, None]).astype(np.float32)).astype(np.float32), 1)
                              ).astype(np.float32)
                        dl = (np.sum(np.where(rmask, dl, F32(0)).astype(np.float32), 0) * sig).astype(np.float32)
                        ddt[b, t, h] = (ddt[b, t, h] + dl).astype(np.float32)
                        factor = np.where(rmask, (d * xv).astype(np.float32), F32(0)).astype(np.float32)
                        db8 = np.sum((v8 * factor[:, None]).astype(np.float32), 0)
                        db4 = np.sum((v4 * factor[:, None]).astype(np.float32), 0)
                        dbd = np.sum((vd * factor[:, None]).astype(np.float32), 0)
                        dc8 = np.sum((h8 * gy[:, None]).astype(np.float32), 0)
                        dc4 = np.sum((h4 * gy[:, None]).astype(np.float32), 0)
                        dcd = np.sum((hd * gy[:, None]).astype(np.float32), 0)
                        for vals, pos, m in ((db8, pos8, None), (db4, pos4, None), (dbd, posd, dmask)):
                            for i, pidx in enumerate(pos):
                                if m is None or m[i]:
                                    dB[b, t, g, pidx] = F32(dB[b, t, g, pidx] + vals[i])
                        for vals, pos, m in ((dc8, pos8, None), (dc4, pos4, None), (dcd, posd, dmask)):
                            for i, pidx in enumerate(pos):
                                if m is None or m[i]:
                                    dC[b, t, g, pidx] = F32(dC[b, t, g, pidx] + vals[i])
                        adj8 = (v8 * decay).astype(np.float32)
                        adj4 = (v4 * decay).astype(np.float32)
                    adj[b, h, r0:r0 + TILE, :16] = adj8
                    adj[b, h, r0:r0 + TILE, 16:] = adj4
    return dx, ddt, dB, dC, cp[:, :, :, :P]
