"""Matched models for parity tests and the CPU baseline (test infrastructure only).

The same packed bytes feed the GPU model (sq325) and the CPU oracle (oracle.model):
real per-layer geometry (d_model 4096, 128 heads x 64, 8 groups, d_state 128), any
number of layers, any vocabulary.  With device=None only the oracle half is built
(bench.py's cpu_baseline leg); the random draws are the same either way."""
from __future__ import annotations

import numpy as np
import torch

from . import codec as oc
from . import fp4 as of
from . import model as om


def packed(rng, rows, cols, mu=-4.0, sigma=0.5):
    return of.synthetic_matrix(rows, cols, rng, mu, sigma)


def build_pair(n_layer=2, vocab=512, layouts=None, seed=0, adapter=True, hard=False, device='cuda'):
    """(gpu_model, oracle_model, statics); gpu_model and statics are None when device is None."""
    gpu = device is not None
    if gpu:
        from sq325 import fp4 as F
        from sq325 import model as M
        from sq325 import resurface as R
    rng = np.random.default_rng(seed)
    layouts = layouts or tuple(oc.LAYOUTS[(seed + i) % 7] for i in range(n_layer))
    gpu_layers, ora_layers = [], []
    bank_V, bank_g, bank_w, bank_b = [], [], [], []
    table = np.stack([np.stack([rng.permutation(128) for _ in range(8)]) for _ in range(n_layer)]).astype(np.uint8)
    bases, scales, preds = [], [], []
    for i, layout in enumerate(layouts):
        n8, n4, nz = oc.layout_counts(layout)
        win = of.synthetic_matrix(18560, 4096, rng, row_mu=np.r_[np.full(18432, -4.0), np.full(128, -7.0)])
        wout = packed(rng, 4096, 8192)
        f16 = lambda a: np.asarray(a, np.float32).astype(np.float16)
        norm_w = f16(1.0 + 0.1 * rng.standard_normal(4096))
        conv_w = f16(0.5 * rng.standard_normal((10240, 4)))
        conv_b = f16(0.1 * rng.standard_normal(10240))
        A_log = f16(np.log(rng.uniform(1.0, 16.0, 128)))
        D = f16(rng.standard_normal(128))
        dt_bias = f16(rng.uniform(-4.0, -1.0, 128))
        gnorm = f16(1.0 + 0.1 * rng.standard_normal(8192))
        basis = f16(rng.standard_normal((8, nz, 2)))
        ls = f16(rng.uniform(0.1, 1.1, (8, 2)))
        pred = f16(rng.standard_normal((8, n8 + n4 + 2, nz)) / np.sqrt(n8 + n4 + 2))
        bases.append(basis); scales.append(ls); preds.append(pred)
        ad = None
        if adapter:
            V = f16(0.05 * rng.standard_normal((128, 128)))
            g = f16(rng.uniform(0.5, 1.5, 128))
            w = f16(0.02 * rng.standard_normal(4096))
            b = f16([-0.5])
            bank_V.append(V); bank_g.append(g); bank_w.append(w); bank_b.append(b)
            ad = (torch.from_numpy(V), torch.from_numpy(g), torch.from_numpy(w), torch.from_numpy(b[0:1]).reshape(()),
                  hard)
        if gpu:
            T = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(device)
            gpu_layers.append(M.MixerWeights(F.from_arrays(*win, device=device), F.from_arrays(*wout, device=device),
                                             T(norm_w), T(conv_w), T(conv_b), T(A_log), T(D), T(dt_bias), T(gnorm)))
        ora_layers.append(om.LayerOracle(
            torch.from_numpy(of.decode(*win)), torch.from_numpy(of.decode(*wout)), torch.from_numpy(norm_w),
            torch.from_numpy(conv_w), torch.from_numpy(conv_b), torch.from_numpy(A_log), torch.from_numpy(D),
            torch.from_numpy(dt_bias), torch.from_numpy(gnorm), layout, torch.from_numpy(table[i]),
            torch.from_numpy(basis), torch.from_numpy(ls), torch.from_numpy(pred), adapter=ad))
    emb = packed(rng, vocab, 4096, mu=-2.0)
    head = packed(rng, vocab, 4096)
    norm_f = (1.0 + 0.1 * rng.standard_normal(4096)).astype(np.float16)
    ora = om.ModelOracle(torch.from_numpy(of.decode(*emb)), torch.from_numpy(of.decode(*head)),
                         torch.from_numpy(norm_f), ora_layers)
    if not gpu:
        return None, ora, None
    gm = M.Mamba2FP4Model(F.from_arrays(*emb, device=device), F.from_arrays(*head, device=device),
                          torch.from_numpy(norm_f).to(device), gpu_layers, vocab=vocab)
    if adapter:
        gm.adapter = R.AdapterBank('hard' if hard else 'soft', [torch.from_numpy(v).to(device) for v in bank_V],
                                   [torch.from_numpy(v).to(device) for v in bank_g],
                                   [torch.from_numpy(v).to(device) for v in bank_w],
                                   [torch.from_numpy(v).to(device) for v in bank_b])
    statics = (torch.from_numpy(table).to(device), tuple(layouts),
               [torch.from_numpy(b).to(device) for b in bases], [torch.from_numpy(s).to(device) for s in scales],
               [torch.from_numpy(p).to(device) for p in preds])
    return gm, ora, statics


def rel_l2(a, b):
    a, b = torch.as_tensor(a).double().cpu(), torch.as_tensor(b).double().cpu()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))
