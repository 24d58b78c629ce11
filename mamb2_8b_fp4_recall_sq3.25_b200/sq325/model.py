"""The Mamba-2 8B LM with packed-resident FP4 weights (host container).

Geometry is MODEL_CONFIG of mamba2_recall/runtime.py:25-33 (d_model 4096, 56 layers,
vocab 256000, d_state 128, d_conv 4, expand 2, headdim 64, ngroups 8, gated RMSNorm
group 1024, fp16 residual, untied embedding/head).  The 114 FP4 matrices (56 in_proj,
56 out_proj, embedding, lm_head) stay packed on the GPU; the 393 other tensors are fp16.
`synthetic_model` builds random weights of that architecture for the benchmark configs
(there is no checkpoint in this environment).
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np
import torch

from . import fp4 as F

MODEL_CONFIG = {
    'd_model': 4096, 'd_intermediate': 0, 'n_layer': 56, 'vocab_size': 256000,
    'ssm_cfg': {'layer': 'Mamba2', 'd_state': 128, 'd_conv': 4, 'expand': 2, 'headdim': 64, 'ngroups': 8,
                'chunk_size': 128, 'rmsnorm': True, 'norm_before_gate': False, 'use_mem_eff_path': False},
    'rms_norm': True, 'residual_in_fp32': False, 'fused_add_norm': False, 'pad_vocab_size_multiple': 128,
    'tie_embeddings': False,
}
D_MODEL, D_INNER, D_XBC, D_ZX, HEADS, HEAD_DIM, GROUPS, D_CONV = 4096, 8192, 10240, 18560, 128, 64, 8, 4
EPS = 1e-5
# log-normal mean of the effective block scale per in_proj output row (z | xBC | dt)
IN_PROJ_ROW_MU = torch.cat([torch.full((D_ZX - HEADS,), -4.0), torch.full((HEADS,), -7.0)])


@dataclass
class MixerWeights:
    in_proj: F.Fp4Tensor          # [18560, 4096]
    out_proj: F.Fp4Tensor         # [4096, 8192]
    norm_weight: torch.Tensor     # Block RMSNorm [4096] fp16
    conv_weight: torch.Tensor     # [10240, 4] fp16 (conv1d.weight[:, 0, :])
    conv_bias: torch.Tensor       # [10240] fp16
    A_log: torch.Tensor           # [128] fp16
    D: torch.Tensor               # [128] fp16
    dt_bias: torch.Tensor         # [128] fp16
    gated_norm_weight: torch.Tensor   # [8192] fp16
    A: torch.Tensor = None        # [128] fp32, -exp(A_log.float()) (fp4_zero_predictor_codec_v1.py:347)

    def __post_init__(self):
        if self.A is None:
            self.A = (-torch.exp(self.A_log.float())).contiguous()


@dataclass(eq=False)            # identity hash: controllers key ownership by model object
class Mamba2FP4Model:
    embedding: F.Fp4Tensor
    lm_head: F.Fp4Tensor
    norm_f: torch.Tensor
    layers: list
    vocab: int = 256000
    eps: float = EPS
    adapter: object = None        # resurface.AdapterBank once install_fp16 ran
    meta: dict = field(default_factory=dict)

    @property
    def n_layer(self):
        return len(self.layers)

    @property
    def device(self):
        return self.norm_f.device

    def packed_weight_bytes(self):
        mats = [self.embedding, self.lm_head] + [m for L in self.layers for m in (L.in_proj, L.out_proj)]
        return sum(m.nbytes for m in mats)

    def fp16_parameter_bytes(self):
        small = [self.norm_f] + [t for L in self.layers for t in (L.norm_weight, L.conv_weight, L.conv_bias, L.A_log,
                                                                   L.D, L.dt_bias, L.gated_norm_weight)]
        return sum(t.numel() * 2 for t in small)


def _fp16(gen, shape, device, kind, **kw):
    t = torch.empty(shape, device=device, dtype=torch.float32)
    if kind == 'normal':
        t.normal_(kw.get('mean', 0.0), kw.get('std', 1.0), generator=gen)
    elif kind == 'uniform':
        t.uniform_(kw['lo'], kw['hi'], generator=gen)
    elif kind == 'ones':
        t.fill_(1.0)
    return t.half().contiguous()


@torch.no_grad()
def synthetic_model(seed=4, n_layer=56, vocab=256000, device='cuda'):
    """Random-init weights of the 8B architecture (config 3/4/5 distributions):
    FP4 codes uniform, effective block scales logNormal(-4, 0.5) — except the 128 dt
    rows of in_proj, which use logNormal(-7, 0.5) so that softplus(dt + dt_bias) stays
    in the small-step range of a trained Mamba-2 (with -4 the raw dt reaches +-15, the
    carry explodes and the fp16 readout overflows); A_log so that A in [-16, -1];
    D ~ N(0,1); dt_bias ~ U[-4,-1]; conv weight ~ N(0, 0.5), conv bias ~ N(0, 0.1);
    norm weights 1."""
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    layers = []
    row_mu = IN_PROJ_ROW_MU.to(device)
    for _ in range(n_layer):
        layers.append(MixerWeights(
            in_proj=F.synthetic(D_ZX, D_MODEL, gen, device, row_mu=row_mu),
            out_proj=F.synthetic(D_MODEL, D_INNER, gen, device),
            norm_weight=_fp16(gen, (D_MODEL,), device, 'ones'),
            conv_weight=_fp16(gen, (D_XBC, D_CONV), device, 'normal', std=0.5),
            conv_bias=_fp16(gen, (D_XBC,), device, 'normal', std=0.1),
            A_log=torch.log(_fp16(gen, (HEADS,), device, 'uniform', lo=1.0, hi=16.0).float()).half(),
            D=_fp16(gen, (HEADS,), device, 'normal'),
            dt_bias=_fp16(gen, (HEADS,), device, 'uniform', lo=-4.0, hi=-1.0),
            gated_norm_weight=_fp16(gen, (D_INNER,), device, 'ones')))
    emb = F.synthetic(vocab, D_MODEL, gen, device)
    head = F.synthetic(vocab, D_MODEL, gen, device)
    return Mamba2FP4Model(emb, head, _fp16(gen, (D_MODEL,), device, 'ones'), layers, vocab=vocab,
                          meta=dict(seed=seed, synthetic=True))


def synthetic_statics(layouts, seed=4, device='cuda'):
    """Permutation table u8[L,8,128], per-layer basis f16[8,nz,2], latent scales f16[8,2]
    (U[0.1,1.1]) and predictors f16[8,n8+n4+2,nz] ~ N(0,1)/sqrt(n8+n4+2) — the shapes of
    the released state_config.pt (scripts/infer_fp4_ridge_resurface_v1.py:21-46)."""
    from .codec import layout_descriptor
    rng = np.random.default_rng(seed)
    L = len(layouts)
    table = np.stack([np.stack([rng.permutation(128) for _ in range(GROUPS)]) for _ in range(L)]).astype(np.uint8)
    bases, scales, preds = [], [], []
    for layout in layouts:
        s = layout_descriptor(layout)
        f = s['n8'] + s['n4'] + 2
        bases.append(torch.from_numpy(rng.standard_normal((GROUPS, s['nzero'], 2)).astype(np.float16)).to(device))
        scales.append(torch.from_numpy((rng.random((GROUPS, 2)) + 0.1).astype(np.float16)).to(device))
        preds.append(torch.from_numpy((rng.standard_normal((GROUPS, f, s['nzero'])) / np.sqrt(f)).astype(np.float16))
                     .to(device))
    return torch.from_numpy(table).to(device), tuple(layouts), bases, scales, preds


# Per-layer tier layouts of the released configuration, as recorded in the reference's
# evaluation/wt2_test_v1/resurface.json (`layer_layouts`).  Benchmark config 4/5 use it.
RELEASED_LAYOUTS = (
    '36_24_68', '16_64_48', '32_32_64', '40_16_72', '16_64_48', '16_64_48', '24_48_56', '32_32_64',
    '32_32_64', '32_32_64', '32_32_64', '36_24_68', '40_16_72', '24_48_56', '8_80_40', '32_32_64',
    '32_32_64', '32_32_64', '32_32_64', '24_48_56', '16_64_48', '16_64_48', '24_48_56', '16_64_48',
    '32_32_64', '24_48_56', '24_48_56', '8_80_40', '40_16_72', '32_32_64', '24_48_56', '24_48_56',
    '40_16_72', '36_24_68', '16_64_48', '8_80_40', '16_64_48', '24_48_56', '44_8_76', '36_24_68',
    '24_48_56', '24_48_56', '16_64_48', '32_32_64', '8_80_40', '32_32_64', '8_80_40', '8_80_40',
    '24_48_56', '8_80_40', '16_64_48', '44_8_76', '44_8_76', '8_80_40', '24_48_56', '32_32_64')


def benchmark_layouts(n_layer=56):
    if n_layer == 56:
        return RELEASED_LAYOUTS
    from .codec import LAYOUTS
    return tuple(LAYOUTS[i % len(LAYOUTS)] for i in range(n_layer))
