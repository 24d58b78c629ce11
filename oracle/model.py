"""torch-CPU restatement of the Mamba-2 layer / model around the SQ3.25 codec (test only).

Reference call graph restated here (all arithmetic as the reference's torch calls
perform it on CUDA: fp16 storage, fp32 accumulation, fp16 rounding at each tensor
boundary):

  Block (mamba_ssm, fused_add_norm=False, residual_in_fp32=False):
      residual = fp16(h + residual); h = RMSNorm(residual)          [UNPINNED: mamba_ssm absent]
  PredictorState._forward            scripts/fp4_zero_predictor_codec_v1.py:314-367
      in_proj -> split z|xBC|dt (8192,10240,128) -> causal conv -> split x|B|C
      -> codec scan (oracle.codec.latent_scan) -> [Resurface pre-hook] -> gated
      RMSNorm (norm_before_gate=False, group 1024) -> out_proj
  StateQuant._convolution            mamba2_recall/state_quant.py:283-317
      step: roll cache, fp16 products summed, + bias, SiLU; prefill: conv1d
      (fp32 accumulate + bias -> fp16) + SiLU, cache <- last 4 raw columns
  _Adapter.forward                   mamba2_recall/resurface_native.py:105-118
  scoring head                       scripts/run_fp4_ridge_resurface_v3.py:105-109
  greedy head                        scripts/infer_fp4_ridge_resurface_v1.py:103-105

The mamba_ssm RMSNorm / gated RMSNorm / Block formulas follow the public Mamba-2
definition (eps 1e-5); their parity with the reference runtime is UNPINNED.
"""
from __future__ import annotations

import numpy as np
import torch

from . import codec as oc

D_MODEL, D_INNER, D_XBC, D_ZX, HEADS, HEAD_DIM, GROUPS = 4096, 8192, 10240, 18560, 128, 64, 8


def h(x):
    return torch.as_tensor(x).half()


def rmsnorm(x16, w16, eps=1e-5):
    x = x16.float()
    rstd = 1.0 / torch.sqrt((x * x).mean(-1, keepdim=True) + eps)
    return ((x * rstd) * w16.float()).half()


def add16(a, b):
    return (a.float() + b.float()).half()


def linear(x16, w16):
    return (x16.float() @ w16.float().T).half()


def silu16(v16):
    v = v16.float()
    return (v / (1.0 + torch.exp(-v))).half()


def conv_prefill(raw16, cache16, tokens_before, w16, b16):
    """raw16 [B,L,C]; cache16 chronological [B,C,4] (slot 3 newest) -> out [B,L,C], new cache."""
    raw = raw16.transpose(1, 2)                                     # [B,C,L]
    prefix = 0
    if tokens_before > 0:
        raw = torch.cat((cache16[:, :, 1:], raw), -1)
        prefix = 3
    width = raw.shape[-1]
    new_cache = torch.nn.functional.pad(raw, (4 - width, 0)) if width < 4 else raw[:, :, -4:]
    x = torch.nn.functional.pad(raw.float(), (3, 0))                # causal padding
    L = raw.shape[-1]
    w = w16.float()
    acc = sum(w[None, :, k:k + 1] * x[:, :, k:k + L] for k in range(4)) + b16.float()[None, :, None]
    out = silu16(acc.half()).transpose(1, 2)                        # [B,L+prefix,C]
    return out[:, prefix:].contiguous(), new_cache.contiguous()


def conv_step(raw16, cache16, w16, b16):
    """raw16 [B,C]; cache chronological [B,C,4] -> (out [B,C], new cache)."""
    cache = torch.roll(cache16, shifts=-1, dims=-1).clone()
    cache[:, :, -1] = raw16
    prods = (cache.float() * w16.float()[None]).half()
    v = prods.float().sum(-1).half()
    v = add16(v, b16)
    return silu16(v), cache


def resurface(y16, u16, V16, g16, w16, b16, hard=False):
    """_Adapter.forward on y [T,H*P], u [T,D] (fp16 params, soft or hard gate)."""
    logit16 = (u16.float() @ w16.float()).half()
    logits = add16(logit16, b16).float()
    gate = (logits > 0).float() if hard else torch.sigmoid(logits)
    yh = y16.reshape(y16.shape[0], HEADS, HEAD_DIM)
    mix = torch.einsum('ij,tjp->tip', V16.float(), yh.float()).half()
    gg = (gate.half()[:, None].float() * g16.float()[None, :]).half()
    corr = (gg[..., None].float() * mix.float()).half()
    return add16(yh, corr).reshape_as(y16)


def gated_rmsnorm(y16, z16, w16, eps=1e-5, group=1024):
    x = y16.float()
    z = z16.float()
    x = x * (z * torch.sigmoid(z))
    xs = x.reshape(*x.shape[:-1], -1, group)
    rstd = 1.0 / torch.sqrt((xs * xs).mean(-1, keepdim=True) + eps)
    return ((xs * rstd).reshape_as(x) * w16.float()).half()


class LayerOracle:
    """Weights (decoded fp16, CPU) + statics of one layer."""

    def __init__(self, w_in, w_out, norm_w, conv_w, conv_b, A_log, D, dt_bias, gnorm_w, layout, perm, basis,
                 latent_scale, predictor, adapter=None):
        self.w_in, self.w_out = w_in, w_out
        self.norm_w, self.conv_w, self.conv_b = norm_w, conv_w, conv_b
        self.A = -torch.exp(A_log.float())
        self.D, self.dt_bias, self.gnorm_w = D, dt_bias, gnorm_w
        self.layout, self.perm, self.basis, self.latent_scale, self.predictor = layout, perm, basis, latent_scale, predictor
        self.adapter = adapter           # None or (V, g, w, b, hard)
        # the codec restatement: numpy (oracle.codec) or its bit-identical C form (oracle.cscan)
        self.scan = oc.latent_scan


def layer_forward(L, cache, u16, tokens_before):
    """One PredictorState._forward; cache = {'state': numpy six arrays, 'conv': [B,C,4] fp16}."""
    B, T, _ = u16.shape
    is_step = tokens_before > 0 and T == 1
    zx = linear(u16.reshape(B * T, -1), L.w_in).reshape(B, T, D_ZX)
    z, xbc, dt = zx[..., :D_INNER], zx[..., D_INNER:D_INNER + D_XBC], zx[..., D_INNER + D_XBC:]
    if is_step:
        out, cache['conv'] = conv_step(xbc[:, 0], cache['conv'], L.conv_w, L.conv_b)
        xbc = out[:, None]
    else:
        xbc, cache['conv'] = conv_prefill(xbc, cache['conv'], tokens_before, L.conv_w, L.conv_b)
    x = xbc[..., :D_INNER].reshape(B, T, HEADS, HEAD_DIM)
    Bm = xbc[..., D_INNER:D_INNER + 1024].reshape(B, T, GROUPS, 128)
    Cm = xbc[..., D_INNER + 1024:].reshape(B, T, GROUPS, 128)
    y = L.scan(x.numpy(), dt.contiguous().numpy(), L.A.numpy(), Bm.numpy(), Cm.numpy(),
               L.D.numpy(), L.dt_bias.numpy(), cache['state'], L.perm.numpy(), L.basis.numpy(),
               L.latent_scale.numpy(), L.predictor.numpy(), L.layout)
    y = torch.from_numpy(y).reshape(B * T, D_INNER)
    if L.adapter is not None:
        V, g, w, b, hard = L.adapter
        y = resurface(y, u16.reshape(B * T, -1), V, g, w, b, hard)
    yn = gated_rmsnorm(y, z.reshape(B * T, D_INNER), L.gnorm_w)
    return linear(yn, L.w_out).reshape(B, T, D_MODEL)


class ModelOracle:
    def __init__(self, embed16, head16, norm_f, layers, eps=1e-5, fast_scan=True):
        self.embed16, self.head16, self.norm_f, self.layers, self.eps = embed16, head16, norm_f, layers, eps
        if fast_scan:
            from . import cscan
            for L in layers:
                L.scan = cscan.latent_scan
        self.caches = None
        self.tokens = 0
        self.capture = None          # a list receives every layer's mixer output when set
        self.capture_inputs = None   # a list receives every layer's normed input u when set

    def reset(self, batch):
        self.caches = [dict(state=oc.allocate_state(batch, HEADS, HEAD_DIM, L.layout),
                            conv=torch.zeros(batch, D_XBC, 4, dtype=torch.float16)) for L in self.layers]
        self.tokens = 0

    def backbone(self, ids):
        ids = torch.as_tensor(ids)
        B, T = ids.shape
        hcur = self.embed16[ids.reshape(-1)].reshape(B, T, D_MODEL)
        res = None
        for L, cache in zip(self.layers, self.caches):
            res = hcur if res is None else add16(hcur, res)
            u = rmsnorm(res, L.norm_w, self.eps)
            if self.capture_inputs is not None:
                self.capture_inputs.append(u.clone())
            hcur = layer_forward(L, cache, u, self.tokens)
            if self.capture is not None:
                self.capture.append(hcur.clone())
        res = add16(hcur, res)
        self.tokens += T
        return rmsnorm(res, self.norm_f, self.eps)

    def logits(self, hidden16):
        return linear(hidden16.reshape(-1, D_MODEL), self.head16)

    def nll(self, hidden16, targets):
        lg = self.logits(hidden16).float()
        return torch.nn.functional.cross_entropy(lg, torch.as_tensor(targets).reshape(-1).long(),
                                                 reduction='none').double()
