"""Resurface post-D adapter: file format and installation (inference only).

Export format of mamba2_recall/resurface_native.py:338-375 (read_fp16 / install_fp16):
a torch-saved dict {'format','variant','gate_mode','geometry','binding','tensors'} with
per-layer fp16 tensors layer{i}.V_read [H,H], g_read [H], router_w [D], router_b [].
Forward semantics (_Adapter.forward :105-118) run inside the fused
resurface + gated-RMSNorm kernel of libsq325.so.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

FORMAT = 'MAMBA2_POST_D_RESURFACE_FP16_V1'
FIELDS = ('V_read', 'g_read', 'router_w', 'router_b')
VARIANT = 'post-D native norm-prehook; memoryless cross-head mixing'


@dataclass
class AdapterBank:
    gate_mode: str          # 'soft' | 'hard'
    V: list                 # per layer fp16 [128,128]
    g: list                 # fp16 [128]
    w: list                 # fp16 [4096]
    b: list                 # fp16 [1]

    @property
    def nbytes(self):
        return sum(t.numel() * 2 for lst in (self.V, self.g, self.w, self.b) for t in lst)


def read_fp16(path, expected_binding=None):
    """Parse and validate an exported adapter file (same checks as the reference :338-360)."""
    payload = torch.load(path, map_location='cpu', weights_only=True)
    if (set(payload) != {'format', 'variant', 'gate_mode', 'geometry', 'binding', 'tensors'}
            or payload['format'] != FORMAT or payload['variant'] != VARIANT
            or payload['gate_mode'] not in ('soft', 'hard') or not isinstance(payload['binding'], dict)):
        raise ValueError('Invalid Resurface export header')
    if expected_binding is not None and payload['binding'] != expected_binding:
        raise ValueError('Resurface binding differs')
    expected = {}
    for index, geo in enumerate(payload['geometry']):
        if set(geo) != {'width', 'heads', 'head_dim'} or any(type(v) is not int or v <= 0 for v in geo.values()):
            raise ValueError('Invalid export geometry')
        expected.update({f'layer{index}.{name}': shape for name, shape in {
            'V_read': (geo['heads'], geo['heads']), 'g_read': (geo['heads'],),
            'router_w': (geo['width'],), 'router_b': ()}.items()})
    if not expected or set(payload['tensors']) != set(expected):
        raise ValueError('Export tensor inventory differs')
    for name, shape in expected.items():
        v = payload['tensors'][name]
        if (not isinstance(v, torch.Tensor) or v.dtype != torch.float16 or tuple(v.shape) != shape
                or not bool(torch.isfinite(v).all())):
            raise ValueError(f'Invalid exported tensor: {name}')
    return payload


def bank_from_payload(payload, n_layer, device):
    geo = payload['geometry']
    if len(geo) != n_layer or any(g != {'width': 4096, 'heads': 128, 'head_dim': 64} for g in geo):
        raise ValueError('Export does not fit actual native model')
    t = payload['tensors']
    get = lambda i, k: t[f'layer{i}.{k}'].to(device=device, dtype=torch.float16).contiguous()
    return AdapterBank(payload['gate_mode'], [get(i, 'V_read') for i in range(n_layer)],
                       [get(i, 'g_read') for i in range(n_layer)], [get(i, 'router_w') for i in range(n_layer)],
                       [get(i, 'router_b').reshape(1) for i in range(n_layer)])


def install_fp16(model, path, *, expected_binding=None, expected_base_hashes=None):
    """Load an exported adapter onto `model` (replaces resurface_native.install_fp16)."""
    if getattr(model, 'adapter', None) is not None:
        raise RuntimeError('A Resurface adapter is already attached to this model')
    payload = read_fp16(path, expected_binding)
    model.adapter = bank_from_payload(payload, model.n_layer, model.device)
    return model.adapter


def remove(model):
    model.adapter = None


def export_fp16(bank, path, binding=None):
    """Write a bank in the reference's export format (used to round-trip test files)."""
    n = len(bank.V)
    tensors = {}
    for i in range(n):
        tensors[f'layer{i}.V_read'] = bank.V[i].cpu()
        tensors[f'layer{i}.g_read'] = bank.g[i].cpu()
        tensors[f'layer{i}.router_w'] = bank.w[i].cpu()
        tensors[f'layer{i}.router_b'] = bank.b[i].reshape(()).cpu()
    torch.save({'format': FORMAT, 'variant': VARIANT, 'gate_mode': bank.gate_mode,
                'geometry': [{'width': 4096, 'heads': 128, 'head_dim': 64}] * n, 'binding': binding or {},
                'tensors': tensors}, path)


@torch.no_grad()
def random_bank(n_layer, seed=5, device='cuda', gate_mode='soft'):
    """Random adapter of the recorded shape (V ~ N(0, .02), g ~ U[.5,1.5], w ~ N(0, .01),
    b = -4 as at initialisation)."""
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    mk = lambda shape, f: f(torch.empty(shape, device=device, dtype=torch.float32)).half().contiguous()
    return AdapterBank(
        gate_mode,
        [mk((128, 128), lambda t: t.normal_(0, 0.02, generator=gen)) for _ in range(n_layer)],
        [mk((128,), lambda t: t.uniform_(0.5, 1.5, generator=gen)) for _ in range(n_layer)],
        [mk((4096,), lambda t: t.normal_(0, 0.01, generator=gen)) for _ in range(n_layer)],
        [torch.full((1,), -4.0, device=device, dtype=torch.float16) for _ in range(n_layer)])
