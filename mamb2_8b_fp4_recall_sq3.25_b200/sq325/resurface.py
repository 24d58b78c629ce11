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
    base_hashes: dict = None  # the base-parameter ledger given to install_fp16, if any

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


def tensor_hash(value):
    """sha256 of a tensor's bytes in row order (resurface_native.tensor_hash, :49-57)."""
    import hashlib
    t = value.detach()
    return hashlib.sha256(t.cpu().contiguous().view(torch.uint8).numpy().tobytes()).hexdigest()


def base_parameter_names(model):
    """The base model's parameter names as the reference's MambaLMHeadModel names them."""
    from .checkpoint import tensor_inventory
    return set(tensor_inventory(model.n_layer, model.vocab))


@torch.no_grad()
def base_tensor_hashes(model, chunk_rows=16384):
    """sha256 ledger of the base parameters under the reference's names, as ResurfaceNative
    hashes them (resurface_native.py:140-141, 285-297): the FP4 matrices as their decoded
    FP16 weights (decoded on the device in row chunks, hashed in row order), the fp16
    tensors as stored (conv1d.weight as its [10240, 1, 4] bytes, identical to [10240, 4])."""
    import hashlib
    from . import fp4 as F
    out = {}

    def packed(name, w):
        d = hashlib.sha256()
        for r0 in range(0, w.rows, chunk_rows):
            rows = min(chunk_rows, w.rows - r0)
            part = F.Fp4Tensor(w.codes[r0:r0 + rows], w.block_scale_bytes[r0:r0 + rows], w.global_scale,
                               (rows, w.cols))
            d.update(F.decode_packet(part).cpu().numpy().tobytes())
        out[name] = d.hexdigest()

    packed('backbone.embedding.weight', model.embedding)
    packed('lm_head.weight', model.lm_head)
    out['backbone.norm_f.weight'] = tensor_hash(model.norm_f)
    for i, L in enumerate(model.layers):
        p = f'backbone.layers.{i}.'
        packed(p + 'mixer.in_proj.weight', L.in_proj)
        packed(p + 'mixer.out_proj.weight', L.out_proj)
        for name, t in (('norm.weight', L.norm_weight), ('mixer.A_log', L.A_log), ('mixer.D', L.D),
                        ('mixer.dt_bias', L.dt_bias), ('mixer.conv1d.weight', L.conv_weight),
                        ('mixer.conv1d.bias', L.conv_bias), ('mixer.norm.weight', L.gated_norm_weight)):
            out[p + name] = tensor_hash(t)
    return out


def install_fp16(model, path, *, expected_binding=None, expected_base_hashes=None):
    """Load an exported adapter onto `model` (replaces resurface_native.install_fp16, :363-375).

    expected_base_hashes, when given, is the independently supplied ledger of the base
    parameters (name -> sha256): it must cover every base parameter exactly (ValueError as in
    ResurfaceNative.__init__ :140-142) and is kept for `assert_base_frozen(check_values=True)`."""
    if getattr(model, 'adapter', None) is not None:
        raise RuntimeError('A Resurface adapter is already attached to this model')
    if expected_base_hashes is not None and set(expected_base_hashes) != base_parameter_names(model):
        raise ValueError('Expected base ledger must cover every original parameter')
    payload = read_fp16(path, expected_binding)
    bank = bank_from_payload(payload, model.n_layer, model.device)
    bank.base_hashes = dict(expected_base_hashes) if expected_base_hashes is not None else None
    model.adapter = bank
    return model.adapter


def assert_base_frozen(model, check_values=False):
    """ResurfaceNative.assert_base_frozen (:285-300): with check_values the base parameters'
    content is re-hashed against the ledger given to install_fp16."""
    bank = getattr(model, 'adapter', None)
    if bank is None:
        raise RuntimeError('No Resurface adapter is attached to this model')
    if check_values:
        if bank.base_hashes is None:
            raise ValueError('Content audit requires an independently supplied base hash ledger')
        now = base_tensor_hashes(model)
        for name, digest in now.items():
            if digest != bank.base_hashes[name]:
                raise RuntimeError(f'Base content changed: {name}')
    return {'tensors': len(base_parameter_names(model)), 'actual_content_checked': bool(check_values)}


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
