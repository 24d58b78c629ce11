"""Packed FP4-G16 checkpoint I/O that keeps the weights packed (no decode to FP16).

On-disk format of mamba2_recall/fp4_checkpoint.py (FORMAT MAMBA2_FP4_G16_PACKED_CHECKPOINT_V1):
safetensors shards with a deterministic header (`__metadata__` first, tensor entries in
sorted order, JSON without spaces, space-padded to a multiple of 8 bytes).  FP4 matrices
are split into row parts of at most `shard_limit_bytes` (rounded to 512-row chunks), each
part holding `codes` U8[rows, cols/2] and `block_scale_bytes` U8[rows, cols/16]; the
first part also holds `global_scale` F32[].  All FP16 tensors live in
`weights-retained-fp16.safetensors` (plan: :67-93, file specs: :100-114, header: :117-127).

`load_packed_model` replaces the reference loader (:345-403): instead of decoding every
chunk to a resident FP16 parameter it uploads the packed bytes as they are, and the
kernels decode on the fly.  `verify_checkpoint` checks the container, the deterministic
headers, file sizes and the SHA256SUMS list; `pinned=True` additionally requires the
reference's pinned ledger identity (only a real release bundle passes that).

`read_state_config` / `write_state_config` handle state_config.pt
(scripts/infer_fp4_ridge_resurface_v1.py:21-46, scripts/release_fp4_ridge_resurface_v1.py:372-375).
"""
from __future__ import annotations

import hashlib
import json
import math
import struct
from pathlib import Path

import numpy as np
import torch

from . import fp4 as F
from . import model as M

FORMAT = 'MAMBA2_FP4_G16_PACKED_CHECKPOINT_V1'
STATE_FORMAT = 'MAMBA2_FP4_G16_SQ325_RIDGE_STATE_V1'
LEDGER_SHA = '55de4189a7e04c9564a48b0fbb5f37428d3d1bb5b6274831d878b41ef4686c9b'
PAYLOAD_BYTES = 4_638_460_360
DTYPE_BYTES = {'U8': 1, 'F16': 2, 'F32': 4}
MAX_HEADER_BYTES = 8 * 1024 * 1024
FP16_FILE = 'weights-retained-fp16.safetensors'


def need(cond, msg):
    if not cond:
        raise ValueError(msg)


def sha_file(path):
    d = hashlib.sha256()
    with Path(path).open('rb') as f:
        for part in iter(lambda: f.read(8 * 1024 * 1024), b''):
            d.update(part)
    return d.hexdigest()


def tensor_hash(t):
    """sha256 of a tensor's little-endian bytes (resurface_native.tensor_hash)."""
    return hashlib.sha256(t.detach().cpu().contiguous().view(torch.uint8).numpy().tobytes()).hexdigest()


# ------------------------------------------------------------------ inventory

def tensor_inventory(n_layer=56, vocab=256000):
    """mamba_ssm state-dict names -> (kind, shape) of the 8B model (507 tensors at 56 layers)."""
    inv = {'backbone.embedding.weight': ('fp4_g16_e4m3', [vocab, 4096]),
           'lm_head.weight': ('fp4_g16_e4m3', [vocab, 4096]),
           'backbone.norm_f.weight': ('fp16', [4096])}
    for i in range(n_layer):
        p = f'backbone.layers.{i}.'
        inv.update({p + 'norm.weight': ('fp16', [4096]),
                    p + 'mixer.A_log': ('fp16', [128]), p + 'mixer.D': ('fp16', [128]),
                    p + 'mixer.dt_bias': ('fp16', [128]),
                    p + 'mixer.conv1d.weight': ('fp16', [10240, 1, 4]), p + 'mixer.conv1d.bias': ('fp16', [10240]),
                    p + 'mixer.in_proj.weight': ('fp4_g16_e4m3', [18560, 4096]),
                    p + 'mixer.out_proj.weight': ('fp4_g16_e4m3', [4096, 8192]),
                    p + 'mixer.norm.weight': ('fp16', [8192])})
    return inv


def make_plan(tensors, shard_limit_bytes):
    """File plan: same rule as the reference (one FP16 file; FP4 matrices split into row
    parts of at most shard_limit_bytes, rounded down to 512-row multiples)."""
    need(type(shard_limit_bytes) is int and shard_limit_bytes >= 1024 * 1024,
         'Shard limit must be an integer of at least one MiB')
    plan, serial = {}, 0
    for name, item in sorted(tensors.items()):
        kind, shape = (item['kind'], item['shape']) if isinstance(item, dict) else item
        if kind == 'fp16':
            plan[name] = {'kind': 'fp16', 'shape': list(shape), 'file': FP16_FILE, 'key': name}
            continue
        need(kind == 'fp4_g16_e4m3' and len(shape) == 2 and shape[1] % 16 == 0, 'Unexpected quantized matrix')
        rows, cols = shape
        per_row = cols // 2 + cols // 16
        max_rows = max(1, (shard_limit_bytes - 4) // per_row)
        if max_rows >= 512:
            max_rows = (max_rows // 512) * 512
        serial += 1
        parts = [{'file': f'weights-fp4-{serial:03d}-part-{n:03d}.safetensors', 'row_start': s,
                  'row_stop': min(rows, s + max_rows)} for n, s in enumerate(range(0, rows, max_rows), 1)]
        plan[name] = {'kind': 'fp4_g16_e4m3', 'shape': list(shape), 'parts': parts,
                      'global_scale_file': parts[0]['file']}
    return plan


def file_specs(plan):
    out = {FP16_FILE: {}}
    for name, item in plan.items():
        if item['kind'] == 'fp16':
            out[item['file']][name] = {'dtype': 'F16', 'shape': item['shape']}
            continue
        cols = item['shape'][1]
        for i, part in enumerate(item['parts']):
            rows = part['row_stop'] - part['row_start']
            spec = {'codes': {'dtype': 'U8', 'shape': [rows, cols // 2]},
                    'block_scale_bytes': {'dtype': 'U8', 'shape': [rows, cols // 16]}}
            if i == 0:
                spec['global_scale'] = {'dtype': 'F32', 'shape': []}
            out[part['file']] = spec
    return out


def header_bytes(spec):
    """Deterministic safetensors header -> (raw bytes, parsed dict, payload size)."""
    offset = 0
    header = {'__metadata__': {'format': FORMAT, 'scale_bytes': 'float8_e4m3fn'}}
    for name, item in sorted(spec.items()):
        size = math.prod(item['shape']) * DTYPE_BYTES[item['dtype']]
        header[name] = dict(item, data_offsets=[offset, offset + size])
        offset += size
    raw = json.dumps(header, separators=(',', ':'), allow_nan=False).encode()
    raw += b' ' * ((-len(raw)) % 8)
    return raw, header, offset


def inspect_shard(path, spec):
    path = Path(path)
    need(path.is_file() and not path.is_symlink(), 'Expected regular safetensors shard')
    with path.open('rb') as f:
        prefix = f.read(8)
        need(len(prefix) == 8, 'Truncated safetensors header prefix')
        size = struct.unpack('<Q', prefix)[0]
        need(2 <= size <= MAX_HEADER_BYTES and size % 8 == 0, 'Invalid safetensors header size/alignment')
        raw = f.read(size)
        need(len(raw) == size, 'Truncated safetensors header')
    expected_raw, expected, payload = header_bytes(spec)
    need(raw == expected_raw and json.loads(raw) == expected, 'Shard tensor inventory/header differs from plan')
    need(path.stat().st_size == 8 + size + payload, 'Shard is truncated or has extra bytes')
    return 8 + size, expected


# ------------------------------------------------------------------ verify / load

def verify_checkpoint(directory, pinned=False):
    """Container-level verification (stdlib + numpy).  Returns (manifest, headers)."""
    d = Path(directory)
    need(d.is_dir() and not d.is_symlink(), 'Regular checkpoint directory required')
    manifest = json.loads((d / 'weight_manifest.json').read_text())
    need(manifest.get('format') == FORMAT and manifest.get('complete') is True, 'Not a complete FP4 G16 checkpoint')
    if pinned:
        need(sha_file(d / 'conversion_receipt.json') == LEDGER_SHA, 'The exact audited FP4 G16 ledger is required')
        need(manifest['logical_weight_payload_bytes'] == PAYLOAD_BYTES, 'Payload differs from the release')
    ledger = json.loads((d / 'conversion_receipt.json').read_text())
    plan = make_plan({k: {'kind': v['kind'], 'shape': v['shape']} for k, v in ledger['tensors'].items()},
                     manifest['shard_limit_bytes'])
    need(manifest['layout'] == plan, 'Manifest layout differs from the deterministic plan')
    specs = file_specs(plan)
    need(set(manifest['files']) == set(specs), 'Manifest shard inventory differs')
    headers = {}
    for name, spec in sorted(specs.items()):
        headers[name] = inspect_shard(d / name, spec)
        need(manifest['files'][name] == {'sha256': sha_file(d / name), 'bytes': (d / name).stat().st_size},
             'Shard file identity differs: ' + name)
    listed = sorted([*specs, 'conversion_receipt.json', 'weight_manifest.json'])
    expected_sums = ''.join(f'{sha_file(d / n)}  {n}\n' for n in listed)
    need((d / 'SHA256SUMS').read_text() == expected_sums, 'Checkpoint checksum list differs')
    return manifest, headers, plan


def _region(path, start, count):
    with Path(path).open('rb') as f:
        f.seek(start)
        data = f.read(count)
    need(len(data) == count, 'Truncated checkpoint data')
    return np.frombuffer(data, dtype=np.uint8)


def load_packed_model(directory, *, device='cuda', verify=True, pinned=False):
    """Build a Mamba2FP4Model whose 114 FP4 matrices stay packed on `device`."""
    d = Path(directory)
    if verify:
        manifest, headers, plan = verify_checkpoint(d, pinned=pinned)
    else:
        manifest = json.loads((d / 'weight_manifest.json').read_text())
        plan = manifest['layout']
        headers = {n: inspect_shard(d / n, s) for n, s in file_specs(plan).items()}
    names = set(plan)
    n_layer = sum(1 for n in names if n.endswith('.mixer.in_proj.weight'))
    vocab = plan['lm_head.weight']['shape'][0]
    need(names == set(tensor_inventory(n_layer, vocab)), 'Native model tensor inventory differs')

    def fp16(name):
        base, header = headers[plan[name]['file']]
        b, e = header[name]['data_offsets']
        arr = _region(d / plan[name]['file'], base + b, e - b).view(np.float16).reshape(plan[name]['shape'])
        return torch.from_numpy(arr.copy()).to(device)

    def packed(name):
        item = plan[name]
        rows, cols = item['shape']
        codes = np.empty((rows, cols // 2), np.uint8)
        scales = np.empty((rows, cols // 16), np.uint8)
        for part in item['parts']:
            base, header = headers[part['file']]
            r0, r1 = part['row_start'], part['row_stop']
            for key, dst, w in (('codes', codes, cols // 2), ('block_scale_bytes', scales, cols // 16)):
                b, e = header[key]['data_offsets']
                dst[r0:r1] = _region(d / part['file'], base + b, e - b).reshape(r1 - r0, w)
        base, header = headers[item['global_scale_file']]
        b, e = header['global_scale']['data_offsets']
        g = _region(d / item['global_scale_file'], base + b, e - b).view(np.float32)[0]
        need(np.isfinite(g) and g > 0, 'Global scale must be finite and positive: ' + name)
        return F.from_arrays(codes, scales, g, device=device)

    layers = []
    for i in range(n_layer):
        p = f'backbone.layers.{i}.'
        layers.append(M.MixerWeights(
            in_proj=packed(p + 'mixer.in_proj.weight'), out_proj=packed(p + 'mixer.out_proj.weight'),
            norm_weight=fp16(p + 'norm.weight'), conv_weight=fp16(p + 'mixer.conv1d.weight').reshape(10240, 4),
            conv_bias=fp16(p + 'mixer.conv1d.bias'), A_log=fp16(p + 'mixer.A_log'), D=fp16(p + 'mixer.D'),
            dt_bias=fp16(p + 'mixer.dt_bias'), gated_norm_weight=fp16(p + 'mixer.norm.weight')))
    model = M.Mamba2FP4Model(packed('backbone.embedding.weight'), packed('lm_head.weight'),
                             fp16('backbone.norm_f.weight'), layers, vocab=vocab,
                             meta=dict(checkpoint=str(d), manifest_sha256=sha_file(d / 'weight_manifest.json')))
    return model


# ------------------------------------------------------------------ export (for tests / converted models)

def _fp16_bytes(t):
    return t.detach().to('cpu', torch.float16).contiguous().view(torch.uint8).numpy().tobytes()


def export_packed(model, directory, shard_limit_bytes=256 * 1024 * 1024):
    """Write `model` in the packed checkpoint format (synthetic ledger; unpinned)."""
    d = Path(directory)
    need(not d.exists(), 'Fresh export directory required')
    d.mkdir(parents=True)
    tensors = {}

    def add(name, kind, value):
        tensors[name] = (kind, value)
    add('backbone.embedding.weight', 'fp4_g16_e4m3', model.embedding)
    add('lm_head.weight', 'fp4_g16_e4m3', model.lm_head)
    add('backbone.norm_f.weight', 'fp16', model.norm_f)
    for i, L in enumerate(model.layers):
        p = f'backbone.layers.{i}.'
        add(p + 'norm.weight', 'fp16', L.norm_weight)
        add(p + 'mixer.A_log', 'fp16', L.A_log)
        add(p + 'mixer.D', 'fp16', L.D)
        add(p + 'mixer.dt_bias', 'fp16', L.dt_bias)
        add(p + 'mixer.conv1d.weight', 'fp16', L.conv_weight.reshape(10240, 1, 4))
        add(p + 'mixer.conv1d.bias', 'fp16', L.conv_bias)
        add(p + 'mixer.in_proj.weight', 'fp4_g16_e4m3', L.in_proj)
        add(p + 'mixer.out_proj.weight', 'fp4_g16_e4m3', L.out_proj)
        add(p + 'mixer.norm.weight', 'fp16', L.gated_norm_weight)
    ledger = {'format_name': 'fp4_g16_e4m3', 'complete': True, 'synthetic': True,
              'tensors': {n: {'kind': k, 'shape': list(v.shape if k == 'fp4_g16_e4m3' else v.shape)}
                          for n, (k, v) in tensors.items()}}
    plan = make_plan({n: {'kind': k, 'shape': ledger['tensors'][n]['shape']} for n, (k, v) in tensors.items()},
                     shard_limit_bytes)
    specs = file_specs(plan)
    blobs = {name: {} for name in specs}
    for name, item in plan.items():
        kind, value = tensors[name]
        if kind == 'fp16':
            blobs[item['file']][name] = _fp16_bytes(value)
            continue
        codes, scales, g = value.to_numpy()
        for i, part in enumerate(item['parts']):
            r0, r1 = part['row_start'], part['row_stop']
            blobs[part['file']]['codes'] = np.ascontiguousarray(codes[r0:r1]).tobytes()
            blobs[part['file']]['block_scale_bytes'] = np.ascontiguousarray(scales[r0:r1]).tobytes()
            if i == 0:
                blobs[part['file']]['global_scale'] = np.float32(g).tobytes()
    for fname, spec in specs.items():
        raw, header, payload = header_bytes(spec)
        with (d / fname).open('xb') as f:
            f.write(struct.pack('<Q', len(raw)))
            f.write(raw)
            for key in sorted(spec):
                f.write(blobs[fname][key])
    (d / 'conversion_receipt.json').write_text(json.dumps(ledger, sort_keys=True, indent=2) + '\n')
    files = {n: {'sha256': sha_file(d / n), 'bytes': (d / n).stat().st_size} for n in sorted(specs)}
    manifest = {'format': FORMAT, 'complete': True, 'format_name': 'fp4_g16_e4m3',
                'logical_weight_payload_bytes': model.packed_weight_bytes() + model.fp16_parameter_bytes(),
                'packed_resident_kernel': True, 'custom_runtime': True, 'shard_limit_bytes': shard_limit_bytes,
                'layout': plan, 'files': files}
    (d / 'weight_manifest.json').write_text(json.dumps(manifest, sort_keys=True, indent=2) + '\n')
    listed = sorted([*specs, 'conversion_receipt.json', 'weight_manifest.json'])
    (d / 'SHA256SUMS').write_text(''.join(f'{sha_file(d / n)}  {n}\n' for n in listed))
    return manifest


# ------------------------------------------------------------------ state_config.pt

def write_state_config(path, table, layouts, bases, scales, predictors, provenance=None):
    prov = dict(provenance or {})
    prov.setdefault('table_sha256', tensor_hash(table))
    prov.setdefault('layouts', list(layouts))
    state = dict(format=STATE_FORMAT, provenance=prov, table=table.cpu().contiguous(), layouts=list(layouts),
                 bases=[x.cpu().contiguous() for x in bases], scales=[x.cpu().contiguous() for x in scales],
                 stackedpredictors=[x.cpu().contiguous() for x in predictors])
    with Path(path).open('xb') as f:
        torch.save(state, f)


def read_state_config(path, expected_provenance=None):
    """-> (table u8[L,8,128], layouts, bases, scales, predictors) with the reference's checks."""
    from .codec import layout_descriptor
    state = torch.load(path, map_location='cpu', weights_only=True)
    need(state.get('format') == STATE_FORMAT, 'State export format differs')
    if expected_provenance is not None:
        need(state['provenance'] == expected_provenance, 'State export/provenance differs')
    table = state['table']
    need(table.dtype == torch.uint8 and table.ndim == 3 and tuple(table.shape[1:]) == (8, 128) and
         torch.equal(table.sort(-1).values, torch.arange(128, dtype=torch.uint8).expand_as(table)),
         'State permutation table differs')
    prov = state['provenance']
    if 'table_sha256' in prov:
        need(tensor_hash(table) == prov['table_sha256'], 'State permutation table hash differs')
    layouts = tuple(state['layouts'])
    bases, scales, preds = state['bases'], state['scales'], state['stackedpredictors']
    need(len(layouts) == table.shape[0] == len(bases) == len(scales) == len(preds), 'Static state inventory differs')
    for layout, b, s, p in zip(layouts, bases, scales, preds):
        spec = layout_descriptor(layout)
        need(tuple(b.shape) == (8, spec['nzero'], 2) and tuple(s.shape) == (8, 2) and
             tuple(p.shape) == (8, spec['n8'] + spec['n4'] + 2, spec['nzero']), 'Static state tensor shape differs')
        need(all(t.dtype == torch.float16 and bool(torch.isfinite(t).all()) for t in (b, s, p)),
             'Static state dtype/finite differs')
    return table, layouts, bases, scales, preds
