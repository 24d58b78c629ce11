"""Packed checkpoint container (reference fp4_checkpoint format) and state_config.pt I/O."""
import json

import numpy as np
import pytest
import torch


@pytest.fixture(scope='module')
def tiny():
    from sq325 import model as M
    return M.synthetic_model(seed=3, n_layer=2, vocab=64, device='cpu')


def test_plan_matches_reference_rule():
    from sq325 import checkpoint as ck
    inv = ck.tensor_inventory(56, 256000)
    assert len(inv) == 507
    assert sum(1 for k in inv.values() if k[0] == 'fp4_g16_e4m3') == 114
    plan = ck.make_plan(inv, 256 * 1024 * 1024)
    head = plan['lm_head.weight']
    per_row = 4096 // 2 + 4096 // 16
    rows = (256 * 1024 * 1024 - 4) // per_row // 512 * 512
    assert [p['row_stop'] - p['row_start'] for p in head['parts'][:-1]] == [rows] * (len(head['parts']) - 1)
    assert head['parts'][0]['file'].startswith('weights-fp4-') and head['global_scale_file'] == head['parts'][0]['file']
    assert {p['file'] for p in plan.values() if p['kind'] == 'fp16'} == {ck.FP16_FILE}


def test_export_verify_load_round_trip(tiny, tmp_path):
    from sq325 import checkpoint as ck
    d = tmp_path / 'weights'
    ck.export_packed(tiny, d, shard_limit_bytes=1024 * 1024)
    manifest, headers, plan = ck.verify_checkpoint(d)
    assert len(plan) == len(ck.tensor_inventory(2, 64))
    # the 2 MB-ish in_proj matrices are split into several row parts
    assert len(plan['backbone.layers.0.mixer.in_proj.weight']['parts']) > 1
    back = ck.load_packed_model(d, device='cpu')
    pairs = [(tiny.embedding, back.embedding), (tiny.lm_head, back.lm_head)]
    pairs += [(a.in_proj, b.in_proj) for a, b in zip(tiny.layers, back.layers)]
    pairs += [(a.out_proj, b.out_proj) for a, b in zip(tiny.layers, back.layers)]
    for a, b in pairs:
        assert torch.equal(a.codes, b.codes) and torch.equal(a.block_scale_bytes, b.block_scale_bytes)
        assert torch.equal(a.global_scale, b.global_scale)
    for a, b in zip(tiny.layers, back.layers):
        for k in ('norm_weight', 'conv_weight', 'conv_bias', 'A_log', 'D', 'dt_bias', 'gated_norm_weight', 'A'):
            assert torch.equal(getattr(a, k), getattr(b, k)), k
    assert torch.equal(tiny.norm_f, back.norm_f)


def test_verify_detects_corruption(tiny, tmp_path):
    from sq325 import checkpoint as ck
    d = tmp_path / 'w'
    ck.export_packed(tiny, d, shard_limit_bytes=1024 * 1024)
    victim = sorted(d.glob('weights-fp4-*.safetensors'))[0]
    raw = bytearray(victim.read_bytes())
    raw[-1] ^= 0xFF
    victim.write_bytes(bytes(raw))
    with pytest.raises(ValueError):
        ck.verify_checkpoint(d)
    with pytest.raises(ValueError):
        ck.verify_checkpoint(d, pinned=True)


def test_state_config_round_trip(tmp_path):
    from sq325 import checkpoint as ck
    from sq325 import model as M
    table, layouts, bases, scales, preds = M.synthetic_statics(M.RELEASED_LAYOUTS[:3], seed=1, device='cpu')
    path = tmp_path / 'state_config.pt'
    ck.write_state_config(path, table, layouts, bases, scales, preds)
    t2, l2, b2, s2, p2 = ck.read_state_config(path)
    assert torch.equal(t2, table) and l2 == layouts
    assert all(torch.equal(a, b) for a, b in zip(b2 + s2 + p2, bases + scales + preds))
    bad = table.clone(); bad[0, 0, :2] = 0
    with pytest.raises(ValueError):
        ck.write_state_config(tmp_path / 's2.pt', bad, layouts, bases, scales, preds)
        ck.read_state_config(tmp_path / 's2.pt')


def _canon(x):
    import hashlib
    return hashlib.sha256(json.dumps(x, sort_keys=True, separators=(',', ':')).encode()).hexdigest()


@pytest.mark.parametrize('key', ['production', 'small'])
def test_plan_specs_headers_match_reference_outputs(key):
    """make_plan / file_specs / header_bytes against the reference's own make_plan, _file_specs
    and _header (mamba2_recall/fp4_checkpoint.py:67-127) run on the same inventory
    (tests/golden/checkpoint_plan.json, written by make_golden.py)."""
    from conftest import GOLDEN
    from sq325 import checkpoint as ck
    gold = json.loads((GOLDEN / 'checkpoint_plan.json').read_text())[key]
    for limit, rec in gold.items():
        inv = ck.tensor_inventory(rec['n_layer'], rec['vocab'])
        plan = ck.make_plan(inv, int(limit))
        specs = ck.file_specs(plan)
        assert len(plan) == rec['tensors'] and len(specs) == rec['files']
        assert _canon(plan) == rec['plan_sha256'] and _canon(specs) == rec['specs_sha256']
        import hashlib
        for f, spec in specs.items():
            raw, _, payload = ck.header_bytes(spec)
            assert hashlib.sha256(raw).hexdigest() == rec['headers_sha256'][f], f
            assert payload == rec['payload_bytes'][f], f


def test_exported_shards_carry_the_reference_headers(tiny, tmp_path):
    """Every shard export_packed writes starts with the exact header bytes the reference's
    _header builds for that file (golden, 2 layers / 64 rows at a 1 MiB limit), and its size
    is 8 + header + payload as the reference's inspect_shard requires (:147-164)."""
    import struct
    from conftest import GOLDEN
    from sq325 import checkpoint as ck
    rec = json.loads((GOLDEN / 'checkpoint_plan.json').read_text())['small'][str(1024 * 1024)]
    d = tmp_path / 'weights'
    ck.export_packed(tiny, d, shard_limit_bytes=1024 * 1024)
    manifest = json.loads((d / 'weight_manifest.json').read_text())
    assert manifest['layout'] == rec['plan']
    assert set(rec['headers_hex']) <= {p.name for p in d.glob('*.safetensors')}
    for f, hexraw in rec['headers_hex'].items():
        raw = bytes.fromhex(hexraw)
        blob = (d / f).read_bytes()
        (n,) = struct.unpack('<Q', blob[:8])
        assert blob[8:8 + n] == raw, f
        assert len(blob) == 8 + n + rec['payload_bytes'][f], f
