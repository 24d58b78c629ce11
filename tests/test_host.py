"""Host-side logic that needs no GPU: controller validation, window geometry, the
adapter file format, and the sharded scoring reduction (gloo ranks on CPU)."""
import math
import os

import numpy as np
import pytest
import torch

from _models import build_pair


@pytest.fixture(scope='module')
def cpu_pair():
    return build_pair(n_layer=2, vocab=64, seed=2, adapter=True, device='cpu')


def test_controller_validation_and_ownership(cpu_pair):
    from sq325 import PredictorState
    gm, _, (table, layouts, bases, scales, preds) = cpu_pair
    with pytest.raises(ValueError):
        PredictorState(gm, table[:1], layouts, bases, scales, preds)
    bad = table.clone(); bad[0, 0, 0] = bad[0, 0, 1]
    with pytest.raises(ValueError):
        PredictorState(gm, bad, layouts, bases, scales, preds)
    with pytest.raises(ValueError):
        PredictorState(gm, table, layouts[:1], bases, scales, preds)
    ex = PredictorState(gm, table, layouts, bases, scales, preds)
    if not torch.cuda.is_available():
        # the native context needs a GPU: installation fails loudly, never falls back
        with pytest.raises(RuntimeError):
            ex.install()
        assert not ex._installed


def test_ppl_windows_geometry():
    from sq325 import ppl_windows
    ids = np.arange(2 * 2048 + 10)
    w = ppl_windows(ids, 2048)
    assert [s for s, _ in w] == [0, 2048, 4096]
    assert [len(x) for _, x in w] == [2049, 2049, 10]
    assert w[1][1][0] == w[0][1][-1]                 # one overlap token


def test_token_digest_matches_reference_definition():
    import hashlib
    from sq325.scoring import token_digest
    ids = np.array([1, 2, 255000], dtype=np.int64)
    assert token_digest(ids) == hashlib.sha256(ids.astype('<i8').tobytes()).hexdigest()


def test_adapter_export_round_trip(tmp_path):
    from sq325 import resurface as R
    bank = R.random_bank(3, seed=1, device='cpu')
    path = tmp_path / 'adapter_fp16.pt'
    R.export_fp16(bank, path, binding={'k': 'v'})
    payload = R.read_fp16(path, expected_binding={'k': 'v'})
    assert payload['gate_mode'] == 'soft'
    with pytest.raises(ValueError):
        R.read_fp16(path, expected_binding={'k': 'other'})
    back = R.bank_from_payload(payload, 3, 'cpu')
    for a, b in zip(bank.V + bank.g + bank.w + bank.b, back.V + back.g + back.w + back.b):
        assert torch.equal(a.reshape(-1), b.reshape(-1))
    assert bank.nbytes == 3 * (128 * 128 + 128 + 4096 + 1) * 2


class _FakeExecution:
    """Stands in for PredictorState on CPU: deterministic per-token NLL from the ids, and the
    controller attributes the report row reads (statics, caches, descriptors)."""
    device = torch.device('cpu')
    layouts = ('32_32_64', '8_80_40')
    bases = [torch.ones(8, 68, 2, dtype=torch.float16), torch.zeros(8, 44, 2, dtype=torch.float16)]
    latent_scales = [torch.ones(8, 2, dtype=torch.float16)] * 2
    predictors = [torch.zeros(8, 62, 68, dtype=torch.float16), torch.zeros(8, 86, 44, dtype=torch.float16)]

    def __init__(self):
        class _E:
            pass
        self._cache = []
        for _ in range(2):
            e = _E()
            e.state = type('S', (), {'tensors': {'lo': torch.zeros(1, 2, 2, dtype=torch.uint8)}})()
            self._cache.append(e)
        self.seen = None

    def backbone(self, ids, reset=False, out=None):
        self.seen = ids.clone()
        return ids.double()[..., None]

    def score(self, hidden, targets, out=None):
        return ((hidden[..., 0] * 7 + targets) % 13).reshape(-1).double() / 3.0

    def conv_chronological(self, layer):
        return self.seen.double().sum().reshape(1, 1, 1).half()

    def cache_breakdown(self):
        return {'total_bytes': 0}

    def storage_descriptor(self):
        return {'format': 'FP4_LATENT_STATE_STORAGE_V1'}


def _worker(rank, world, port, windows, q):
    import torch.distributed as dist
    from sq325.scoring import evaluate_ppl
    os.environ.update(MASTER_ADDR='127.0.0.1', MASTER_PORT=str(port))
    dist.init_process_group('gloo', rank=rank, world_size=world)
    try:
        res = evaluate_ppl(_FakeExecution(), windows, batch_windows=2, rank=rank, world=world)
        if rank == 0:
            q.put((res['nll'], res['target_tokens'], [r['start'] for r in res['windows']]))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize('world', [2, 4])
def test_window_sharding_gloo(world):
    import socket
    import torch.multiprocessing as mp
    from sq325.scoring import evaluate_ppl, ppl_windows
    ids = np.random.default_rng(0).integers(0, 1000, 5 * 16 + 7)
    windows = [(s, torch.from_numpy(w)) for s, w in ppl_windows(ids, 16)]
    single = evaluate_ppl(_FakeExecution(), windows, batch_windows=2)
    s = socket.socket(); s.bind(('127.0.0.1', 0)); port = s.getsockname()[1]; s.close()
    ctx = mp.get_context('spawn')
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, windows, q)) for r in range(world)]
    for p in procs:
        p.start()
    nll, count, starts = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert math.isclose(nll, single['nll'], rel_tol=1e-12)
    assert count == single['target_tokens']
    assert starts == [w[0] for w in windows]


def test_evaluate_ppl_report_row_and_probe(tmp_path):
    """The reference's report contract (run_fp4_ridge_resurface_v3.py:81-121): the row is
    written with the static hashes and the repeated-reset probe, rewritten per batch, and
    marked complete with the pooled figures."""
    import json
    from sq325.scoring import evaluate_ppl, ppl_windows
    ids = np.random.default_rng(1).integers(0, 1000, 3 * 16 + 5)
    windows = [(s, torch.from_numpy(w)) for s, w in ppl_windows(ids, 16)]
    path = tmp_path / 'ppl.json'
    res = evaluate_ppl(_FakeExecution(), windows, batch_windows=2, path=path, common={'arm': 'test'}, probe_tokens=8)
    row = json.loads(path.read_text())
    assert row['arm'] == 'test' and row['complete'] is True and row['ppl_complete'] is True
    assert row['layer_layouts'] == ['32_32_64', '8_80_40']
    assert len(row['static_basis_sha256']) == 2 and len(row['static_predictor_sha256'][0]) == 8
    probe = row['repeated_reset_probe']
    assert probe['tokens'] == 8 and probe['hidden_and_cache_exact'] is True
    assert set(probe['cache_tensor_sha256']) == {'0.lo', '0.conv', '1.lo', '1.conv'}
    assert math.isclose(row['ppl']['nll'], res['nll']) and row['ppl']['target_tokens'] == res['target_tokens']
    assert [w['start'] for w in row['ppl']['windows']] == [s for s, _ in windows]


def test_install_fp16_requires_a_complete_base_ledger(tmp_path):
    """ResurfaceNative's rule (resurface_native.py:140-142): an expected base ledger must name
    every base parameter, no more and no less."""
    from sq325 import model as M, resurface as R
    model = M.synthetic_model(seed=1, n_layer=2, vocab=64, device='cpu')
    path = tmp_path / 'adapter_fp16.pt'
    R.export_fp16(R.random_bank(2, seed=1, device='cpu'), path)
    names = R.base_parameter_names(model)
    assert len(names) == 3 + 9 * 2
    with pytest.raises(ValueError, match='cover every original parameter'):
        R.install_fp16(model, path, expected_base_hashes={n: '0' for n in list(names)[1:]})
    bank = R.install_fp16(model, path, expected_base_hashes={n: '0' for n in names})
    assert bank.base_hashes is not None and model.adapter is bank


def test_mk_cases_match_reference_digest():
    """sq325.recall.synthetic_mk_cases reproduces the reference's public MK prompts
    (mamba2_recall/evaluation.py:82-119) exactly: same canonical-JSON digest for both splits."""
    import hashlib
    import json
    from sq325.recall import synthetic_mk_cases
    from conftest import GOLDEN
    ref = json.loads((GOLDEN / 'mk_cases.json').read_text())
    for split in ('validation', 'test'):
        cases = [{k: v for k, v in c.items() if k != 'records'} for c in synthetic_mk_cases(split, 8)]
        raw = json.dumps(cases, sort_keys=True, separators=(',', ':')).encode()
        assert len(cases) == ref[split]['count'] == 96
        assert hashlib.sha256(raw).hexdigest() == ref[split]['sha256']


def test_mk_classification_and_matching():
    from sq325.recall import SIX_DIGITS, classify_prediction
    assert SIX_DIGITS.search(' 1234567 and 654321.').group() == '654321'
    row = dict(answer='600001', condition='normal', records=[(100001, 600001), (100002, 600002)])
    assert classify_prediction(dict(row, prediction='600001')) == 'correct_target'
    assert classify_prediction(dict(row, prediction='600002')) == 'wrong_present_value'
    assert classify_prediction(dict(row, prediction=None)) == 'unparseable'
    assert classify_prediction(dict(row, prediction='999999')) == 'not_present_value'
    assert classify_prediction(dict(row, condition='target_removed', prediction='600001')) == 'removed_target_match'
