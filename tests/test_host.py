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
    """Stands in for PredictorState on CPU: deterministic per-token NLL from the ids."""
    device = torch.device('cpu')

    def backbone(self, ids, reset=False, out=None):
        return ids.double()[..., None]

    def score(self, hidden, targets, out=None):
        return ((hidden[..., 0] * 7 + targets) % 13).reshape(-1).double() / 3.0


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


def test_window_sharding_gloo_two_ranks():
    import socket
    import torch.multiprocessing as mp
    from sq325.scoring import evaluate_ppl, ppl_windows
    ids = np.random.default_rng(0).integers(0, 1000, 5 * 16 + 7)
    windows = [(s, torch.from_numpy(w)) for s, w in ppl_windows(ids, 16)]
    single = evaluate_ppl(_FakeExecution(), windows, batch_windows=2)
    s = socket.socket(); s.bind(('127.0.0.1', 0)); port = s.getsockname()[1]; s.close()
    ctx = mp.get_context('spawn')
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, windows, q)) for r in range(2)]
    for p in procs:
        p.start()
    nll, count, starts = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert math.isclose(nll, single['nll'], rel_tol=1e-12)
    assert count == single['target_tokens']
    assert starts == [w[0] for w in windows]
