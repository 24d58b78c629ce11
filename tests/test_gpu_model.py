"""GPU parity of the full native model path (embedding -> layers -> norm_f -> heads)
against the CPU oracle on matched tiny models (real layer geometry, 2 layers)."""
import math

import numpy as np
import pytest
import torch

from _models import build_pair, rel_l2

pytestmark = pytest.mark.gpu

NLL_RTOL = 1e-3      # north-star tolerance on per-window NLL


@pytest.fixture(scope='module')
def pair():
    return build_pair(n_layer=2, vocab=512, seed=1, adapter=True)


@pytest.fixture(scope='module')
def hard_pair():
    return build_pair(n_layer=2, vocab=512, seed=3, adapter=True, hard=True)


def _ids(rng, B, T, vocab):
    return rng.integers(0, vocab, (B, T)).astype(np.int64)


@pytest.mark.parametrize('B,T', [(2, 16), (2, 48)])
def test_prefill_hidden_and_nll(pair, B, T):
    from sq325 import PredictorState
    gm, ora, statics = pair
    rng = np.random.default_rng(B * 100 + T)
    ids = _ids(rng, B, T + 1, gm.vocab)
    with PredictorState(gm, *statics) as ex:
        hid = ex.backbone(torch.from_numpy(ids[:, :-1]).cuda(), reset=True)
        nll = ex.score(hid, torch.from_numpy(ids[:, 1:]).cuda())
        torch.cuda.synchronize()
        ex.check()
    ora.reset(B)
    href = ora.backbone(ids[:, :-1])
    nref = ora.nll(href, ids[:, 1:])
    assert rel_l2(hid.float(), href.float()) < 2e-2
    got = nll.double().cpu().view(B, T).sum(1)
    exp = nref.view(B, T).sum(1)
    assert torch.allclose(got, exp, rtol=NLL_RTOL, atol=0), (got, exp)


@pytest.mark.parametrize('exact', [False, True])
def test_decode_steps_and_greedy(pair, exact):
    """Decode-time projections (<= 64 rows) in both numerics: factored global scale (default)
    and per-weight fp16 decode; both against the oracle's decoded-FP16-weight model."""
    from sq325 import PredictorState
    gm, ora, statics = pair
    rng = np.random.default_rng(5)
    B, T = 2, 12
    ids = _ids(rng, B, T, gm.vocab)
    with PredictorState(gm, *statics) as ex:
        ex.set_exact_projections(exact)
        h = ex.backbone(torch.from_numpy(ids).cuda(), reset=True)
        ora.reset(B)
        hr = ora.backbone(ids)
        assert rel_l2(h.float(), hr.float()) < 2e-2
        for step in range(4):
            nxt = rng.integers(0, gm.vocab, (B, 1)).astype(np.int64)
            h = ex.backbone(torch.from_numpy(nxt).cuda())
            hr = ora.backbone(nxt)
            assert rel_l2(h.float(), hr.float()) < 3e-2, step
            # conv ring in the reference's chronological order; it holds raw in_proj
            # outputs, which carry the upstream layers' (tolerance-level) differences
            for layer in range(gm.n_layer):
                got = ex.conv_chronological(layer).cpu().float()
                ref = ora.caches[layer]['conv'].float()
                assert rel_l2(got, ref) < 2e-2, (step, layer)
        logits = torch.empty(B, gm.vocab, device='cuda', dtype=torch.float16)
        tok = ex.greedy(h[:, -1], logits=logits)
        torch.cuda.synchronize()
        lref = ora.logits(h[:, -1].cpu())
        assert rel_l2(logits.float(), lref.float()) < 1e-2
        # argmax of the GPU's own fp16 logits, first index on ties
        assert torch.equal(tok.cpu(), logits.float().cpu().argmax(-1))


def test_repeated_reset_is_bit_identical(pair):
    """scripts/run_fp4_ridge_resurface_v3.py:90-98: the same probe twice after reset gives
    identical hidden states and identical cache bytes."""
    from sq325 import PredictorState
    gm, _, statics = pair
    ids = torch.from_numpy(np.random.default_rng(9).integers(0, gm.vocab, (1, 128))).cuda()
    with PredictorState(gm, *statics) as ex:
        a = ex.backbone(ids, reset=True).clone()
        ca = [{k: v.clone() for k, v in e.state.tensors.items()} for e in ex._cache]
        b = ex.backbone(ids, reset=True)
        torch.cuda.synchronize()
        assert torch.equal(a, b)
        for x, e in zip(ca, ex._cache):
            for k in x:
                assert torch.equal(x[k].view(torch.uint8), e.state.tensors[k].view(torch.uint8))
        ex.assert_finite_cache()
        desc = ex.storage_descriptor()
        assert desc['row_bytes'] == 52 and len(desc['layers']) == gm.n_layer


def test_bad_token_id_is_reported(pair):
    from sq325 import PredictorState
    gm, _, statics = pair
    with PredictorState(gm, *statics) as ex:
        ids = torch.tensor([[1, 2, gm.vocab + 5]], device='cuda')
        ex.backbone(ids, reset=True)
        with pytest.raises(ValueError):
            ex.check()


def test_scoring_driver_pooled_ppl(pair):
    from sq325 import PredictorState, ppl_windows, evaluate_ppl
    gm, ora, statics = pair
    rng = np.random.default_rng(11)
    ids = rng.integers(0, gm.vocab, 3 * 32 + 11).astype(np.int64)
    windows = [(s, torch.from_numpy(w)) for s, w in ppl_windows(ids, 32)]
    assert [len(w) for _, w in windows] == [33, 33, 33, 11]
    with PredictorState(gm, *statics) as ex:
        res = evaluate_ppl(ex, windows, batch_windows=2)
    total = 0.0
    for (s, w), rec in zip(windows, res['windows']):
        ora.reset(1)
        hr = ora.backbone(w[None, :-1].numpy())
        ref = float(ora.nll(hr, w[None, 1:].numpy()).sum())
        assert math.isclose(rec['nll'], ref, rel_tol=NLL_RTOL), (rec['nll'], ref)
        total += ref
    assert math.isclose(res['nll'], total, rel_tol=NLL_RTOL)
    assert res['target_tokens'] == sum(len(w) - 1 for _, w in windows)


def test_graphed_decode_matches_eager(pair):
    """Greedy tokens from CUDA-graph replays (four residue graphs) equal the eager loop."""
    from sq325 import PredictorState, generate
    gm, _, statics = pair
    prompt = np.random.default_rng(21).integers(0, gm.vocab, (2, 9))
    with PredictorState(gm, *statics) as ex:
        eager = generate(ex, prompt, 11)
        graphed = generate(ex, prompt, 11, graphs=True)
        torch.cuda.synchronize()
        ex.check()
    assert eager.shape == (2, 11)
    assert torch.equal(eager.cpu(), graphed.cpu())


def test_factored_scale_projections_track_exact(pair):
    """The factored-scale decode-step projections differ from the per-weight fp16 decode only
    by the fp16 rounding of each weight: hidden states and logits agree closely."""
    from sq325 import PredictorState
    gm, _, statics = pair
    rng = np.random.default_rng(9)
    prompt = torch.from_numpy(_ids(rng, 1, 20, gm.vocab)).cuda()
    steps = [torch.from_numpy(_ids(rng, 1, 1, gm.vocab)).cuda() for _ in range(3)]
    outs = {}
    for exact in (True, False):
        with PredictorState(gm, *statics) as ex:
            ex.set_exact_projections(exact)
            ex.backbone(prompt, reset=True)
            for s in steps:
                h = ex.backbone(s)
            logits = torch.empty(1, gm.vocab, device='cuda', dtype=torch.float16)
            ex.greedy(h[:, -1], logits=logits)
            torch.cuda.synchronize()
            outs[exact] = (h.float(), logits.float())
    assert rel_l2(outs[False][0], outs[True][0]) < 5e-3
    assert rel_l2(outs[False][1], outs[True][1]) < 5e-3


@pytest.mark.parametrize('exact', [False, True])
def test_persistent_decode_matches_graph_replay(pair, exact):
    """The one-launch-per-token decode kernel reproduces the multi-kernel graph replay:
    identical greedy tokens, identical packed states and conv rings; with the factored global
    scale and with the exactly decoded fp16 weights (the reference's)."""
    from sq325 import PredictorState, generate
    gm, _, statics = pair
    prompt = np.random.default_rng(31).integers(0, gm.vocab, (1, 9))
    runs = {}
    for persistent in (False, True):
        with PredictorState(gm, *statics) as ex:
            ex.set_exact_projections(exact)
            seq = generate(ex, prompt, 13, graphs=True, persistent=persistent)
            torch.cuda.synchronize()
            ex.check()
            states = [{k: v.view(torch.uint8).clone() for k, v in e.state.tensors.items()} for e in ex._cache]
            rings = [ex.conv_chronological(l).clone() for l in range(gm.n_layer)]
            runs[persistent] = (seq.cpu(), states, rings)
    assert runs[True][0].shape == (1, 13)
    assert torch.equal(runs[True][0], runs[False][0])
    for a, b in zip(runs[True][1], runs[False][1]):
        for k in a:
            assert torch.equal(a[k], b[k]), k
    for a, b in zip(runs[True][2], runs[False][2]):
        assert torch.equal(a, b)


def test_persistent_decode_split_calls_match_one_call(pair):
    """Several tokens in one persistent launch equal the same tokens from separate calls."""
    from sq325 import PredictorState
    gm, _, statics = pair
    prompt = torch.from_numpy(np.random.default_rng(41).integers(0, gm.vocab, (1, 7))).cuda()
    outs = []
    for split in (False, True):
        with PredictorState(gm, *statics) as ex:
            tok = ex.greedy(ex.backbone(prompt, reset=True)[:, -1]).clone()
            if split:
                seq = torch.cat([ex.decode_persistent(tok, 3), ex.decode_persistent(tok, 2), ex.decode_persistent(tok, 4)])
            else:
                seq = ex.decode_persistent(tok, 9)
            torch.cuda.synchronize()
            ex.check()
            outs.append((seq.cpu(), [e.state.tensors['lo'].clone() for e in ex._cache]))
    assert torch.equal(outs[0][0], outs[1][0])
    for a, b in zip(outs[0][1], outs[1][1]):
        assert torch.equal(a, b)


def test_hard_gate_prefill_and_decode(hard_pair):
    """Resurface with the hard (threshold) gate (resurface_native.py:112-115): prefill hidden
    state, window NLL and decode steps against the oracle's hard-gate adapter."""
    from sq325 import PredictorState
    gm, ora, statics = hard_pair
    assert gm.adapter.gate_mode == 'hard'
    rng = np.random.default_rng(17)
    B, T = 2, 24
    ids = _ids(rng, B, T + 1, gm.vocab)
    with PredictorState(gm, *statics) as ex:
        hid = ex.backbone(torch.from_numpy(ids[:, :-1]).cuda(), reset=True)
        nll = ex.score(hid, torch.from_numpy(ids[:, 1:]).cuda())
        torch.cuda.synchronize()
        ex.check()
        ora.reset(B)
        href = ora.backbone(ids[:, :-1])
        nref = ora.nll(href, ids[:, 1:])
        assert rel_l2(hid.float(), href.float()) < 2e-2
        got = nll.double().cpu().view(B, T).sum(1)
        assert torch.allclose(got, nref.view(B, T).sum(1), rtol=NLL_RTOL, atol=0)
        for _ in range(3):
            nxt = rng.integers(0, gm.vocab, (B, 1)).astype(np.int64)
            h = ex.backbone(torch.from_numpy(nxt).cuda())
            assert rel_l2(h.float(), ora.backbone(nxt).float()) < 3e-2


def test_persistent_decode_matches_graph_replay_full_size():
    """The benchmarked size: 56 layers (released layouts), vocabulary 256,000, 16 greedy tokens
    after a 64-token prompt.  The one-launch persistent kernel and the multi-kernel CUDA-graph
    replay must give identical tokens, identical packed states and conv rings, with the
    factored global scale and with the exactly decoded fp16 weights (the reference's)."""
    from sq325 import model as M, resurface as R
    from sq325.state import PredictorState
    model = M.synthetic_model(seed=4, n_layer=56, vocab=256000, device='cuda')
    model.adapter = R.random_bank(56, seed=5, device='cuda')
    statics = M.synthetic_statics(M.RELEASED_LAYOUTS, seed=4, device='cuda')
    prompt = torch.from_numpy(np.random.default_rng(77).integers(0, 256000, (1, 64))).cuda()
    for exact in (False, True):
        runs = {}
        for persistent in (False, True):
            with PredictorState(model, *statics) as ex:
                ex.set_exact_projections(exact)
                tok = ex.greedy(ex.backbone(prompt, reset=True)[:, -1]).clone()
                if persistent:
                    seq = ex.decode_persistent(tok, 16)
                else:
                    ex.capture_decode(tok)
                    seq = ex.replay_decode(16)
                torch.cuda.synchronize()
                ex.check()
                states = [{k: v.view(torch.uint8).clone() for k, v in e.state.tensors.items()} for e in ex._cache]
                rings = [ex.conv_chronological(l).clone() for l in range(56)]
                runs[persistent] = (seq.cpu(), states, rings)
                del ex
        assert torch.equal(runs[True][0], runs[False][0]), (exact, runs[True][0].ravel(), runs[False][0].ravel())
        for layer, (a, b) in enumerate(zip(runs[True][1], runs[False][1])):
            for k in a:
                assert torch.equal(a[k], b[k]), (exact, layer, k)
        for a, b in zip(runs[True][2], runs[False][2]):
            assert torch.equal(a, b), exact


def test_projection_gemm_timer_counts_large_m_launches(pair):
    """sq_model_time_gemm brackets every large-M in_proj GEMM launch (one per layer when
    batch x tokens > 256) and nothing else; records are discarded once read, and nothing is
    recorded after the timer is switched off."""
    from sq325 import PredictorState
    gm, _, statics = pair
    rng = np.random.default_rng(9)
    big = lambda: torch.from_numpy(_ids(rng, 2, 200, gm.vocab)).cuda()     # 400 rows: tcgen05 GEMM
    small = lambda: torch.from_numpy(_ids(rng, 2, 8, gm.vocab)).cuda()     # 16 rows: fused FP4 linear
    with PredictorState(gm, *statics) as ex:
        ex.reserve(400)
        ex.backbone(big(), reset=True)
        ex.time_projection_gemm(True)
        ex.backbone(big(), reset=True)
        ex.backbone(small(), reset=True)
        sec, n = ex.projection_gemm_time()
        assert n == gm.n_layer and sec > 0
        assert ex.projection_gemm_time() == (0.0, 0)
        ex.time_projection_gemm(False)
        ex.backbone(big(), reset=True)
        assert ex.projection_gemm_time() == (0.0, 0)
        ex.check()
