"""The MK recall harness end to end on the GPU (sq325.recall, the reference's
mamba2_recall/evaluation.py:82-190 protocol): prefill, greedy decode of at most 12 tokens
through the persistent batch-1 kernel, six-digit matching and the summaries.  A character
tokenizer over a small-vocabulary model stands in for the release's SentencePiece model."""
import numpy as np
import pytest
import torch

from _models import build_pair

pytestmark = pytest.mark.gpu


class CharTokenizer:
    eos_token_id = 0

    def encode(self, text):
        return [min(ord(c), 511) for c in text]

    def decode(self, ids):
        return ''.join(chr(i) if 32 <= i < 127 or i == 10 else '' for i in ids)


def test_mk_harness_generates_the_eager_greedy_tokens():
    from sq325 import PredictorState
    from sq325.recall import evaluate_mk, synthetic_mk_cases
    gm, ora, statics = build_pair(n_layer=2, vocab=512, seed=13, adapter=True)
    cases = synthetic_mk_cases('test', 2)[:3]
    tok = CharTokenizer()
    with PredictorState(gm, *statics) as ex:
        fast = evaluate_mk(ex, tok, cases=cases, persistent=True)
        slow = evaluate_mk(ex, tok, cases=cases, persistent=False)
        ex.check()
    assert [r['generated_ids'] for r in fast['rows']] == [r['generated_ids'] for r in slow['rows']]
    for r in fast['rows']:
        assert 1 <= len(r['generated_ids']) <= 12
        assert r['prediction_category'] in ('correct_target', 'removed_target_match', 'unparseable',
                                            'wrong_present_value', 'other_present_value', 'not_present_value')
    assert fast['summary']['normal']['count'] + fast['summary']['target_removed']['count'] == len(cases)
    # the first generated token is the oracle model's greedy pick after the same prompt
    ids = tok.encode(cases[0]['prompt'])
    ora.reset(1)
    logits = ora.logits(ora.backbone(np.asarray([ids]))[:, -1]).float()
    top2 = torch.topk(logits[0], 2).values
    if float(top2[0] - top2[1]) > 1e-2:                 # skip a near-tie
        assert int(logits[0].argmax()) == fast['rows'][0]['generated_ids'][0]
