"""Synthetic multi-key (MK) recall harness over a PredictorState.

Restates the reference's public MK protocol (mamba2_recall/evaluation.py:82-190,
"public-mamba8-mk-v1") and the scoring loop of scripts/run_fp4_ridge_resurface_v3.py:124-158:

  synthetic_mk_cases  seeded key/value record prompts in three templates at N = 16 / 64
                      records, the query position cycling over the sequence, each paired
                      with a control whose target record is replaced (evaluation.py:82-119)
  generate_greedy     prefill from a reset state, then greedy tokens, at most 12, stopping
                      at EOS (evaluation.py:122-146; run_fp4_ridge_resurface_v3.py:131-142);
                      batch 1 decode runs the persistent decode kernel when available
  evaluate_mk         prediction = the first standalone six-digit integer of the decoded
                      output, correct when it equals the answer; summary per condition, cells
                      per N x template x condition (evaluation.py:149-190), and the
                      prediction categories / strata of scripts/run_state_resurface_v11.py:162-194

The tokenizer is any object with encode(str) -> list[int], decode(list[int]) -> str and
eos_token_id (the release uses the model's SentencePiece tokenizer, absent here).
"""
from __future__ import annotations

import random
import re
import time

import numpy as np
import torch

from .scoring import token_digest

PROTOCOL = 'public-mamba8-mk-v1'
SIX_DIGITS = re.compile(r'(?<!\d)\d{6}(?!\d)')


def synthetic_mk_cases(split='test', samples_per_cell=8, sizes=(16, 64)):
    """Frozen public prompts; validation and test use disjoint keys and value ranges."""
    if split not in ('validation', 'test'):
        raise ValueError(split)
    offset = 0 if split == 'validation' else 100000
    rng = random.Random(834901 if split == 'validation' else 834902)
    cases = []
    for size in sizes:
        for template in range(3):
            for sample in range(samples_per_cell):
                keys = rng.sample(range(100000 + offset, 180000 + offset), size)
                values = rng.sample(range(600000 + offset, 680000 + offset), size)
                pairs = list(zip(keys, values))
                position = (sample * max(1, size - 1)) // max(1, samples_per_cell - 1)
                key, value = pairs[position]
                case_id = f'{split}-n{size}-t{template}-s{sample}'
                base = dict(id=case_id, N=size, template=template, query_position=position, key=key,
                            answer=str(value))
                cases.append(dict(base, prompt=_render(template, pairs, key), condition='normal', records=pairs))
                removed = pairs.copy()
                removed[position] = (190000 + offset + sample, 690000 + offset + sample)
                cases.append(dict(base, id=case_id + '-removed', prompt=_render(template, removed, key),
                                  condition='target_removed', records=removed))
    return cases


def _render(template, records, key):
    if template == 0:
        body = '\n'.join(f'{k}: {v}' for k, v in records)
        return f'Key-value records:\n{body}\n\nLookup the value for key {key}.\nValue:'
    if template == 1:
        body = '\n'.join(f'Key {k} has value {v}.' for k, v in records)
        return f'{body}\n\nQuestion: What is the value of key {key}?\nAnswer:'
    body = '\n'.join(f'{k} -> {v}' for k, v in records)
    return f'Dictionary:\n{body}\n\nReturn the stored value.\n{key} ->'


@torch.no_grad()
def generate_greedy(execution, ids, max_new_tokens=12, eos_token_id=None, persistent=True):
    """Greedy tokens after a prefill of `ids` (int list) from a reset state: at most
    max_new_tokens, stopping at (and including) EOS."""
    if len(ids) == 0:
        raise ValueError('Empty recall prompt')
    prompt = torch.tensor(ids, dtype=torch.long, device=execution.device)[None]
    hidden = execution.backbone(prompt, reset=True)[:, -1]
    tok = execution.greedy(hidden)
    out = [int(tok)]
    if out[0] == eos_token_id or max_new_tokens == 1:
        return out
    if persistent and not getattr(execution, '_exact_projections', False):
        # one persistent launch for the rest; EOS stops are applied afterwards (the kernel
        # runs a fixed number of tokens)
        rest = execution.decode_persistent(tok.clone(), max_new_tokens - 1)[:, 0].tolist()
        for t in rest:
            out.append(int(t))
            if t == eos_token_id:
                break
        return out
    for _ in range(max_new_tokens - 1):
        tok = execution.greedy(execution.backbone(tok[:, None].contiguous())[:, 0])
        out.append(int(tok))
        if out[-1] == eos_token_id:
            break
    return out


def classify_prediction(row):
    """scripts/run_state_resurface_v11.py:162-169."""
    prediction = row['prediction']
    if prediction == row['answer']:
        return 'correct_target' if row['condition'] == 'normal' else 'removed_target_match'
    if prediction is None:
        return 'unparseable'
    if int(prediction) in {value for _, value in row['records']}:
        return 'wrong_present_value' if row['condition'] == 'normal' else 'other_present_value'
    return 'not_present_value'


def _summary_rows(rows):
    correct = sum(r['correct'] for r in rows)
    categories = {}
    for r in rows:
        k = classify_prediction(r)
        categories[k] = categories.get(k, 0) + 1
    return dict(count=len(rows), correct=correct, accuracy=correct / len(rows) if rows else None,
                prediction_categories=dict(sorted(categories.items())))


@torch.no_grad()
def evaluate_mk(execution, tokenizer, split='test', samples_per_cell=8, cases=None, max_new_tokens=12,
                persistent=True):
    """Greedy recall over the MK cases; returns the reference's result dict."""
    cases = synthetic_mk_cases(split, samples_per_cell) if cases is None else cases
    eos = getattr(tokenizer, 'eos_token_id', None)
    rows = []
    started = time.time()
    for case in cases:
        ids = tokenizer.encode(case['prompt'])
        generated = generate_greedy(execution, ids, max_new_tokens, eos, persistent=persistent)
        output = tokenizer.decode(generated)
        match = SIX_DIGITS.search(output)
        prediction = match.group() if match else None
        row = {**{k: v for k, v in case.items() if k != 'prompt'}, 'prompt_tokens': len(ids),
               'prompt_token_sha256_int64le': token_digest(np.asarray(ids, dtype=np.int64)),
               'prompt': case['prompt'], 'output': output, 'generated_ids': generated,
               'prediction': prediction, 'correct': prediction == case['answer']}
        row['prediction_category'] = classify_prediction(row)
        rows.append(row)
    summary = {c: _summary_rows([r for r in rows if r['condition'] == c]) for c in ('normal', 'target_removed')}
    sizes = sorted({r['N'] for r in rows})
    cells = []
    for size in sizes:
        for template in range(3):
            for condition in ('normal', 'target_removed'):
                sel = [r for r in rows if r['N'] == size and r['template'] == template and r['condition'] == condition]
                cells.append(dict(N=size, template=template, condition=condition,
                                  correct=sum(r['correct'] for r in sel), count=len(sel),
                                  query_positions=[r['query_position'] for r in sel],
                                  paired_case_ids=[r['id'] for r in sel]))
    normal = [r for r in rows if r['condition'] == 'normal']
    strata = {}
    for label, key in (('normal_by_N', lambda r: str(r['N'])), ('normal_by_template', lambda r: str(r['template'])),
                       ('normal_by_N_template', lambda r: f"N{r['N']}_t{r['template']}"),
                       ('normal_by_N_position_quartile', lambda r: f"N{r['N']}_q{4 * r['query_position'] // r['N']}")):
        groups = {}
        for r in normal:
            groups.setdefault(key(r), []).append(r)
        strata[label] = {name: _summary_rows(g) for name, g in sorted(groups.items())}
    return dict(protocol=PROTOCOL, split=split, generation=f'greedy, at most {max_new_tokens} tokens, stop at EOS',
                matching='first standalone six-digit integer equals answer', summary=summary, cells=cells,
                strata=strata, rows=rows, elapsed_seconds=time.time() - started)
