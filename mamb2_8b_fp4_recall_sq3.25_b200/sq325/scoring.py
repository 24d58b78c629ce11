"""Teacher-forced window scoring and greedy generation over a PredictorState.

  ppl_windows      mamba2_recall/evaluation.py:27-33 (2048 targets + 1 overlap token,
                   stride 2048, final partial window kept)
  evaluate_ppl     scripts/run_fp4_ridge_resurface_v3.py:81-121: every window starts from a
                   reset state; NLL = sum of next-token cross entropies of fp16 logits;
                   pooled PPL = exp(sum NLL / sum targets).  Windows of equal length are
                   batched (B windows per forward).  With world > 1 the windows are sharded
                   round-robin over ranks and ONE all-reduce of [sum NLL, sum targets]
                   (fp64) combines them; per-window records are gathered on rank 0.
  generate         scripts/infer_fp4_ridge_resurface_v1.py:100-110 (prefill, then greedy
                   argmax tokens fed back one at a time).
"""
from __future__ import annotations

import hashlib
import json
import math

import numpy as np
import torch


def token_digest(ids):
    return hashlib.sha256(np.asarray(ids, dtype='<i8').tobytes()).hexdigest()


def ppl_windows(ids, seqlen, nwin=None):
    if nwin is not None:
        usable = len(ids)
        if seqlen + 1 <= 0 or nwin <= 0 or usable < (seqlen + 1) * nwin:
            raise ValueError('Insufficient tokens for the requested nonoverlapping windows')
        span = usable - (seqlen + 1)
        starts = [0] if nwin == 1 else [(i * span) // (nwin - 1) for i in range(nwin)]
        return [(s, ids[s:s + seqlen + 1]) for s in starts]
    return [(s, ids[s:min(s + seqlen + 1, len(ids))]) for s in range(0, len(ids) - 1, seqlen)]


@torch.no_grad()
def score_local(execution, windows, batch_windows=16, on_batch=None):
    """Score windows on this device; returns per-window records in input order.
    `on_batch(records)` is called after every batch (records of unscored windows are None)."""
    dev = execution.device
    records = [None] * len(windows)
    by_len = {}
    for i, (start, w) in enumerate(windows):
        by_len.setdefault(len(w), []).append(i)
    for length, idxs in sorted(by_len.items()):
        if length < 2:
            raise ValueError('A window needs at least one target token')
        for c in range(0, len(idxs), batch_windows):
            chunk = idxs[c:c + batch_windows]
            toks = torch.stack([torch.as_tensor(windows[i][1], dtype=torch.long) for i in chunk])
            host = toks if toks.device.type == 'cpu' else None
            toks = toks.to(dev)
            hidden = execution.backbone(toks[:, :-1].contiguous(), reset=True)
            nll = execution.score(hidden, toks[:, 1:].contiguous())
            sums = nll.view(len(chunk), length - 1).double().sum(1).cpu().tolist()
            if host is None:                          # windows resident on the device
                host = toks.cpu()
            for k, (i, s) in enumerate(zip(chunk, sums)):
                if not math.isfinite(s):
                    raise FloatingPointError('Nonfinite PPL NLL')
                records[i] = dict(start=int(windows[i][0]), target_tokens=length - 1,
                                  token_sha256_int64le=token_digest(host[k].numpy()), nll=s,
                                  ppl=math.exp(s / (length - 1)))
            if on_batch is not None:
                on_batch(records)
    return records


def cache_identity(execution):
    """sha256 of every cache tensor, keyed '<layer>.<name>' (the six PackedState tensors and
    'conv' in the reference's chronological [batch, 10240, 4] order), as the reference's
    evaluation scripts record it (scripts/run_fp4_latent_state_quality_v1.py:49-61)."""
    from .resurface import tensor_hash
    out = {}
    for index, entry in enumerate(execution._cache):
        for key, value in entry.state.tensors.items():
            out[f'{index}.{key}'] = tensor_hash(value)
        out[f'{index}.conv'] = tensor_hash(execution.conv_chronological(index))
    return out


def _put(path, row):
    """Write the report row atomically (the reference rewrites its JSON after every window)."""
    from pathlib import Path
    path = Path(path)
    tmp = path.with_suffix(path.suffix + '.tmp')
    tmp.write_text(json.dumps(row, indent=1, allow_nan=False) + '\n')
    tmp.replace(path)


@torch.no_grad()
def repeated_reset_probe(execution, window, tokens=128):
    """scripts/run_fp4_ridge_resurface_v3.py:90-98: the first `tokens` of a window scored twice
    from a reset state must give identical hidden states and identical cache bytes."""
    from .resurface import tensor_hash
    probe = torch.as_tensor(window[:tokens], dtype=torch.long).to(execution.device)[None]
    first = execution.backbone(probe, reset=True).clone()
    identity = cache_identity(execution)
    second = execution.backbone(probe, reset=True)
    if not (torch.equal(first, second) and identity == cache_identity(execution) and
            bool(torch.isfinite(first).all())):
        raise RuntimeError('Repeated reset differs')
    return dict(tokens=int(probe.shape[1]), hidden_sha256=tensor_hash(first), hidden_and_cache_exact=True,
                cache_tensor_sha256=identity, token_sha256_int64le=token_digest(probe.cpu().numpy()),
                cache=execution.cache_breakdown())


@torch.no_grad()
def evaluate_ppl(execution, windows, batch_windows=16, rank=0, world=1, group=None, *, path=None, common=None,
                 frozen=None, probe_tokens=128):
    """Pooled perplexity over `windows` (a list of (start, int64 tokens)); sharded over
    `world` ranks when world > 1: rank r scores windows r, r + world, ... and ONE all-reduce of
    [sum NLL, sum targets] (fp64) combines them; the per-window records are gathered so every
    rank returns the full list in window order.

    With `path`, rank 0 keeps the reference's report (run_fp4_ridge_resurface_v3.py:81-121):
    a JSON row {**common, complete, ppl: {windows, nll, target_tokens, ppl}, static basis /
    scale / predictor sha256, layer_layouts, repeated_reset_probe, cache, storage_descriptor}
    rewritten after every batch of windows, and the repeated-reset probe on the first
    `probe_tokens` of window 0 before scoring.  `frozen`, if given, is an object whose
    check() result is recorded at the end (the reference's frozen-source check)."""
    from .resurface import tensor_hash
    local = list(range(rank, len(windows), world))
    report = path is not None and rank == 0
    row = None
    if report:
        row = dict(common or {}, complete=False, ppl=dict(windows=[]),
                   static_basis_sha256=[tensor_hash(x) for x in execution.bases],
                   static_scale_sha256=[tensor_hash(x) for x in execution.latent_scales],
                   static_predictor_sha256=[[tensor_hash(x) for x in p] for p in execution.predictors],
                   layer_layouts=list(execution.layouts))
        _put(path, row)
        row['repeated_reset_probe'] = repeated_reset_probe(execution, windows[0][1], probe_tokens)
        row['storage_descriptor_probe'] = execution.storage_descriptor()

    def progress(recs):
        if report:
            row['ppl']['windows'] = [r for r in recs if r is not None]
            done = row['ppl']['windows']
            nll = sum(r['nll'] for r in done)
            count = sum(r['target_tokens'] for r in done)
            row['ppl'].update(nll=nll, target_tokens=count, ppl=math.exp(nll / count))
            row['cache'], row['storage_descriptor'] = execution.cache_breakdown(), execution.storage_descriptor()
            _put(path, row)

    recs = score_local(execution, [windows[i] for i in local], batch_windows, on_batch=progress) if local else []
    total = sum(r['nll'] for r in recs)
    count = sum(r['target_tokens'] for r in recs)
    if world > 1:
        import torch.distributed as dist
        backend = dist.get_backend(group)
        dev = execution.device if backend == 'nccl' else 'cpu'
        buf = torch.tensor([total, float(count)], dtype=torch.float64, device=dev)
        dist.all_reduce(buf, group=group)
        total, count = float(buf[0]), int(round(float(buf[1])))
        gathered = [None] * world
        dist.all_gather_object(gathered, [(i, r) for i, r in zip(local, recs)], group=group)
        merged = sorted((x for part in gathered for x in part), key=lambda t: t[0])
        recs = [r for _, r in merged]
    result = dict(ppl=math.exp(total / count), nll=total, target_tokens=count, windows=recs)
    if report:
        row['ppl'] = dict(windows=recs, nll=total, target_tokens=count, ppl=result['ppl'])
        row.update(complete=True, ppl_complete=True)
        if frozen is not None:
            row['frozen_source'] = frozen.check()
        _put(path, row)
    return result


@torch.no_grad()
def generate(execution, prompt_ids, max_new_tokens, eos_token_id=None, graphs=False, persistent=True):
    """Greedy decode: returns int64 [batch, n_generated] (n <= max_new_tokens).

    graphs=True runs the token loop without host synchronisation (an EOS stop is then
    applied after the fact by truncation): at batch 1 with the factored-scale projections
    one persistent kernel launch per token (persistent=True), otherwise a captured CUDA
    graph per token."""
    dev = execution.device
    prompt = torch.as_tensor(prompt_ids, dtype=torch.long).to(dev)
    if prompt.ndim == 1:
        prompt = prompt[None]
    hidden = execution.backbone(prompt.contiguous(), reset=True)[:, -1]
    if graphs:
        tok = execution.greedy(hidden).clone()
        first = tok.clone()
        use_kernel = (persistent and prompt.shape[0] == 1 and max_new_tokens > 1 and
                      not getattr(execution, '_exact_projections', False))
        rest = None
        if use_kernel:
            rest = execution.decode_persistent(tok, max_new_tokens - 1)
        elif max_new_tokens > 1:
            execution.capture_decode(tok)
            rest = execution.replay_decode(max_new_tokens - 1)
        seq = first[:, None] if rest is None else torch.cat([first[:, None], rest.T], 1)
        if eos_token_id is not None:
            hit = (seq == eos_token_id).all(0).nonzero()
            if hit.numel():
                seq = seq[:, :int(hit[0]) + 1]
        return seq
    out = []
    for step in range(max_new_tokens):
        tok = execution.greedy(hidden)
        out.append(tok)
        if step + 1 == max_new_tokens:
            break
        if eos_token_id is not None and bool((tok == eos_token_id).all()):
            break
        hidden = execution.backbone(tok[:, None].contiguous())[:, 0]
    return torch.stack(out, 1)
