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
def score_local(execution, windows, batch_windows=16):
    """Score windows on this device; returns per-window records in input order."""
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
            toks = torch.stack([torch.as_tensor(windows[i][1], dtype=torch.long) for i in chunk]).to(dev)
            hidden = execution.backbone(toks[:, :-1].contiguous(), reset=True)
            nll = execution.score(hidden, toks[:, 1:].contiguous())
            sums = nll.view(len(chunk), length - 1).double().sum(1).cpu().tolist()
            for i, s in zip(chunk, sums):
                if not math.isfinite(s):
                    raise FloatingPointError('Nonfinite PPL NLL')
                start, w = windows[i]
                records[i] = dict(start=int(start), target_tokens=length - 1,
                                  token_sha256_int64le=token_digest(np.asarray(w)), nll=s,
                                  ppl=math.exp(s / (length - 1)))
    return records


@torch.no_grad()
def evaluate_ppl(execution, windows, batch_windows=16, rank=0, world=1, group=None):
    """Pooled perplexity over `windows`; sharded over `world` ranks when world > 1."""
    local = list(range(rank, len(windows), world))
    recs = score_local(execution, [windows[i] for i in local], batch_windows) if local else []
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
    return dict(ppl=math.exp(total / count), nll=total, target_tokens=count, windows=recs)


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
