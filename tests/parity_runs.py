"""Long-horizon parity runs of the GPU path against the CPU oracle (GPU, test infrastructure).

  config1_run   BASELINE config 1: one Mamba-2 layer's SQ3.25 carry ([1, 128 heads, 64, 128]),
                2,048 sequential one-token scan calls (each decodes, updates, requantises and
                repacks the carry), seed 0.  Per step: INT8 / INT4 code agreement between the
                GPU (sq_scan) and the oracle (oracle.cscan, bit-exact with the reference
                kernel), max-abs / relative error of the decoded carry and of the readout
                against the oracle and against the fp32 unquantised recurrence; teacher-forced
                (every step starts from the oracle's carry) and free-running.
  model_run     a full-depth forward (56 layers, the released per-layer layouts) of a short
                window plus decode steps, GPU against oracle.model: per layer, teacher-forced
                (the GPU mixer, sq_model_mixer_forward, gets the oracle's input of that layer)
                the mixer output error, state code agreement and conv ring; free-running
                (sq_model_forward) the per-layer drift, final hidden state, logits and NLL.

The -m gpu tests (test_gpu_parity_long.py) run these and assert the bars; running this file
directly writes the full per-step / per-layer report:

    python tests/parity_runs.py --out gpurun_out/parity   [--steps 2048] [--layers 56]
"""
from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[1]
for p in (str(ROOT), str(ROOT / 'mamb2_8b_fp4_recall_sq3.25_b200')):
    if p not in sys.path:
        sys.path.insert(0, p)

from oracle import codec as oc  # noqa: E402
from oracle import cscan  # noqa: E402

H, P, G = 128, 64, 8


def _rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@torch.no_grad()
def config1_run(layout, steps=2048, seed=0, teacher_forced=False):
    """Returns per-step arrays and a summary dict (see the module docstring).

    Free-running (default): GPU and oracle each carry their own state for all steps, so a
    code that flips at a rounding boundary (CUDA expf / logf and FMA contraction against
    numpy's unfused fp32) persists through the decay (up to 0.99 per step here) and the two
    carries drift apart.  teacher_forced=True copies the oracle's carry into the GPU state
    before every step: each step then measures one call's own arithmetic."""
    from sq325 import codec
    n8, n4, nz = oc.layout_counts(layout)
    NS = n8 + n4
    rng = np.random.default_rng(seed)
    # statics: seeded permutation per group, basis N(0,1), latent scales U[0.1,1.1],
    # predictor N(0,1)/sqrt(group features)
    perm = np.stack([rng.permutation(128) for _ in range(G)]).astype(np.uint8)
    basis = rng.standard_normal((G, nz, 2)).astype(np.float16)
    ls = rng.uniform(0.1, 1.1, (G, 2)).astype(np.float16)
    pred = (rng.standard_normal((G, NS + 2, nz)) / np.sqrt(NS + 2)).astype(np.float16)
    # per-head decay exp(-U[0.01, 0.5]) at dt ~= 1: A = log(decay), dt_raw = log(e - 1), no bias
    decay_h = np.exp(-rng.uniform(0.01, 0.5, H))
    A = np.log(decay_h).astype(np.float32)
    D = rng.standard_normal(H).astype(np.float16)
    dtb = np.zeros(H, np.float16)
    dt_raw = np.full((1, 1, H), np.log(np.e - 1.0), np.float16)
    # initial carry: N(0, sigma_h^2), sigma_h log-uniform in [1e-3, 1], coordinates already in
    # tier order; stored with the reference's diagnostic encode_state_ rule, latent z = 0
    sigma = np.exp(rng.uniform(np.log(1e-3), 0.0, H)).astype(np.float32)
    dense = (rng.standard_normal((1, H, P, 128)) * sigma[None, :, None, None]).astype(np.float32)
    st_o = oc.encode_diagnostic(dense[..., :NS], layout)
    st_o = {k: np.ascontiguousarray(v) for k, v in st_o.items()}
    st_g = codec.allocate_state(1, H, P, 128, 'cuda', layout=layout)
    for k, v in st_o.items():
        t = torch.from_numpy(v.copy()).cuda()
        st_g.tensors[k].copy_(t.view(torch.float8_e4m3fn) if k == 'latent' else t)
    T = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    gperm, gbasis, gls, gpred, gA, gD, gdtb, gdt = (T(a) for a in (perm, basis, ls, pred, A, D, dtb, dt_raw))
    # fp32 unquantised recurrence in tier order (the zero tier carries state here too)
    gidx = np.arange(H) // (H // G)
    s_full = np.ascontiguousarray(dense[0])                                             # [H,P,128] fp32
    dtv, dec = cscan.per_token_scalars(dt_raw, A, dtb)
    dtv, dec = dtv[0, 0], dec[0, 0]                                                     # [H] fp32
    Df = D.astype(np.float32)
    rows = dict(agree8=[], agree4=[], maxcode=[], within1=[], carry_abs_oracle=[], carry_rel_oracle=[],
                carry_rel_fp32=[], y_abs_oracle=[], y_rel_oracle=[], y_rel_fp32=[], y_bits_oracle=[])

    def rel32(a, b):
        a = np.asarray(a, np.float32).ravel()
        b = np.asarray(b, np.float32).ravel()
        d = a - b
        return float(np.sqrt(np.dot(d, d)) / max(np.sqrt(np.dot(b, b)), 1e-30))

    for step in range(steps):
        if teacher_forced:
            for k, v in st_o.items():
                t = torch.from_numpy(v.copy()).cuda()
                st_g.tensors[k].copy_(t.view(torch.float8_e4m3fn) if k == 'latent' else t)
        x = rng.standard_normal((1, 1, H, P)).astype(np.float16)
        Bm = rng.standard_normal((1, 1, G, 128)).astype(np.float16)
        Cm = rng.standard_normal((1, 1, G, 128)).astype(np.float16)
        y_g, _ = codec.scan(T(x), gdt, gA, T(Bm), T(Cm), gD, gdtb, st_g, gperm, gbasis, gls, gpred, layout=layout)
        y_o = cscan.latent_scan(x, dt_raw, A, Bm, Cm, D, dtb, st_o, perm, basis, ls, pred, layout)
        # unquantised fp32 recurrence, coordinates in tier order per group
        b_tier = np.take_along_axis(Bm[0, 0].astype(np.float32), perm.astype(np.int64), 1)     # [G,128]
        c_tier = np.take_along_axis(Cm[0, 0].astype(np.float32), perm.astype(np.int64), 1)
        xv = x[0, 0].astype(np.float32)                                                         # [H,P]
        s_full *= dec[:, None, None]
        s_full += (b_tier[gidx] * dtv[:, None])[:, None, :] * xv[:, :, None]
        y_f = np.einsum('hpn,hn->hp', s_full, c_tier[gidx]) + xv * Df[:, None]
        sg = {k: (v.view(torch.uint8) if v.dtype == torch.float8_e4m3fn else v).cpu().numpy()
              for k, v in st_g.tensors.items()}
        q8, q4 = oc.decode_codes(sg, layout)
        r8, r4 = oc.decode_codes(st_o, layout)
        tg, _ = oc.decode_state(sg, layout, ls, H // G)
        to, _ = oc.decode_state(st_o, layout, ls, H // G)
        yg = y_g.cpu().numpy()
        d8, d4 = np.abs(q8 - r8), np.abs(q4 - r4)
        rows['agree8'].append(float((d8 == 0).mean()))
        rows['agree4'].append(float((d4 == 0).mean()))
        rows['maxcode'].append(int(max(d8.max(), d4.max())))
        rows['within1'].append(float(((d8 <= 1).sum() + (d4 <= 1).sum()) / (d8.size + d4.size)))
        rows['carry_abs_oracle'].append(float(np.abs(tg - to).max()))
        rows['carry_rel_oracle'].append(rel32(tg, to))
        rows['carry_rel_fp32'].append(rel32(tg[0], s_full[..., :NS]))
        rows['y_abs_oracle'].append(float(np.abs(yg.astype(np.float32) - y_o.astype(np.float32)).max()))
        rows['y_rel_oracle'].append(rel32(yg, y_o))
        rows['y_rel_fp32'].append(rel32(yg[0, 0], y_f))
        rows['y_bits_oracle'].append(float((yg.view(np.uint16) == y_o.view(np.uint16)).mean()))
    summary = dict(layout=layout, steps=steps, mode='teacher-forced' if teacher_forced else 'free-running',
                   codes_within_one_step_min=min(rows['within1']),
                   code_agreement_min=min(min(rows['agree8']), min(rows['agree4'])),
                   code_agreement_mean=float(np.mean(rows['agree8'] + rows['agree4'])),
                   max_code_step=max(rows['maxcode']),
                   carry_max_abs_vs_oracle=max(rows['carry_abs_oracle']),
                   carry_rel_vs_oracle_max=max(rows['carry_rel_oracle']),
                   carry_rel_vs_fp32_final=rows['carry_rel_fp32'][-1],
                   carry_rel_vs_fp32_max=max(rows['carry_rel_fp32']),
                   y_max_abs_vs_oracle=max(rows['y_abs_oracle']),
                   y_rel_vs_oracle_max=max(rows['y_rel_oracle']),
                   y_bits_identical_mean=float(np.mean(rows['y_bits_oracle'])),
                   y_rel_vs_fp32_mean=float(np.mean(rows['y_rel_fp32'])))
    return rows, summary


@torch.no_grad()
def model_run(n_layer=56, vocab=2048, tokens=16, decode_steps=4, seed=7):
    """Full-depth GPU forward against oracle.model (released layouts); per-layer figures."""
    from oracle.pair import build_pair
    from sq325 import PredictorState
    from sq325.model import RELEASED_LAYOUTS, benchmark_layouts
    layouts = RELEASED_LAYOUTS if n_layer == 56 else benchmark_layouts(n_layer)
    gm, ora, statics = build_pair(n_layer=n_layer, vocab=vocab, layouts=layouts, seed=seed, adapter=True)
    rng = np.random.default_rng(seed)
    ids = rng.integers(0, vocab, (1, tokens + decode_steps + 1)).astype(np.int64)
    prompt = ids[:, :tokens]
    layers = []
    with PredictorState(gm, *statics) as ex:
        cap = ex.capture_layers(tokens)
        hid = ex.backbone(torch.from_numpy(prompt).cuda(), reset=True)
        nll = ex.score(hid, torch.from_numpy(ids[:, 1:tokens + 1]).cuda())
        torch.cuda.synchronize()
        ex.check()
        gcap = cap.float().cpu().numpy()
        ora.reset(1)
        ora.capture = []
        ora.capture_inputs = []
        href = ora.backbone(prompt)
        nref = ora.nll(href, ids[:, 1:tokens + 1])
        # scoring head on the oracle's own final hidden state (teacher-forced head)
        nll_tf = float(ex.score(href.cuda(), torch.from_numpy(ids[:, 1:tokens + 1]).cuda()).double().sum())
        for l in range(n_layer):
            got, ref = gcap[l, :tokens], ora.capture[l].reshape(tokens, -1).float().numpy()
            layers.append(dict(layer=l, layout=layouts[l], mixer_rel_l2=_rel(got, ref),
                               mixer_max_abs=float(np.abs(got - ref).max()),
                               mixer_ref_max=float(np.abs(ref).max())))
        hid_rel = _rel(hid.float().cpu().numpy(), href.float().numpy())
        nll_g = float(nll.double().sum())
        nll_o = float(nref.sum())
        # prefill end state: code agreement per layer
        for l, e in enumerate(ex._cache):
            sg = {k: (v.view(torch.uint8) if v.dtype == torch.float8_e4m3fn else v).cpu().numpy()
                  for k, v in e.state.tensors.items()}
            q8, q4 = oc.decode_codes(sg, layouts[l])
            r8, r4 = oc.decode_codes(ora.caches[l]['state'], layouts[l])
            layers[l]['prefill_code_agreement'] = float(np.concatenate([(q8 == r8).ravel(), (q4 == r4).ravel()]).mean())
        ex.capture_layers(0)
        # teacher-forced per layer: every GPU layer gets the oracle's normed input for that
        # layer (fresh states), so its error is its own, not the upstream layers'
        ex.reset(1)
        for l in range(n_layer):
            u = ora.capture_inputs[l].cuda()
            got = ex.mixer_forward(l, u).float().cpu().numpy().reshape(tokens, -1)
            ref = ora.capture[l].reshape(tokens, -1).float().numpy()
            sg = {k: (v.view(torch.uint8) if v.dtype == torch.float8_e4m3fn else v).cpu().numpy()
                  for k, v in ex._cache[l].state.tensors.items()}
            q8, q4 = oc.decode_codes(sg, layouts[l])
            r8, r4 = oc.decode_codes(ora.caches[l]['state'], layouts[l])
            diff = np.concatenate([np.abs(q8 - r8).ravel(), np.abs(q4 - r4).ravel()])
            layers[l].update(tf_mixer_rel_l2=_rel(got, ref), tf_code_agreement=float((diff == 0).mean()),
                             tf_max_code_step=int(diff.max()), tf_codes_within_one=float((diff <= 1).mean()),
                             tf_conv_ring_rel=_rel(ex.conv_chronological(l).float().cpu().numpy(),
                                                   ora.caches[l]['conv'].float().numpy()))
        tf_step = []
        for s_ in range(decode_steps):
            nxt = ids[:, tokens + s_:tokens + s_ + 1]
            ora.capture, ora.capture_inputs = [], []
            ora.backbone(nxt)
            worst = 0.0
            for l in range(n_layer):
                got = ex.mixer_forward(l, ora.capture_inputs[l].cuda()).float().cpu().numpy()
                worst = max(worst, _rel(got.reshape(-1), ora.capture[l].float().numpy().reshape(-1)))
            tf_step.append(worst)
        ora.capture = ora.capture_inputs = None
        # free-running decode steps from the free-running prefill
        ex.backbone(torch.from_numpy(prompt).cuda(), reset=True)
        ora.reset(1)
        ora.backbone(prompt)
        step_rel = []
        for s in range(decode_steps):
            nxt = ids[:, tokens + s:tokens + s + 1]
            h = ex.backbone(torch.from_numpy(nxt).cuda())
            hr = ora.backbone(nxt)
            step_rel.append(_rel(h.float().cpu().numpy(), hr.float().numpy()))
        logits = torch.empty(1, vocab, device='cuda', dtype=torch.float16)
        ex.greedy(h[:, -1], logits=logits)
        torch.cuda.synchronize()
        lref = ora.logits(h[:, -1].cpu())
        logits_rel = _rel(logits.float().cpu().numpy(), lref.float().numpy())
    summary = dict(n_layer=n_layer, vocab=vocab, tokens=tokens, decode_steps=decode_steps,
                   tf_mixer_rel_l2_max=max(x['tf_mixer_rel_l2'] for x in layers),
                   tf_code_agreement_min=min(x['tf_code_agreement'] for x in layers),
                   tf_max_code_step=max(x['tf_max_code_step'] for x in layers),
                   tf_codes_within_one_min=min(x['tf_codes_within_one'] for x in layers),
                   tf_conv_ring_rel_max=max(x['tf_conv_ring_rel'] for x in layers),
                   tf_decode_mixer_rel_l2_max=max(tf_step),
                   tf_head_nll_rel=abs(nll_tf - nll_o) / abs(nll_o),
                   hidden_rel_l2=hid_rel, window_nll_gpu=nll_g, window_nll_oracle=nll_o,
                   window_nll_rel=abs(nll_g - nll_o) / abs(nll_o), decode_hidden_rel_l2=step_rel,
                   decode_logits_rel_l2=logits_rel,
                   mixer_rel_l2_max=max(x['mixer_rel_l2'] for x in layers),
                   prefill_code_agreement_min=min(x['prefill_code_agreement'] for x in layers))
    return layers, summary


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument('--out', type=Path, required=True)
    ap.add_argument('--steps', type=int, default=2048)
    ap.add_argument('--layers', type=int, default=56)
    ap.add_argument('--skip-model', action='store_true')
    args = ap.parse_args()
    args.out.mkdir(parents=True, exist_ok=True)
    report = dict(config1=[], model=None)
    for tf in (True, False):
        for layout in oc.LAYOUTS:
            rows, summary = config1_run(layout, steps=args.steps, teacher_forced=tf)
            report['config1'].append(summary)
            np.savez_compressed(args.out / f"config1_{'tf' if tf else 'free'}_{layout}.npz",
                                **{k: np.asarray(v) for k, v in rows.items()})
            print(json.dumps(summary), flush=True)
    if not args.skip_model:
        layers, summary = model_run(n_layer=args.layers)
        report['model'] = dict(summary=summary, layers=layers)
        print(json.dumps(summary), flush=True)
    (args.out / 'parity_report.json').write_text(json.dumps(report, indent=1))


if __name__ == '__main__':
    main()
