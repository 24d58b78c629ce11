#!/usr/bin/env python3
"""Regenerate the golden vectors in this directory from the reference's own code.

Runs ONLY in the build container, where the reference tree is mounted (path
given by the required --reference argument). The GPU box never runs it;
tests read the committed .npz files.

What is recorded
  codec_<layout>.npz   the production latent codec kernel `_latent_scan`
                       (scripts/fp4_zero_predictor_codec_v1.py:76-181) executed
                       by the Triton CPU interpreter, with the host correction of
                       :221-225, on seeded inputs: one multi-token call from
                       random packed bytes, and one known-answer call (A=0,
                       x=0 => decay 1, no update: decode -> requant -> pack).
  fp4_g16.npz          mamba2_recall/fp4.py quantize_chunk + decode_packet on a
                       seeded matrix (codes, E4M3 block bytes, global, FP16).
  adapter.npz          mamba2_recall/resurface_native._Adapter.forward (soft
                       gate, FP16 parameters) on CPU.
  mk_cases.json        sha256 of the reference's public MK recall prompts
                       (mamba2_recall/evaluation.py:82-119, both splits).
  s16.npz              the FP16-state control scan `_s16_scan`
                       (mamba2_recall/state_codec.py:65-102) under the interpreter,
                       without and with the calibration statistics (:256-262).
  ste.npz              the legacy sq3p25 scan `_sq_scan` (mamba2_recall/state_codec.py:105-176)
                       from a random packed state and from the zero state, and the
                       straight-through training backward of
                       mamba2_recall/state_training_scan.py (_carry_checkpoints,
                       _chunk_history, _chunk_backward, :24-179) over 3 chunks, all
                       under the interpreter.
  checkpoint_plan.json the packed-checkpoint container rules of
                       mamba2_recall/fp4_checkpoint.py run on this model's tensor
                       inventory: `make_plan` (:67-93) at two shard limits for the
                       production 56-layer / 256,000-row model (sha256 of the
                       canonical JSON) and for a 2-layer / 64-row model at 1 MiB
                       (in full), `_file_specs` (:100-114) and every shard's
                       `_header` bytes (:117-127; sha256 for production, hex in
                       full for the small model).

Interpreter shims (the interpreter cannot run two device intrinsics as the
GPU does):
  * libdevice.round -> C round() semantics (nearest, ties away from zero).
  * fp32 <-> float8e4nv casts -> torch's float8_e4m3fn cast (round to nearest
    even), matching the GPU's cvt.rn.satfinite on the kernel's +-448 clamp.
"""
from __future__ import annotations

import argparse
import os
import sys
from pathlib import Path

os.environ['TRITON_INTERPRET'] = '1'
HERE = Path(__file__).resolve().parent

import numpy as np  # noqa: E402
import torch  # noqa: E402
import triton  # noqa: E402
import triton.language as tl  # noqa: E402


@triton.jit
def _round_half_away(x):
    a = tl.abs(x)
    r = tl.floor(a)
    r = tl.where(a - r >= 0.5, r + 1.0, r)
    return tl.where(x < 0, -r, r)


def install_shims(reference):
    sys.path.insert(0, str(reference / 'scripts'))
    sys.path.insert(0, str(reference))
    from triton.runtime import interpreter as interp
    import state_ppl_codec_v6 as v6

    class _Libdevice:
        round = _round_half_away

    v6.libdevice = _Libdevice
    original = interp._convert_float

    def convert(data, src, dst, rounding_mode):
        names = (str(src), str(dst))
        if names == ('fp32', 'fp8e4nv'):
            t = torch.from_numpy(np.ascontiguousarray(data).view(np.float32).copy())
            return t.to(torch.float8_e4m3fn).view(torch.uint8).numpy()
        if names == ('fp8e4nv', 'fp32'):
            t = torch.from_numpy(np.ascontiguousarray(data).view(np.uint8).copy())
            return t.view(torch.float8_e4m3fn).float().numpy().view(np.uint32)
        return original(data, src, dst, rounding_mode)

    interp._convert_float = convert
    import fp4_zero_predictor_codec_v1 as ref
    return ref


def random_state(gen, batch, heads, dim, spec):
    w = spec['tensor_widths']
    t = {}
    for k in ('lo', 'hi', 'q4'):
        t[k] = torch.randint(0, 256, (batch, heads, dim, w[k]), generator=gen, dtype=torch.uint8)
    lat = torch.randint(0, 256, (batch, heads, dim, 2), generator=gen, dtype=torch.uint8)
    lat = torch.where((lat & 0x7F) == 0x7F, lat ^ 0x01, lat)          # no NaN bytes
    t['latent'] = lat.view(torch.float8_e4m3fn)
    for k, lim in (('s8', 1e-2), ('s4', 1e-1)):
        t[k] = (torch.rand(batch, heads, dim, generator=gen) * lim + 1e-5).half()
    return t


def codec_case(ref, layout, seed, batch=2, length=4, heads=4, dim=32, groups=2, known_answer=False):
    spec = ref.layout_descriptor(layout)
    n8, n4, nz = spec['n8'], spec['n4'], spec['nzero']
    gen = torch.Generator().manual_seed(seed)
    x = torch.randn(batch, length, heads, dim, generator=gen).half()
    dt = (torch.randn(batch, length, heads, generator=gen) * 0.7).half()
    A = -(torch.rand(heads, generator=gen) * 3 + 0.05).float()
    Bm = torch.randn(batch, length, groups, 128, generator=gen).half()
    Cm = torch.randn(batch, length, groups, 128, generator=gen).half()
    D = torch.randn(heads, generator=gen).half()
    dt_bias = (torch.rand(heads, generator=gen) * 3 - 4).half()
    perm = torch.stack([torch.randperm(128, generator=gen) for _ in range(groups)]).to(torch.uint8)
    basis = torch.randn(groups, nz, 2, generator=gen).half()
    ls = (torch.rand(groups, 2, generator=gen) + 0.1).half()
    pred = (torch.randn(groups, n8 + n4 + 2, nz, generator=gen) / np.sqrt(n8 + n4 + 2)).half()
    if known_answer:
        length = 1
        x = torch.zeros(batch, 1, heads, dim).half()
        dt, Bm, Cm = dt[:, :1].contiguous(), Bm[:, :1].contiguous(), Cm[:, :1].contiguous()
        A = torch.zeros(heads).float()
    state = random_state(gen, batch, heads, dim, spec)
    initial = {k: v.clone() for k, v in state.items()}
    dead = perm[:, n8 + n4:].long()
    dead_c = Cm.float().gather(3, dead[None, None].expand(batch, length, -1, -1))
    corr = torch.einsum('blgd,gfd->blgf', dead_c, pred.float()).contiguous()
    out = torch.empty_like(x)
    ref._latent_scan[(batch, heads, triton.cdiv(dim, 16))](
        x, dt, A, Bm, Cm, corr, D, dt_bias, perm,
        *(state[k] for k in ('lo', 'hi', 'q4', 'latent', 's8', 's4')),
        basis, ls, out, length, heads, dim, groups, n8, n4, nz,
        triton.next_power_of_2(n8), triton.next_power_of_2(n4), triton.next_power_of_2(nz), 16,
        num_warps=4)

    def np_(t):
        if t.dtype == torch.float8_e4m3fn:
            return t.view(torch.uint8).numpy()
        return t.numpy()
    rec = dict(x=x, dt=dt, A=A, B=Bm, C=Cm, D=D, dt_bias=dt_bias, permutation=perm, basis=basis,
               latent_scale=ls, predictor=pred, corr=corr, y=out)
    rec = {k: np_(v) for k, v in rec.items()}
    rec.update({'in_' + k: np_(v) for k, v in initial.items()})
    rec.update({'out_' + k: np_(v) for k, v in state.items()})
    return rec


def s16_case(reference, seed, collect, batch=2, length=5, heads=4, dim=24, groups=2):
    """mamba2_recall/state_codec.py _s16_scan (:65-102), launched as scan() does for the s16
    mode (:245-253) — scan() itself refuses CPU tensors — with the statistics reduction of
    :256-262 applied to the kernel's per-4-row tiles."""
    sys.path.insert(0, str(reference))
    from mamba2_recall import state_codec as sc
    gen = torch.Generator().manual_seed(seed)
    x = torch.randn(batch, length, heads, dim, generator=gen).half()
    dt = (torch.randn(batch, length, heads, generator=gen) * 0.7).half()
    A = -(torch.rand(heads, generator=gen) * 3 + 0.05).float()
    Bm = torch.randn(batch, length, groups, 128, generator=gen).half()
    Cm = torch.randn(batch, length, groups, 128, generator=gen).half()
    D = torch.randn(heads, generator=gen).half()
    dt_bias = (torch.rand(heads, generator=gen) * 3 - 4).half()
    state = (torch.randn(batch, heads, dim, 128, generator=gen) * 0.3).half()
    initial = state.clone()
    out = torch.empty_like(x)
    ntile = triton.cdiv(dim, sc.S16_TILE)
    stats = torch.empty((batch, heads, ntile, 128), dtype=torch.float32) if collect else None
    sc._s16_scan[(batch, heads, ntile)](x, dt, A, Bm, Cm, D, dt_bias, state, out,
                                        stats if stats is not None else out, length, heads, dim, groups,
                                        collect, sc.S16_TILE, num_warps=4)
    rec = dict(x=x, dt=dt, A=A, B=Bm, C=Cm, D=D, dt_bias=dt_bias, state_in=initial, state_out=state, y=out)
    if collect:
        target = triton.cdiv(dim, sc.RP)
        if stats.shape[2] != target * (sc.RP // sc.S16_TILE):
            pad = torch.zeros((batch, heads, target * (sc.RP // sc.S16_TILE) - stats.shape[2], 128))
            stats = torch.cat((stats, pad), 2)
        rec['stats'] = stats.reshape(batch, heads, target, sc.RP // sc.S16_TILE, 128).sum(3)
    return {k: v.numpy() for k, v in rec.items()}


def mk_case(reference):
    """Digest of the reference's public MK prompts (mamba2_recall/evaluation.py:82-119) for
    both splits: sha256 of the canonical JSON of the case list, plus the counts."""
    import hashlib
    import json
    sys.path.insert(0, str(reference))
    from mamba2_recall import evaluation as ev
    out = {}
    for split in ('validation', 'test'):
        cases = ev.synthetic_mk_cases(split, 8)
        raw = json.dumps(cases, sort_keys=True, separators=(',', ':')).encode()
        out[split] = dict(count=len(cases), sha256=hashlib.sha256(raw).hexdigest(),
                          first_id=cases[0]['id'], first_answer=cases[0]['answer'])
    return out


def fp4_case(reference, seed=7):
    sys.path.insert(0, str(reference))
    from mamba2_recall import fp4
    gen = torch.Generator().manual_seed(seed)
    rows, cols = 48, 256
    w = torch.randn(rows, cols, generator=gen) * torch.exp(torch.randn(rows, cols // 16, 1, generator=gen)).repeat(1, 1, 16).reshape(rows, cols) * 0.02
    w[3, 16:32] = 0                        # an all-zero group
    w[5, :] *= 1e-4                        # tiny row (fp16 subnormal decode)
    w[7, 0] = 0.7                          # a large outlier sets the global scale
    w = w.half()
    g = fp4.tensor_global_scale(w)
    packet = fp4.quantize_chunk(w, 'fp4_g16_e4m3', g)
    decoded = fp4.decode_packet(packet)
    ties = torch.tensor([.25, .75, 1.25, 1.75, 2.5, 3.5, 5.0, -.25, -.75, -5.0, 0.0, -0.0, 7.0, -7.0])
    return dict(source=w.numpy(), codes=packet['packed'].numpy(),
                block_scale_bytes=packet['scales'].view(torch.uint8).numpy(),
                global_scale=np.asarray(packet['global_scale'].item(), np.float32),
                decoded=decoded.numpy(), tie_values=ties.numpy(),
                tie_codes=fp4.encode_e2m1(ties.float()).numpy())


def checkpoint_case(reference):
    """The reference's plan / file-spec / header builders (pure stdlib) on the tensor
    inventory of the model (names and shapes of the mamba_ssm state dict, 507 tensors at 56
    layers).  The inventory itself comes from sq325.checkpoint.tensor_inventory, which the
    test also pins by count."""
    import hashlib
    import json
    sys.path.insert(0, str(reference))
    sys.path.insert(0, str(HERE.parents[1] / 'mamb2_8b_fp4_recall_sq3.25_b200'))
    from mamba2_recall import fp4_checkpoint as rc
    from sq325 import checkpoint as ck

    def canon(x):
        return hashlib.sha256(json.dumps(x, sort_keys=True, separators=(',', ':')).encode()).hexdigest()

    out = {'production': {}, 'small': {}}
    for n_layer, vocab, limits, key in ((56, 256000, (256 * 1024 * 1024, 1024 ** 3), 'production'),
                                        (2, 64, (1024 * 1024,), 'small')):
        inv = ck.tensor_inventory(n_layer, vocab)
        ledger = {'tensors': {k: {'kind': v[0], 'shape': list(v[1])} for k, v in inv.items()}}
        for limit in limits:
            plan = rc.make_plan(ledger, limit)
            specs = rc._file_specs(plan)
            headers = {f: rc._header(spec) for f, spec in specs.items()}
            rec = dict(n_layer=n_layer, vocab=vocab, shard_limit_bytes=limit, tensors=len(plan),
                       files=len(specs), plan_sha256=canon(plan), specs_sha256=canon(specs),
                       headers_sha256={f: hashlib.sha256(h[0]).hexdigest() for f, h in headers.items()},
                       payload_bytes={f: h[2] for f, h in headers.items()})
            if key == 'small':
                rec['plan'] = plan
                rec['headers_hex'] = {f: h[0].hex() for f, h in headers.items()}
            out[key][str(limit)] = rec
    return out


def ste_case(reference, seed=500, batch=2, length=10, heads=4, dim=16, groups=2, chunk=4):
    """sq3p25 forward (random packed start and fresh zero start) and the STE backward, run by
    the interpreter exactly as scan / _StateQuantSTE.backward launch them."""
    sys.path.insert(0, str(reference))
    from mamba2_recall import state_codec as sc
    from mamba2_recall import state_training_scan as sts

    class _Libdevice:
        round = _round_half_away

    sc.libdevice = _Libdevice
    sts.libdevice = _Libdevice
    gen = torch.Generator().manual_seed(seed)
    x = torch.randn(batch, length, heads, dim, generator=gen).half()
    dt = (torch.randn(batch, length, heads, generator=gen) * 0.7).half()
    A = -(torch.rand(heads, generator=gen) * 3 + 0.05).float()
    Bm = torch.randn(batch, length, groups, 128, generator=gen).half()
    Cm = torch.randn(batch, length, groups, 128, generator=gen).half()
    D = torch.randn(heads, generator=gen).half()
    dt_bias = (torch.rand(heads, generator=gen) * 3 - 4).half()
    perm = torch.stack([torch.randperm(128, generator=gen) for _ in range(groups)]).to(torch.uint8)
    dy = torch.randn(batch, length, heads, dim, generator=gen).half()
    rec = dict(x=x, dt=dt, A=A, B=Bm, C=Cm, D=D, dt_bias=dt_bias, permutation=perm, dy=dy)
    grid = (batch, heads, triton.cdiv(dim, 16))
    for tag, random_start in (('rand_', True), ('zero_', False)):
        st = {k: torch.zeros((batch, heads, dim, w), dtype=torch.uint8) for k, w in (('lo', 8), ('hi', 8), ('q4', 32))}
        st.update({k: torch.zeros((batch, heads, dim), dtype=torch.float16) for k in ('s8', 's4')})
        if random_start:
            for k in ('lo', 'hi', 'q4'):
                st[k] = torch.randint(0, 256, st[k].shape, generator=gen, dtype=torch.uint8)
            st['s8'] = (torch.rand(batch, heads, dim, generator=gen) * 1e-2 + 1e-5).half()
            st['s4'] = (torch.rand(batch, heads, dim, generator=gen) * 1e-1 + 1e-5).half()
        rec.update({tag + 'in_' + k: v.clone() for k, v in st.items()})
        out = torch.empty_like(x)
        sc._sq_scan[grid](x, dt, A, Bm, Cm, D, dt_bias, perm, st['lo'], st['hi'], st['q4'], st['s8'], st['s4'],
                          out, length, heads, dim, groups, 16)
        rec[tag + 'y'] = out
        rec.update({tag + 'out_' + k: v for k, v in st.items()})
    nc = triton.cdiv(length, chunk)
    cp = torch.empty((batch, nc, heads, dim, 80), dtype=torch.float32)
    hist = torch.empty((batch, chunk, heads, dim, 80), dtype=torch.float32)
    adj = torch.zeros((batch, heads, dim, 80), dtype=torch.float32)
    dx = torch.empty(x.shape, dtype=torch.float32)
    ddt = torch.zeros(dt.shape, dtype=torch.float32)
    db = torch.zeros(Bm.shape, dtype=torch.float32)
    dc = torch.zeros(Cm.shape, dtype=torch.float32)
    sts._carry_checkpoints[grid](x, dt, A, Bm, dt_bias, perm, cp, length, heads, dim, groups, chunk, nc, 16)
    for c in reversed(range(nc)):
        sts._chunk_history[grid](x, dt, A, Bm, dt_bias, perm, cp, hist, length, heads, dim, groups, chunk, nc, c, 16)
        sts._chunk_backward[grid](x, dt, A, Bm, Cm, D, dt_bias, perm, hist, adj, dy, dx, ddt, db, dc, length, heads,
                                  dim, groups, chunk, c, 16)
    rec.update(checkpoints=cp, dx=dx, ddt=ddt, db=db, dc=dc, chunk=torch.tensor(chunk))
    # the diagnostic encode / decode (state_codec.py:265-331) through the reference's own
    # functions: a dense carry in permuted order with an all-zero row (scale floor 1e-8) and
    # exact half-step values (ties away from zero), then decode in both coordinate orders
    dense = torch.randn(batch, heads, dim, 128, generator=gen) * 3
    dense[0, 0, 0] = 0
    dense[0, 0, 1, :16] = torch.linspace(-127, 127, 16)
    dense[0, 0, 1, 3] = -2.5
    dense[0, 0, 1, 16:80] = torch.linspace(-7, 7, 64)
    dense[0, 0, 1, 20] = 3.5
    dense[0, 0, 1, 21] = -0.5
    state = sc.allocate_state(batch, heads, dim, 128, 'sq3p25', 'cpu')
    sc.encode_state_(state, dense)
    rec['enc_dense'] = dense
    rec.update({'enc_' + k: v.clone() for k, v in state.tensors.items()})
    rec['dec_plain'] = sc.decode_state(state)
    rec['dec_perm'] = sc.decode_state(state, perm)
    return {k: v.numpy() for k, v in rec.items()}


def adapter_case(reference, seed=11):
    sys.path.insert(0, str(reference))
    from mamba2_recall import resurface_native as native
    gen = torch.Generator().manual_seed(seed)
    width, heads, hd, tokens = 256, 16, 8, 5
    ad = native._Adapter(width, heads, device='cpu', trainable=False)
    with torch.no_grad():
        ad.V_read.copy_((torch.randn(heads, heads, generator=gen) * 0.1).half())
        ad.g_read.copy_((torch.rand(heads, generator=gen) + 0.5).half())
        ad.router_w.copy_((torch.randn(width, generator=gen) * 0.05).half())
        ad.router_b.copy_(torch.tensor(-0.5).half())
    y = torch.randn(2, tokens, heads * hd, generator=gen).half()
    u = torch.randn(2, tokens, width, generator=gen).half()
    with torch.no_grad():
        out, logits = ad(y, u, heads, hd, 'soft', False)
    return dict(V=ad.V_read.numpy(), g=ad.g_read.numpy(), w=ad.router_w.numpy(),
                b=ad.router_b.numpy(), y=y.numpy(), u=u.numpy(), out=out.numpy(),
                logits=logits.numpy())


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument('--reference', type=Path, required=True,
                    help='root of a checkout of the reference repository (read only)')
    ap.add_argument('--cases', default='codec,s16,mk,checkpoint,ste',
                    help='comma list: codec (+ fp4, adapter), s16, mk, checkpoint, ste')
    args = ap.parse_args()
    ap_cases = args.cases.split(',')
    if 's16' in ap_cases:
        rec = {}
        for tag, seed, collect in (('plain_', 300, False), ('stats_', 301, True)):
            rec.update({tag + k: v for k, v in s16_case(args.reference, seed, collect).items()})
        np.savez_compressed(HERE / 's16.npz', **rec)
        print('wrote s16')
    if 'mk' in ap_cases:
        import json
        (HERE / 'mk_cases.json').write_text(json.dumps(mk_case(args.reference), indent=1, sort_keys=True) + '\n')
        print('wrote mk')
    if 'ste' in ap_cases:
        np.savez_compressed(HERE / 'ste.npz', **ste_case(args.reference))
        # three 16-row tiles (the last one half masked), a partial last chunk, batch 1
        np.savez_compressed(HERE / 'ste_ragged.npz',
                            **ste_case(args.reference, seed=501, batch=1, length=9, heads=4, dim=40, groups=2,
                                       chunk=4))
        print('wrote ste')
    if 'checkpoint' in ap_cases:
        import json
        (HERE / 'checkpoint_plan.json').write_text(
            json.dumps(checkpoint_case(args.reference), indent=1, sort_keys=True) + '\n')
        print('wrote checkpoint')
    if 'codec' not in ap_cases:
        return
    ref = install_shims(args.reference)
    layouts = ('32_32_64', '16_64_48', '8_80_40', '24_48_56', '36_24_68', '40_16_72', '44_8_76')
    for i, layout in enumerate(layouts):
        scan = codec_case(ref, layout, seed=100 + i)
        ka = codec_case(ref, layout, seed=200 + i, known_answer=True)
        rec = {'scan_' + k: v for k, v in scan.items()}
        rec.update({'ka_' + k: v for k, v in ka.items()})
        np.savez_compressed(HERE / f'codec_{layout}.npz', **rec)
        print('wrote', layout)
    np.savez_compressed(HERE / 'fp4_g16.npz', **fp4_case(args.reference))
    np.savez_compressed(HERE / 'adapter.npz', **adapter_case(args.reference))
    print('done')


if __name__ == '__main__':
    main()
