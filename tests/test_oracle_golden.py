"""The CPU oracle is pinned to the reference: bit-exact on every golden vector.

Golden vectors were produced by the reference's own code (tests/golden/make_golden.py):
the production codec kernel under the Triton interpreter, fp4.quantize_chunk /
decode_packet, and the Resurface adapter forward.
"""
import numpy as np
import pytest
import torch

from oracle import codec as oc
from oracle import fp4 as of
from oracle import model as om


@pytest.mark.parametrize('layout', oc.LAYOUTS)
@pytest.mark.parametrize('case', ['scan_', 'ka_'])
def test_codec_oracle_matches_reference_kernel(golden, layout, case):
    d = golden(f'codec_{layout}.npz')
    g = lambda k: d[case + k]
    st = {k: g('in_' + k).copy() for k in ('lo', 'hi', 'q4', 'latent', 's8', 's4')}
    corr = oc.predictor_correction(g('C'), g('permutation'), g('predictor'), layout)
    assert np.array_equal(corr.view(np.uint32), g('corr').view(np.uint32))
    y = oc.latent_scan(g('x'), g('dt'), g('A'), g('B'), g('C'), g('D'), g('dt_bias'), st, g('permutation'),
                       g('basis'), g('latent_scale'), g('predictor'), layout)
    assert np.array_equal(y.view(np.uint16), g('y').view(np.uint16))
    for k in st:
        assert np.array_equal(st[k].view(np.uint8), g('out_' + k).view(np.uint8)), k


@pytest.mark.parametrize('layout', oc.LAYOUTS)
def test_known_answer_is_decode_requant_pack(golden, layout):
    """A=0, x=0: one kernel token re-encodes the decoded rows; the oracle's standalone
    decode -> encode reproduces the reference kernel's bytes exactly."""
    d = golden(f'codec_{layout}.npz')
    g = lambda k: d['ka_' + k]
    st = {k: g('in_' + k) for k in ('lo', 'hi', 'q4', 'latent', 's8', 's4')}
    hpg = g('x').shape[2] // g('B').shape[2]
    tiers, z = oc.decode_state(st, layout, g('latent_scale'), hpg)
    enc = oc.encode_state(tiers, z, layout, g('latent_scale'), hpg)
    for k in enc:
        a, b = enc[k].view(np.uint8), g('out_' + k).view(np.uint8)
        if k == 'latent':
            # a zero latent keeps or loses its sign in the kernel depending on the sign of
            # the (zero) update term (x*dt)*dot_b; both bytes decode to 0.0
            a, b = np.where(a == 0x80, 0, a), np.where(b == 0x80, 0, b)
        assert np.array_equal(a, b), k


def test_layout_counts_match_reference_shift():
    assert [oc.layout_counts(l) for l in oc.LAYOUTS] == [
        (32, 28, 68), (16, 60, 52), (8, 76, 44), (24, 44, 60), (36, 20, 72), (40, 12, 76), (44, 4, 80)]
    for l in oc.LAYOUTS:
        n8, n4, nz = oc.layout_counts(l)
        assert n8 // 2 * 2 + n4 // 2 + 2 + 4 == 52


def test_e4m3_table_known_answers():
    v = oc.E4M3_VALUES
    finite = np.isfinite(v)
    assert finite.sum() == 254                        # docs/evidence/.../v13/cpu_reference.json
    assert len(np.unique(v[finite])) == 253           # +0 and -0 coincide
    t = torch.arange(256, dtype=torch.uint8).view(torch.float8_e4m3fn).float().numpy()
    assert np.array_equal(np.isnan(t), np.isnan(v))
    assert np.array_equal(t[finite], v[finite])


def test_f32_to_e4m3_matches_torch_rne():
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.standard_normal(200000) * s for s in (1e-3, 0.05, 1, 30, 200)]).astype(np.float32)
    x = np.clip(x, -448, 448)
    ties = (oc.E4M3_VALUES[np.isfinite(oc.E4M3_VALUES)].astype(np.float64))
    ties = np.unique(ties)
    mids = ((ties[1:] + ties[:-1]) / 2).astype(np.float32)            # exact midpoints
    x = np.concatenate([x, mids, -mids, np.float32([0, -0.0, 448, -448, 2 ** -10, 2 ** -9])])
    ref = torch.from_numpy(x).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert np.array_equal(oc.f32_to_e4m3(x), ref)


def test_round_half_away_and_quantize():
    q = np.float32([0.5, 1.5, 2.5, -0.5, -2.5, 0.49999997, 126.5, -7.5, 7.49])
    assert oc.round_half_away(q).tolist() == [1, 2, 3, -1, -3, 0, 127, -8, 7]
    codes = oc.stored_quantize(np.float32([1.0, -3.5, 100.0, 0.0]), np.float32([1.0, 1.0, 0.5, 0.0]), 7)
    assert codes.tolist() == [1, -4, 7, 0]


def test_markstein_division_is_exact():
    """The kernel's division: q0 = a*rcp(s); r = fma(-q0,s,a); q = fma(r,rcp(s),q0) == RN(a/s).
    Emulated exactly on the CPU (float64 holds the fp32 products and remainders exactly)."""
    rng = np.random.default_rng(1)
    n = 400000
    s = np.float32(np.exp(rng.uniform(np.log(6e-8), np.log(2.0), n)).astype(np.float16).astype(np.float32))
    s = s[s > 0]
    k = rng.integers(-127, 128, s.shape[0]).astype(np.float32)
    # values at and around half-integer quotients
    a = ((k + np.float32(0.5)) * s).astype(np.float32)
    a = np.concatenate([a, np.nextafter(a, np.float32(np.inf)), np.nextafter(a, np.float32(-np.inf)),
                        (rng.uniform(-127, 127, s.shape[0]).astype(np.float32) * s).astype(np.float32)])
    ss = np.tile(s, 4)
    inv = (np.float32(1.0) / ss).astype(np.float32)

    def fma(x, y, z):
        return (x.astype(np.float64) * y.astype(np.float64) + z.astype(np.float64)).astype(np.float32)
    q0 = (a * inv).astype(np.float32)
    r = fma(-q0, ss, a)
    q = fma(r, inv, q0)
    assert np.array_equal(q, (a / ss).astype(np.float32))


def test_fp4_oracle_matches_reference_decode(golden):
    d = golden('fp4_g16.npz')
    dec = of.decode(d['codes'], d['block_scale_bytes'], d['global_scale'])
    assert np.array_equal(dec.view(np.uint16), d['decoded'].view(np.uint16))


def test_fp4_tie_table():
    d_vals = np.float32([.25, .75, 1.25, 1.75, 2.5, 3.5, 5.0])
    assert of.encode_e2m1(d_vals).tolist() == [0, 2, 2, 4, 4, 6, 6]
    assert of.encode_e2m1(-d_vals).tolist() == [0, 10, 10, 12, 12, 14, 14]
    assert of.encode_e2m1(np.float32([0.0, -0.0, 7.0, -7.0])).tolist() == [0, 0, 7, 15]


def test_fp4_oracle_encode_matches_reference(golden):
    d = golden('fp4_g16.npz')
    assert of.encode_e2m1(d['tie_values']).tolist() == d['tie_codes'].tolist()
    codes = of.unpack(d['codes'], d['decoded'].shape[1])
    assert np.array_equal(of.pack(codes), d['codes'])


def test_adapter_oracle_matches_reference(golden):
    """The adapter forward restated in oracle.model (fp32 accumulation, fp16 rounding at
    each tensor boundary) against the reference _Adapter.forward run on CPU; CPU half
    matmuls round partial sums differently, so the bound is a few fp16 ulps."""
    d = golden('adapter.npz')
    heads, hd = d['V'].shape[0], d['y'].shape[-1] // d['V'].shape[0]
    y = torch.from_numpy(d['y']).reshape(-1, heads * hd)
    u = torch.from_numpy(d['u']).reshape(y.shape[0], -1)
    old = om.HEADS, om.HEAD_DIM
    om.HEADS, om.HEAD_DIM = heads, hd
    try:
        out = om.resurface(y, u, torch.from_numpy(d['V']), torch.from_numpy(d['g']), torch.from_numpy(d['w']),
                           torch.from_numpy(d['b']))
    finally:
        om.HEADS, om.HEAD_DIM = old
    ref = torch.from_numpy(d['out']).reshape_as(out)
    assert torch.allclose(out.float(), ref.float(), rtol=2e-3, atol=2e-3)


@pytest.mark.parametrize('layout', oc.LAYOUTS)
def test_c_restatement_matches_reference_goldens(golden, layout):
    """oracle/csrc/latent_scan.c (the fast checker) reproduces the reference kernel's golden
    runs bit for bit: readouts and packed state bytes."""
    from oracle import cscan
    d = golden(f'codec_{layout}.npz')
    for pre in ('scan_', 'ka_'):
        st = {k: d[pre + 'in_' + k].copy() for k in ('lo', 'hi', 'q4', 'latent', 's8', 's4')}
        y = cscan.latent_scan(*(d[pre + k] for k in ('x', 'dt', 'A', 'B', 'C', 'D', 'dt_bias')), st,
                              *(d[pre + k] for k in ('permutation', 'basis', 'latent_scale', 'predictor')), layout)
        assert np.array_equal(y.view(np.uint16), d[pre + 'y'].view(np.uint16)), pre
        for k in ('lo', 'hi', 'q4', 's8', 's4'):
            assert np.array_equal(st[k].view(np.uint8), d[pre + 'out_' + k].view(np.uint8)), (pre, k)


@pytest.mark.parametrize('layout', oc.LAYOUTS)
def test_c_restatement_matches_numpy_restatement(layout):
    """Random multi-token calls at 32 heads x 64 rows (random packed rows and latents):
    the C and numpy restatements give identical readouts and state bytes."""
    from oracle import cscan
    n8, n4, nz = oc.layout_counts(layout)
    rng = np.random.default_rng(40 + oc.LAYOUTS.index(layout))
    B, L, H, P, G = 2, 9, 32, 64, 8
    args = (rng.standard_normal((B, L, H, P)).astype(np.float16), (rng.standard_normal((B, L, H)) * 0.5).astype(np.float16),
            -(rng.random(H) * 3 + 0.1).astype(np.float32), rng.standard_normal((B, L, G, 128)).astype(np.float16),
            rng.standard_normal((B, L, G, 128)).astype(np.float16), rng.standard_normal(H).astype(np.float16),
            (rng.random(H) * 3 - 4).astype(np.float16))
    tables = (np.stack([rng.permutation(128) for _ in range(G)]).astype(np.uint8),
              rng.standard_normal((G, nz, 2)).astype(np.float16), (rng.random((G, 2)) + 0.1).astype(np.float16),
              (rng.standard_normal((G, n8 + n4 + 2, nz)) / np.sqrt(n8 + n4 + 2)).astype(np.float16))
    st = oc.allocate_state(B, H, P, layout)
    for k in ('lo', 'hi', 'q4'):
        st[k][...] = rng.integers(0, 256, st[k].shape, dtype=np.uint8)
    for k in ('s8', 's4'):
        st[k][...] = (rng.random(st[k].shape) * 0.05).astype(np.float16)
    st['latent'][...] = oc.f32_to_e4m3(rng.standard_normal(st['latent'].shape).astype(np.float32) * 8)
    st2 = {k: v.copy() for k, v in st.items()}
    y1 = oc.latent_scan(*args, st, *tables, layout)
    y2 = cscan.latent_scan(*args, st2, *tables, layout)
    assert np.array_equal(y1.view(np.uint16), y2.view(np.uint16))
    for k in st:
        assert np.array_equal(st[k].view(np.uint8), st2[k].view(np.uint8)), k


@pytest.mark.parametrize('tag', ['plain_', 'stats_'])
def test_s16_oracle_matches_reference_kernel(golden, tag):
    """oracle.codec.s16_scan against the reference's _s16_scan run by the interpreter
    (mamba2_recall/state_codec.py:65-102), statistics reduction included (:256-262)."""
    d = golden('s16.npz')
    st = d[tag + 'state_in'].copy()
    y, stats = oc.s16_scan(*(d[tag + k] for k in ('x', 'dt', 'A', 'B', 'C', 'D', 'dt_bias')), st,
                           collect_stats=(tag == 'stats_'))
    assert np.array_equal(y.view(np.uint16), d[tag + 'y'].view(np.uint16))
    assert np.array_equal(st.view(np.uint16), d[tag + 'state_out'].view(np.uint16))
    if tag == 'stats_':
        assert np.array_equal(stats.view(np.uint32), d['stats_stats'].view(np.uint32))


@pytest.mark.parametrize('case', ['ste.npz', 'ste_ragged.npz'])
@pytest.mark.parametrize('tag', ['rand_', 'zero_'])
def test_sq3p25_oracle_matches_reference_kernel(golden, tag, case):
    """oracle.ste.sq3p25_scan against the reference's packed `_sq_scan` run by the interpreter
    (mamba2_recall/state_codec.py:105-176): readout and every state byte, from a random and
    from a zero state; ste_ragged has a half-masked 16-row tile (dim 40)."""
    from oracle import ste
    d = golden(case)
    st = {k: d[f'{tag}in_{k}'].copy() for k in ('lo', 'hi', 'q4', 's8', 's4')}
    y = ste.sq3p25_scan(*(d[k] for k in ('x', 'dt', 'A', 'B', 'C', 'D', 'dt_bias')), st, d['permutation'])
    assert np.array_equal(y.view(np.uint16), d[tag + 'y'].view(np.uint16))
    for k, v in st.items():
        assert np.array_equal(v.view(np.uint8), d[f'{tag}out_{k}'].view(np.uint8)), k


@pytest.mark.parametrize('case', ['ste.npz', 'ste_ragged.npz'])
def test_ste_backward_oracle_matches_reference_kernels(golden, case):
    """oracle.ste.ste_backward against `_carry_checkpoints` / `_chunk_history` /
    `_chunk_backward` run by the interpreter (mamba2_recall/state_training_scan.py:24-211):
    checkpoints, dx, ddt, dB and dC bit for bit; ste_ragged has three row tiles (the last
    half masked) and a partial last chunk."""
    from oracle import ste
    d = golden(case)
    dx, ddt, db, dc, cp = ste.ste_backward(*(d[k] for k in ('x', 'dt', 'A', 'B', 'C', 'D', 'dt_bias',
                                                            'permutation', 'dy')), int(d['chunk']))
    for name, got in (('checkpoints', cp), ('dx', dx), ('ddt', ddt), ('db', db), ('dc', dc)):
        assert np.array_equal(got.view(np.uint32), d[name].view(np.uint32)), name


def test_ste_oracle_device_math_hook_is_neutral(golden):
    """Supplying numpy's own softplus / decay / sigmoid through `device_math` reproduces the
    golden runs: the hook only swaps the transcendental values, nothing else."""
    from oracle import ste
    d = golden('ste.npz')
    raw = (d['dt'].astype(np.float32) + d['dt_bias'].astype(np.float32)[None, None, :]).astype(np.float32)
    soft = np.where(raw <= np.float32(20), np.log(np.exp(raw) + np.float32(1)), raw).astype(np.float32)
    math = {'softplus': soft, 'decay': np.exp((d['A'][None, None, :] * soft).astype(np.float32)).astype(np.float32),
            'sigmoid': np.where(raw <= np.float32(20), (np.float32(1) / (np.float32(1) + np.exp(-raw))).astype(np.float32),
                                np.float32(1)).astype(np.float32)}
    st = {k: d[f'zero_in_{k}'].copy() for k in ('lo', 'hi', 'q4', 's8', 's4')}
    y = ste.sq3p25_scan(*(d[k] for k in ('x', 'dt', 'A', 'B', 'C', 'D', 'dt_bias')), st, d['permutation'],
                        device_math=math)
    assert np.array_equal(y.view(np.uint16), d['zero_y'].view(np.uint16))
    got = ste.ste_backward(*(d[k] for k in ('x', 'dt', 'A', 'B', 'C', 'D', 'dt_bias', 'permutation', 'dy')),
                           int(d['chunk']), device_math=math)
    for name, g in zip(('dx', 'ddt', 'db', 'dc', 'checkpoints'), got):
        assert np.array_equal(g.view(np.uint32), d[name].view(np.uint32)), name
