"""Host side of the 'sq3p25' state mode and the training scan (no GPU): the diagnostic
encode / decode of mamba2_recall/state_codec.py:265-331, the workspace count and argument
checks of mamba2_recall/state_training_scan.py:214-239, and the C-ABI's validation."""
import ctypes as C

import numpy as np
import pytest
import torch

from sq325 import _lib
from sq325 import state_codec as sc
from sq325 import state_training as stt


def _decode_np(st, perm=None):
    """Independent numpy decode of the 52-byte rows: INT8 from the lo / hi nibble planes,
    INT4 from q4, 48 zeros; scattered to original coordinates when a permutation is given."""
    def nib(v):
        return np.stack((v & 15, v >> 4), -1).reshape(*v.shape[:-1], -1).astype(np.int32)
    q8 = (nib(st['hi']) << 4) | nib(st['lo'])
    q8 = np.where(q8 > 127, q8 - 256, q8)
    q4 = nib(st['q4'])
    q4 = np.where(q4 > 7, q4 - 16, q4)
    v = np.concatenate((q8 * st['s8'].astype(np.float32)[..., None], q4 * st['s4'].astype(np.float32)[..., None],
                        np.zeros((*q8.shape[:-1], 48), np.float32)), -1).astype(np.float32)
    if perm is None:
        return v
    b, h, p, _ = v.shape
    out = np.zeros_like(v)
    per = h // perm.shape[0]
    for hh in range(h):
        out[:, hh, :, perm[hh // per].astype(np.int64)] = np.moveaxis(v[:, hh], -1, 0)
    return out


def test_sq3p25_decode_matches_golden_state_bytes(golden):
    d = golden('ste.npz')
    st = sc.allocate_state(2, 4, 16, 128, 'sq3p25', 'cpu')
    ref = {k: d[f'rand_out_{k}'] for k in ('lo', 'hi', 'q4', 's8', 's4')}
    for k, v in ref.items():
        st.tensors[k].copy_(torch.from_numpy(v))
    assert np.array_equal(sc.decode_state(st).numpy(), _decode_np(ref))
    perm = torch.from_numpy(d['permutation'])
    assert np.array_equal(sc.decode_state(st, perm).numpy(), _decode_np(ref, d['permutation']))


def test_sq3p25_encode_round_trip_and_tie_rule():
    rng = np.random.default_rng(3)
    st = sc.allocate_state(1, 2, 8, 128, 'sq3p25', 'cpu')
    v = torch.from_numpy((rng.standard_normal((1, 2, 8, 128)) * 2).astype(np.float32))
    sc.encode_state_(st, v)
    back = sc.decode_state(st)
    s8 = st.tensors['s8'].float()[..., None]
    s4 = st.tensors['s4'].float()[..., None]
    # half a step, plus |code| x the fp16 rounding of the fp32 denominator the codes used
    assert torch.all((back[..., :16] - v[..., :16]).abs() <= s8 * (0.5 + 127 * 2.0 ** -11) + 1e-6)
    assert torch.all((back[..., 16:80] - v[..., 16:80]).abs() <= s4 * (0.5 + 7 * 2.0 ** -11) + 1e-6)
    assert torch.all(back[..., 80:] == 0)
    # ties: 7 * 0.5 / 7 of the row maximum rounds away from zero
    w = torch.zeros(1, 2, 8, 128)
    w[..., 16] = 7.0
    w[..., 17] = 2.5
    w[..., 18] = -2.5
    sc.encode_state_(st, w)
    q = sc.decode_state(st)[..., 16:19] / st.tensors['s4'].float()[..., None]
    assert torch.equal(q.round(), torch.tensor([7.0, 3.0, -3.0]).expand_as(q))


def test_sq3p25_state_checks():
    with pytest.raises(ValueError):
        sc.allocate_state(1, 4, 16, 64, 'sq3p25', 'cpu')
    st = sc.allocate_state(1, 4, 16, 128, 'sq3p25', 'cpu')
    assert {k: (tuple(v.shape), v.dtype) for k, v in st.tensors.items()} == {
        'lo': ((1, 4, 16, 8), torch.uint8), 'hi': ((1, 4, 16, 8), torch.uint8),
        'q4': ((1, 4, 16, 32), torch.uint8), 's8': ((1, 4, 16), torch.float16), 's4': ((1, 4, 16), torch.float16)}
    with pytest.raises(ValueError, match='match state shape'):
        sc.encode_state_(st, torch.zeros(1, 4, 16, 127))
    with pytest.raises(ValueError, match='FP16'):
        sc.encode_state_(st, torch.full((1, 4, 16, 128), 1e7))


def test_training_workspace_bytes_and_library_count():
    got = stt.training_workspace_bytes(2, 100, heads=8, dim=64, groups=2, chunk_size=32)
    nc = 4
    carries = 2 * (nc + 32 + 1) * 8 * 64 * 80 * 4
    assert got == {'carry_scratch_bytes': carries, 'gradient_scratch_bytes': 2 * 100 * (8 * 64 + 8 + 2 * 2 * 128) * 4,
                   'total_scratch_bytes': carries + 2 * 100 * (8 * 64 + 8 + 2 * 2 * 128) * 4}
    # the library's scratch: the same carries plus one chunk of dB / dC partials per
    # (head, 16-row tile); the gradients themselves are the caller's outputs
    assert _lib.load().sq_ste_workspace(2, 100, 8, 64, 32) == carries + 2 * 32 * 8 * 4 * 256 * 4


def test_scan_training_checks_match_reference():
    z = torch.zeros(1)
    with pytest.raises(ValueError, match='sq3p25 only'):
        stt.scan_training(z, z, z, z, z, z, z, z, mode='s16')
    for bad in (0, 257, 1.5):
        with pytest.raises(ValueError, match='chunk_size'):
            stt.scan_training(z, z, z, z, z, z, z, z, chunk_size=bad)
    with pytest.raises(ValueError, match='frozen'):
        stt.scan_training(z, z, torch.zeros(1, requires_grad=True), z, z, z, z, z)


def test_ste_abi_validation_needs_no_gpu():
    lib = _lib.load()
    a = _lib.Sq3p25Args()
    assert lib.sq_sq3p25_scan(C.byref(a), None) == _lib.SQ_EINVAL
    assert b'null pointer' in lib.sq_last_error()
    assert lib.sq_ste_backward(C.byref(a), 4, None, None, None, None, None, None, 0, None) == _lib.SQ_EINVAL


@pytest.mark.parametrize('case', ['ste.npz', 'ste_ragged.npz'])
def test_sq3p25_encode_decode_match_reference(golden, case):
    """encode_state_ and decode_state (both coordinate orders) against the reference's own
    functions run on the same dense carry (state_codec.py:265-331): packed bytes and scales
    bit for bit, including an all-zero row and exact half-step ties."""
    d = golden(case)
    b, h, p, _ = d['enc_dense'].shape
    st = sc.allocate_state(b, h, p, 128, 'sq3p25', 'cpu')
    sc.encode_state_(st, torch.from_numpy(d['enc_dense']))
    for k in ('lo', 'hi', 'q4', 's8', 's4'):
        assert np.array_equal(st.tensors[k].numpy().view(np.uint8), d['enc_' + k].view(np.uint8)), k
    assert np.array_equal(sc.decode_state(st).numpy().view(np.uint32), d['dec_plain'].view(np.uint32))
    perm = torch.from_numpy(d['permutation'])
    assert np.array_equal(sc.decode_state(st, perm).numpy().view(np.uint32), d['dec_perm'].view(np.uint32))
