"""GPU parity of the packed 'sq3p25' scan (sq_sq3p25_scan) and its straight-through training
backward (sq_ste_backward, scan_training) against the reference kernels' golden runs
(tests/golden/ste.npz: mamba2_recall/state_codec.py:105-176 and
mamba2_recall/state_training_scan.py:24-211 under the Triton interpreter) and the oracle.

Every product and sum is rounded once in the reference's order and the requantisation
divides exactly, so the forward differs from the golden runs only where CUDA's expf / logf
(softplus, decay) differ from numpy's by an ulp.  Bars: >= 99% of readouts and state bytes
identical, readouts within 2e-2.  The backward accumulates dB / dC over heads and ddt over
rows with atomics, whose order differs from the reference's tile order; bars: relative L2
error <= 1e-4 and every element within 1e-3 of the largest magnitude (float32 sums), and
checkpoints (no atomics) >= 99% bit-identical."""
import ctypes as C

import numpy as np
import pytest
import torch

from oracle import ste as ost

pytestmark = pytest.mark.gpu

KEYS = ('x', 'dt', 'A', 'B', 'C', 'D', 'dt_bias')
STATE = ('lo', 'hi', 'q4', 's8', 's4')


def _cuda(d, k):
    return torch.from_numpy(np.ascontiguousarray(d[k])).cuda()


def _forward(d, state_in=None):
    from sq325 import state_codec as sc
    x = _cuda(d, 'x')
    st = sc.allocate_state(x.shape[0], x.shape[2], x.shape[3], 128, 'sq3p25', 'cuda')
    if state_in is not None:
        for k in STATE:
            st.tensors[k].copy_(torch.from_numpy(state_in[k]))
    y, stats = sc.scan(x, *(_cuda(d, k) for k in KEYS[1:]), st, permutation=_cuda(d, 'permutation'))
    torch.cuda.synchronize()
    assert stats is None
    return y.cpu().numpy(), {k: st.tensors[k].cpu().numpy() for k in STATE}


def _check_forward(y, st, y_ref, st_ref):
    assert np.allclose(y.astype(np.float32), y_ref.astype(np.float32), rtol=2e-2, atol=2e-2)
    assert (y.view(np.uint16) == y_ref.view(np.uint16)).mean() >= 0.99
    for k in STATE:
        assert (st[k].view(np.uint8) == st_ref[k].view(np.uint8)).mean() >= 0.99, k


def _close(got, ref, name):
    got, ref = np.asarray(got, np.float64), np.asarray(ref, np.float64)
    scale = max(np.abs(ref).max(), 1e-30)
    rel_l2 = np.linalg.norm(got - ref) / max(np.linalg.norm(ref), 1e-30)
    worst = np.abs(got - ref).max() / scale
    assert rel_l2 <= 1e-4 and worst <= 1e-3, f'{name}: rel_l2 {rel_l2:.3e}, max/scale {worst:.3e}'


def _backward_abi(d, chunk):
    """sq_ste_backward called directly; returns the gradients and the checkpoint region of the
    workspace ([B][NC][H][P][80] fp32 at offset 0)."""
    from sq325 import _lib
    from sq325.state_codec import sq3p25_args
    t = {k: _cuda(d, k) for k in (*KEYS, 'permutation', 'dy')}
    b, length, h, p = t['x'].shape
    out = {k: torch.empty(t[src].shape, device='cuda', dtype=torch.float32)
           for k, src in (('dx', 'x'), ('ddt', 'dt'), ('db', 'B'), ('dc', 'C'))}
    nbytes = int(_lib.load().sq_ste_workspace(b, length, h, p, chunk))
    work = torch.empty(nbytes, device='cuda', dtype=torch.uint8)
    a = sq3p25_args(*(t[k] for k in KEYS), t['permutation'])
    _lib.call('sq_ste_backward', C.byref(a), chunk, t['dy'].data_ptr(), *(out[k].data_ptr() for k in
              ('dx', 'ddt', 'db', 'dc')), work.data_ptr(), nbytes, _lib.stream_ptr())
    torch.cuda.synchronize()
    nc = -(-length // chunk)
    cp = work[:b * nc * h * p * 80 * 4].view(torch.float32).view(b, nc, h, p, 80)
    return {k: v.cpu().numpy() for k, v in out.items()}, cp.cpu().numpy()


@pytest.mark.parametrize('tag', ['rand_', 'zero_'])
def test_sq3p25_scan_matches_reference_golden(golden, tag):
    d = golden('ste.npz')
    y, st = _forward(d, {k: d[f'{tag}in_{k}'] for k in STATE})
    _check_forward(y, st, d[tag + 'y'], {k: d[f'{tag}out_{k}'] for k in STATE})


@pytest.mark.parametrize('dim', [64, 40])
def test_sq3p25_scan_matches_oracle_at_model_geometry(dim):
    """32 heads over 4 groups, 33 tokens, batch 2, random start state; dim 40 leaves a
    partial warp."""
    rng = np.random.default_rng(dim)
    d = _inputs(rng, 2, 33, 32, dim, 4)
    from sq325 import state_codec as sc
    dense = torch.from_numpy((rng.standard_normal((2, 32, dim, 128)) * 0.3).astype(np.float32))
    st0 = sc.allocate_state(2, 32, dim, 128, 'sq3p25', 'cpu')
    sc.encode_state_(st0, dense)
    state_in = {k: v.numpy() for k, v in st0.tensors.items()}
    st_ref = {k: v.copy() for k, v in state_in.items()}
    y_ref = ost.sq3p25_scan(*(d[k] for k in KEYS), st_ref, d['permutation'])
    y, st = _forward(d, state_in)
    _check_forward(y, st, y_ref, st_ref)


def test_ste_backward_matches_reference_golden(golden):
    d = golden('ste.npz')
    grads, cp = _backward_abi(d, int(d['chunk']))
    assert cp.shape == d['checkpoints'].shape
    assert (cp.view(np.uint32) == d['checkpoints'].view(np.uint32)).mean() >= 0.99
    assert np.allclose(cp, d['checkpoints'], rtol=1e-3, atol=1e-3)
    for k in ('dx', 'ddt', 'db', 'dc'):
        _close(grads[k], d[k], k)


def test_scan_training_autograd_matches_reference_golden(golden):
    """The autograd path: zero-state forward equal to the golden zero-start readout, and the
    fp16 gradients of x, dt, B, C equal to the golden fp32 gradients rounded to fp16."""
    from sq325.state_training import scan_training
    d = golden('ste.npz')
    t = {k: _cuda(d, k) for k in (*KEYS, 'permutation', 'dy')}
    for k in ('x', 'dt', 'B', 'C'):
        t[k].requires_grad_(True)
    y = scan_training(*(t[k] for k in KEYS), t['permutation'], chunk_size=int(d['chunk']))
    y.backward(t['dy'])
    torch.cuda.synchronize()
    ynp = y.detach().cpu().numpy()
    assert (ynp.view(np.uint16) == d['zero_y'].view(np.uint16)).mean() >= 0.99
    for k, g in (('x', 'dx'), ('dt', 'ddt'), ('B', 'db'), ('C', 'dc')):
        grad = t[k].grad
        assert grad.dtype == torch.float16 and tuple(grad.shape) == d[g].shape
        ref = d[g].astype(np.float16).astype(np.float32)
        assert np.allclose(grad.float().cpu().numpy(), ref, rtol=2e-3, atol=1e-3 * np.abs(ref).max()), k
    assert t['A'].grad is None and t['D'].grad is None


def _inputs(rng, b, length, h, p, g):
    perm = np.stack([rng.permutation(128) for _ in range(g)]).astype(np.uint8)
    return dict(x=rng.standard_normal((b, length, h, p)).astype(np.float16),
                dt=(rng.standard_normal((b, length, h)) * 0.5).astype(np.float16),
                A=-(rng.random(h) * 3 + 0.1).astype(np.float32),
                B=rng.standard_normal((b, length, g, 128)).astype(np.float16),
                C=rng.standard_normal((b, length, g, 128)).astype(np.float16),
                D=rng.standard_normal(h).astype(np.float16),
                dt_bias=(rng.random(h) * 3 - 4).astype(np.float16), permutation=perm,
                dy=rng.standard_normal((b, length, h, p)).astype(np.float16))


def test_ste_backward_matches_oracle_and_is_chunk_invariant():
    """24 tokens, 8 heads over 2 groups, dim 64: the oracle at chunk 8, and the same
    gradients at chunks 1, 5, 24 and 256 (a chunk longer than the sequence)."""
    rng = np.random.default_rng(7)
    d = _inputs(rng, 2, 24, 8, 64, 2)
    ref = ost.ste_backward(*(d[k] for k in (*KEYS, 'permutation', 'dy')), 8)
    grads, cp = _backward_abi(d, 8)
    assert np.allclose(cp, ref[4], rtol=1e-3, atol=1e-3)
    for k, r in zip(('dx', 'ddt', 'db', 'dc'), ref[:4]):
        _close(grads[k], r, k)
    for chunk in (1, 5, 24, 256):
        other, _ = _backward_abi(d, chunk)
        for k in ('dx', 'ddt', 'db', 'dc'):
            _close(other[k], grads[k], f'{k} chunk {chunk}')


def test_ste_backward_rejects_bad_arguments():
    from sq325 import _lib
    from sq325.state_codec import sq3p25_args
    rng = np.random.default_rng(1)
    d = _inputs(rng, 1, 4, 4, 16, 2)
    t = {k: _cuda(d, k) for k in (*KEYS, 'permutation', 'dy')}
    a = sq3p25_args(*(t[k] for k in KEYS), t['permutation'])
    buf = torch.empty(64, device='cuda', dtype=torch.float32)
    small = torch.empty(16, device='cuda', dtype=torch.uint8)
    for chunk, work, nbytes, match in ((0, small, 16, 'chunk_size'), (257, small, 16, 'chunk_size'),
                                       (4, small, 16, 'workspace')):
        with pytest.raises(ValueError, match=match):
            _lib.call('sq_ste_backward', C.byref(a), chunk, t['dy'].data_ptr(), *(buf.data_ptr(),) * 4,
                      work.data_ptr(), nbytes, _lib.stream_ptr())
