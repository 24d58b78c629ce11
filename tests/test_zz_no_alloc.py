"""sq_fp4_linear_static (the allocation-free FP4-G16 linear, staging in a static device
array) against the workspace entry point sq_fp4_linear, through the C-ABI.

Collected last on purpose: it must pass alone and after every other test has run in the
same process (the static array is set up once per device on its first call)."""
import ctypes as C

import numpy as np
import pytest
import torch

from oracle import fp4 as of

pytestmark = pytest.mark.gpu


def _static_linear(w, x, y):
    from sq325 import _lib
    m = x.shape[0]
    _lib.call('sq_fp4_linear_static', _lib.ptr(w.codes), _lib.ptr(w.block_scale_bytes), _lib.ptr(w.global_scale),
              w.rows, w.cols, _lib.ptr(x), w.cols, m, _lib.ptr(y), w.rows, _lib.stream_ptr())


# (m, n, k): m > 64 stages decoded rows in chunks of 16 MiB / (2 k) rows (1024 rows at
# k = 8192: three chunks, the last one partial; 2048 rows at k = 4096: ten chunks, a 128-row
# tail); m <= 64 runs the streaming skinny GEMM, which needs no stage.
@pytest.mark.parametrize('mnk', [(128, 2304, 8192), (300, 18560, 4096), (16, 4096, 8192), (65, 333 * 16, 128)])
def test_static_matches_workspace_entry_point(mnk):
    from sq325 import fp4
    m, n, k = mnk
    rng = np.random.default_rng(m * 7 + n)
    codes, blocks, g = of.synthetic_matrix(n, k, rng)
    w = fp4.from_arrays(codes, blocks, g)
    x = torch.from_numpy(rng.standard_normal((m, k)).astype(np.float16)).cuda()
    ref = fp4.linear(w, x).float()                      # sq_fp4_linear with a caller workspace
    tol = 2e-3 * ref.abs() + 1e-3 * ref.abs().mean()
    outs = [torch.full((m, n), float('nan'), device='cuda', dtype=torch.float16) for _ in range(3)]
    _static_linear(w, x, outs[0])                       # first call on this shape
    torch.cuda.synchronize()
    free_before = torch.cuda.mem_get_info()[0]
    _static_linear(w, x, outs[1])                       # two consecutive calls
    _static_linear(w, x, outs[2])
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free_before, 'device memory changed across the calls'
    for y in outs:
        err = (y.float() - ref).abs()
        assert bool((err <= tol).all()), float(err.max())


def test_static_rejects_k_beyond_the_scratch():
    from sq325 import _lib, fp4
    lib = _lib.load()
    kmax = lib.sq_fp4_linear_static_max_k()
    assert kmax == 32768
    k = kmax + 128
    rng = np.random.default_rng(3)
    codes, blocks, g = of.synthetic_matrix(16, k, rng)
    w = fp4.from_arrays(codes, blocks, g)
    x = torch.zeros((128, k), device='cuda', dtype=torch.float16)
    y = torch.zeros((128, 16), device='cuda', dtype=torch.float16)
    rc = lib.sq_fp4_linear_static(_lib.ptr(w.codes), _lib.ptr(w.block_scale_bytes), _lib.ptr(w.global_scale),
                                  16, k, _lib.ptr(x), k, 128, _lib.ptr(y), 16, C.c_void_p(0))
    assert rc == _lib.SQ_EINVAL
    assert b'exceeds the static scratch' in lib.sq_last_error()
    assert bool((y == 0).all())
    # m <= 64 needs no stage, so the same k is accepted there
    _static_linear(w, x[:8], y[:8])
    torch.cuda.synchronize()
    ref = fp4.linear(w, x[:8])
    assert bool((y[:8] == ref).all())


@pytest.mark.parametrize('bad', ['ldy', 'ldx'])
def test_static_rejects_short_row_strides(bad):
    """ldy < n (or ldx < k) is refused before any chunk runs: with m > 64 the chunked GEMM sees
    only one chunk's columns at a time, so it cannot catch a short output stride itself.  The
    output buffer is sized for the (wrong) strides and must come back untouched."""
    from sq325 import _lib, fp4
    lib = _lib.load()
    m, n, k = 128, 2048, 4096
    rng = np.random.default_rng(11)
    codes, blocks, g = of.synthetic_matrix(n, k, rng)
    w = fp4.from_arrays(codes, blocks, g)
    ldx = k if bad == 'ldy' else k - 128
    ldy = n - 256 if bad == 'ldy' else n
    x = torch.zeros((m, k), device='cuda', dtype=torch.float16)
    y = torch.full((m * ldy,), 7.0, device='cuda', dtype=torch.float16)
    rc = lib.sq_fp4_linear_static(_lib.ptr(w.codes), _lib.ptr(w.block_scale_bytes), _lib.ptr(w.global_scale),
                                  n, k, _lib.ptr(x), ldx, m, _lib.ptr(y), ldy, C.c_void_p(0))
    assert rc == _lib.SQ_EINVAL
    assert b'row strides' in lib.sq_last_error()
    torch.cuda.synchronize()
    assert bool((y == 7.0).all())
