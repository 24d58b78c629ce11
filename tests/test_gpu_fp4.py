"""GPU parity of the FP4-G16 weight kernels: exact decode, skinny GEMM (M <= 64) and the
tcgen05 GEMM path, against the oracle decode and a torch fp32 reference product."""
import numpy as np
import pytest
import torch

from oracle import fp4 as of

pytestmark = pytest.mark.gpu


def test_decode_matches_reference_golden(golden):
    from sq325 import fp4
    d = golden('fp4_g16.npz')
    w = fp4.from_arrays(d['codes'], d['block_scale_bytes'], d['global_scale'])
    out = fp4.decode_packet(w).cpu().numpy()
    assert np.array_equal(out.view(np.uint16), d['decoded'].view(np.uint16))


@pytest.mark.parametrize('shape', [(18560, 4096), (4096, 8192), (333, 128)])
def test_decode_bit_exact_random(shape):
    from sq325 import fp4
    rng = np.random.default_rng(shape[0])
    codes, blocks, g = of.synthetic_matrix(*shape, rng)
    blocks[0, :4] = 0                                         # zero block scale ...
    codes[0, :32] = rng.choice(np.array([0x00, 0x08, 0x80, 0x88], np.uint8), 32)   # ... with +-0 codes only
    blocks[1, :4] = 1                                         # e4m3 subnormal block scale
    w = fp4.from_arrays(codes, blocks, g)
    out = fp4.decode_packet(w).cpu().numpy()
    ref = of.decode(codes, blocks, g)
    assert np.array_equal(out.view(np.uint16), ref.view(np.uint16))


def _ref_linear(x16, wdec16):
    return (x16.float() @ wdec16.float().T)


@pytest.mark.parametrize('m', [1, 3, 8, 16, 33, 64, 65, 128, 300])
@pytest.mark.parametrize('shape', [(18560, 4096), (4096, 8192)])
def test_linear_matches_fp32_reference(m, shape):
    """fp16 out of an fp32-accumulated product of exactly decoded weights: compare with a
    fp32 reference; the only differences are accumulation order and the final fp16 rounding."""
    from sq325 import fp4
    rng = np.random.default_rng(m + shape[0])
    codes, blocks, g = of.synthetic_matrix(*shape, rng)
    w = fp4.from_arrays(codes, blocks, g)
    wdec = torch.from_numpy(of.decode(codes, blocks, g)).cuda()
    x = torch.from_numpy(rng.standard_normal((m, shape[1])).astype(np.float16)).cuda()
    y = fp4.linear(w, x).float()
    ref = _ref_linear(x, wdec)
    err = (y - ref).abs()
    tol = 2e-3 * ref.abs() + 1e-2 * ref.abs().mean()
    assert bool((err <= tol).all()), float((err / (ref.abs() + 1e-6)).max())


@pytest.mark.parametrize('mnk', [(128, 256, 64), (256, 512, 1024), (200, 300, 4096), (1000, 18560, 4096),
                                 (4096, 4096, 8192)])
def test_tcgen05_gemm(mnk):
    import ctypes as C
    from sq325 import _lib
    m, n, k = mnk
    gen = torch.Generator(device='cuda').manual_seed(m + n + k)
    a = torch.randn(m, k, device='cuda', generator=gen).half()
    b = torch.randn(n, k, device='cuda', generator=gen).half()
    c = torch.empty(m, n, device='cuda', dtype=torch.float16)
    _lib.call('sq_gemm_f16', _lib.ptr(a), k, _lib.ptr(b), k, _lib.ptr(c), n, m, n, k, _lib.stream_ptr())
    ref = a.float() @ b.float().T
    err = (c.float() - ref).abs()
    assert float(err.max()) <= 2e-3 * float(ref.abs().max()) + 1e-2, float(err.max())


@pytest.mark.parametrize('case', ['zero_scale_code', 'negative_scale', 'nan_scale', 'overflow'])
def test_decode_packet_rejects_what_the_reference_rejects(case):
    """mamba2_recall/fp4.py:235-249: a nonzero code in a zero-scale group, a negative or NaN
    block scale, and a weight that decodes past fp16's range are refused with the
    reference's ValueError messages; a clean matrix with zero-scale groups holding only
    +-0 codes decodes."""
    from sq325 import fp4
    rng = np.random.default_rng(12)
    codes, blocks, g = of.synthetic_matrix(64, 256, rng)
    blocks[3, 2] = 0                                  # a zero-scale group ...
    codes[3, 16:24] = np.array([0x80, 0x08, 0x00, 0x88] * 2, np.uint8)   # ... holding only +-0 codes
    fp4.decode_packet(fp4.from_arrays(codes, blocks, g))                  # accepted
    msg = {'zero_scale_code': 'Nonzero code in a zero-scale group', 'negative_scale': 'Invalid stored scale',
           'nan_scale': 'Invalid stored scale', 'overflow': 'Nonfinite decoded FP16 weights'}[case]
    if case == 'zero_scale_code':
        codes[3, 20] = 0x10
    elif case == 'negative_scale':
        blocks[5, 1] = 0x80 | 0x38
    elif case == 'nan_scale':
        blocks[7, 0] = 0x7F
    else:
        g = np.float32(1e6)                           # 6 * 448 * 1e6 overflows fp16
    with pytest.raises(ValueError, match=msg):
        fp4.decode_packet(fp4.from_arrays(codes, blocks, g))


@pytest.mark.parametrize('m', [2, 16, 17, 100, 256])
@pytest.mark.parametrize('shape', [(5328, 4096), (4096, 8192), (18560, 4096), (1000, 256)])
def test_tensor_core_linear_with_fused_decode(m, shape):
    """Batches of 2..256 rows run the tcgen05 linear that decodes the FP4 weights in shared
    memory (one CTA per 128 weight rows and K slice; 5328 and 1000 rows leave a partial last
    tile; 5328 x 4096 and 4096 x 8192 split K over a cluster of 4 CTAs and reduce through
    distributed shared memory, 18560 x 4096 runs unsplit, K = 256 cannot be split).  Same bar
    as the other projections: fp32 reference product of the exactly decoded weights within
    2e-3 relative + 1% of the mean magnitude."""
    from sq325 import _lib, fp4
    rng = np.random.default_rng(3 * m + shape[0])
    codes, blocks, g = of.synthetic_matrix(*shape, rng)
    w = fp4.from_arrays(codes, blocks, g)
    x = torch.from_numpy(rng.standard_normal((m, shape[1])).astype(np.float16)).cuda()
    y = fp4.linear(w, x)
    torch.cuda.synchronize()
    assert _lib.load().sq_device_check(_lib.stream_ptr()) == _lib.SQ_OK
    ref = _ref_linear(x.cpu(), torch.from_numpy(of.decode(codes, blocks, g)))
    err = (y.float().cpu() - ref).abs()
    tol = 2e-3 * ref.abs() + 1e-2 * ref.abs().mean()
    assert bool((err <= tol).all()), float(err.max())
