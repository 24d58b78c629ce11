"""Failure detection on the GPU without a fault: a bounded wait that runs out.

The skinny-GEMM kernel's pipeline waits take their limit from sq_set_wait_limit_ns.  A 1 ns
limit makes them expire (the consumers give up on a stage the copy engine has not filled
yet, the producer on a stage the consumers never free); the kernel then records an error
bit, drains its own copies with the default limit and returns.  The tests check that the
host sees SQ_ETIMEOUT through the entry point's check, and that the context stays usable:
the next call, with the default limit back, gives the exact result.
"""
import numpy as np
import pytest
import torch

from oracle import fp4 as of

pytestmark = pytest.mark.gpu


def test_expired_wait_reports_timeout_and_context_stays_usable():
    from sq325 import _lib, fp4
    lib = _lib.load()
    rng = np.random.default_rng(5)
    w = fp4.from_arrays(*of.synthetic_matrix(4096, 4096, rng))
    x = torch.from_numpy(rng.standard_normal((1, 4096)).astype(np.float16)).cuda()   # one row: the skinny GEMM
    ref = fp4.linear(w, x)
    assert lib.sq_device_check(_lib.stream_ptr()) == _lib.SQ_OK
    try:
        _lib.call('sq_set_wait_limit_ns', 1)
        fp4.linear(w, x)
        rc = lib.sq_device_check(_lib.stream_ptr())
    finally:
        _lib.call('sq_set_wait_limit_ns', 0)
    assert rc == _lib.SQ_ETIMEOUT, rc
    assert b'bounded wait' in lib.sq_last_error()
    # the word was cleared by the check; the next call runs normally and exactly
    y = fp4.linear(w, x)
    assert lib.sq_device_check(_lib.stream_ptr()) == _lib.SQ_OK
    assert torch.equal(y, ref)


def test_expired_wait_in_a_decode_step_raises_device_timeout():
    """The model runtime's decode-step projections run the same kernel: the controller's
    check() raises DeviceTimeout (the reference's RuntimeError family), and after a reset the
    controller decodes normally again."""
    from _models import build_pair
    from sq325 import PredictorState, _lib
    gm, _, statics = build_pair(n_layer=2, vocab=512, seed=6, adapter=True)
    ids = torch.from_numpy(np.random.default_rng(8).integers(0, 512, (1, 9))).cuda()
    with PredictorState(gm, *statics) as ex:
        ex.backbone(ids, reset=True)
        ref = ex.backbone(ids[:, :1]).clone()
        ex.check()
        ex.backbone(ids, reset=True)
        try:
            _lib.call('sq_set_wait_limit_ns', 1)
            ex.backbone(ids[:, :1])
            with pytest.raises(_lib.DeviceTimeout):
                ex.check()
        finally:
            _lib.call('sq_set_wait_limit_ns', 0)
        ex.backbone(ids, reset=True)
        again = ex.backbone(ids[:, :1])
        ex.check()
        assert torch.equal(again, ref)
