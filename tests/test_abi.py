"""The C-ABI library loads and exports every symbol include/sq325.h declares (no GPU needed)."""
import ctypes as C
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / 'include' / 'sq325.h'


def declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r'\b(sq_[a-z0-9_]+)\s*\(', text)))


@pytest.fixture(scope='module')
def lib():
    from sq325 import _lib
    return _lib.load()


def test_header_declares_entry_points():
    syms = declared_symbols()
    assert {'sq_scan', 'sq_state_encode', 'sq_state_decode', 'sq_fp4_decode', 'sq_fp4_linear',
            'sq_model_forward', 'sq_model_score', 'sq_model_greedy'} <= set(syms)


def test_every_declared_symbol_is_exported(lib):
    for name in declared_symbols():
        assert hasattr(lib, name), name


def test_binding_prototypes_cover_header():
    from sq325 import _lib
    assert set(declared_symbols()) == set(_lib.exported_symbols())


def test_host_only_entry_points(lib):
    assert lib.sq_abi_version() == 1
    from sq325 import codec
    for i, name in enumerate(codec.LAYOUTS):
        assert lib.sq_layout_index(name.encode()) == i
        n8, n4, nz = C.c_int(), C.c_int(), C.c_int()
        assert lib.sq_layout_counts(i, C.byref(n8), C.byref(n4), C.byref(nz)) == 0
        d = codec.layout_descriptor(name)
        assert (n8.value, n4.value, nz.value) == (d['n8'], d['n4'], d['nzero'])
    assert lib.sq_layout_index(b'12_34_56') == -1
    assert lib.sq_layout_counts(7, None, None, None) == 1
    assert b'unknown layout' in lib.sq_last_error()
    assert lib.sq_state_bytes(1, 128, 64) == 425984


def test_argument_validation_needs_no_gpu(lib):
    from sq325 import _lib
    a = _lib.ScanArgs()
    assert lib.sq_scan(C.byref(a), None) == _lib.SQ_EINVAL
    assert b'null pointer' in lib.sq_last_error()
    with pytest.raises(ValueError):
        _lib.call('sq_scan', None, None)
    cfg = _lib.ModelConfig(0, 256000, 1e-5)
    h = C.c_void_p()
    assert lib.sq_model_create(C.byref(cfg), C.byref(h)) == _lib.SQ_EINVAL


def test_gemm_timer_validation_needs_no_gpu(lib):
    from sq325 import _lib
    assert lib.sq_model_time_gemm(None, 1) == _lib.SQ_EINVAL
    sec, n = C.c_double(), C.c_int64()
    assert lib.sq_model_gemm_time(None, C.byref(sec), C.byref(n)) == _lib.SQ_EINVAL
    assert b'null' in lib.sq_last_error()
