"""The C-ABI library without a GPU: it loads, exports every function include/tcq_b200.h declares, and rejects bad
arguments on the host before touching the device."""
import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / 'include' / 'tcq_b200.h'


def declared():
    src = HEADER.read_text()
    src = re.sub(r'/\*.*?\*/', '', src, flags=re.S)
    return sorted(set(re.findall(r'^\s*(?:int|size_t|const char\*)\s+(tcq_\w+)\s*\(', src, flags=re.M)))


@pytest.fixture(scope='module')
def L():
    from yanlongvla_b200 import _lib
    return _lib


def test_header_parses():
    names = declared()
    assert 'tcq_pre' in names and 'tcq_gemm_tcq' in names and len(names) >= 15


def test_every_declared_symbol_is_exported(L):
    for name in declared():
        assert hasattr(L.lib, name), name
        assert name in L.SIGNATURES, f'{name} has no ctypes signature in _lib.py'


def test_version_and_status_strings(L):
    assert L.lib.tcq_abi_version() == 1
    assert L.lib.tcq_status_string(0) == b'ok'
    for s in range(1, 8):
        assert L.lib.tcq_status_string(s) not in (b'ok', b'unknown status')


def test_workspace_query(L):
    assert L.lib.tcq_gemm_tcq_workspace(1, 4096) == (4096 + 256) * 4
    assert L.lib.tcq_gemm_tcq_workspace(0, 16) == 0


# Fake, 256-byte aligned "device" addresses: every call below must fail validation before any CUDA call.
A = 1 << 20
B = 2 << 20
C = 3 << 20
D = 4 << 20


@pytest.mark.parametrize('K,expect', [(17, 1), (0, 1), (16400, 1), (32768, 1)])
def test_pre_rejects_widths(L, K, expect):
    assert L.lib.tcq_pre(A, L.DT_BF16, B, C, None, D, 4, K, 0, None) == expect


def test_pre_rejects_args(L):
    assert L.lib.tcq_pre(None, L.DT_BF16, B, C, None, D, 4, 64, 0, None) == 4          # x NULL
    assert L.lib.tcq_pre(A, L.DT_BF16, B, None, None, D, 4, 64, 0, None) == 4          # no output
    assert L.lib.tcq_pre(A, L.DT_BF16, B, None, C, D, 4, 64, 2, None) == 4             # ldq < M
    assert L.lib.tcq_pre(A + 2, L.DT_BF16, B, C, None, D, 4, 64, 0, None) == 2         # misaligned x
    assert L.lib.tcq_pre(A, 9, B, C, None, D, 4, 64, 0, None) == 3                     # unknown dtype


def test_post_rejects(L):
    assert L.lib.tcq_post(A, L.DT_I32, None, C, D, None, B, 2, 64, 64, 0, None) == 4   # I32 needs s, rs
    assert L.lib.tcq_post(A, L.DT_I32, B, C, D, None, B, 2, 64, 32, 0, None) == 1      # lda < col0 + N
    assert L.lib.tcq_post(A, L.DT_I32, B, C, D, None, B, 2, 64, 66, 2, None) == 2      # col0 breaks 16-byte loads


def test_trellis_rejects(L):
    assert L.lib.tcq_decode(A, B, C, 20, 32, None) == 1
    assert L.lib.tcq_gemm_tcq(A, B, C, D, A, B, 17, 64, 64, 1 << 30, 1 << 30, C, 1 << 20, None) == 1   # M > 16
    assert L.lib.tcq_gemm_tcq(A, B, C, D, A, B, 1, 64, 64, 1 << 30, 1 << 30, None, 0, None) == 7      # workspace
    assert L.lib.tcq_gemm_tcq(A, B, C, D, A, B, 1, 64, 64, 1 << 30, 1 << 30, C, 8, None) == 7         # too small
    assert L.lib.tcq_gemm_w8(A, B, C, D, A, 1, 64, 20, None) == 1


def test_python_wrapper_raises(L):
    assert issubclass(L.TcqError, RuntimeError)
    with pytest.raises(L.TcqError, match='unsupported shape'):
        L.check(L.lib.tcq_decode(A, B, C, 20, 32, None), 'tcq_decode')
