"""ctypes binding of the C ABI (include/tcq_b200.h) in libtcq_b200.so.

The library is built in-tree by `python -m yanlongvla_b200.build`. There is no fallback: if the library is missing
or does not load, importing this module raises, so nothing can silently run another implementation.
"""
import ctypes
import os
from pathlib import Path

_PKG = Path(__file__).resolve().parent
LIB_PATH = Path(os.environ.get('TCQ_B200_LIB', _PKG / 'libtcq_b200.so'))

P = ctypes.c_void_p
I = ctypes.c_int
SZ = ctypes.c_size_t
F = ctypes.c_float

# name -> argument types (every function returns int, except where noted)
SIGNATURES = {
    'tcq_abi_version': [],
    'tcq_status_string': [I],
    'tcq_quantize': [P, I, P, P, I, I, P],
    'tcq_pre': [P, I, P, P, P, P, I, I, I, P],
    'tcq_pre2': [P, P, P, P, P, P, I, I, I, P],
    'tcq_pre_h': [P, I, P, P, P, I, I, I, P],
    'tcq_post': [P, I, P, P, P, P, P, I, I, I, I, P],
    'tcq_post3': [P, I, P, P, P, P, P, P, P, I, I, I, I, I, P],
    'tcq_postg': [P, I, P, P, P, P, P, P, P, P, I, I, I, I, I, I, P],
    'tcq_mid2': [P, I, P, P, P, P, P, P, P, P, I, I, I, I, P],
    'tcq_mid1': [P, I, P, P, P, P, P, P, P, P, P, I, I, I, I, P],
    'tcq_rotate': [P, I, P, P, I, I, I, I, P],
    'tcq_decode': [P, P, P, I, I, P],
    'tcq_decode_bf16': [P, P, P, I, I, P],
    'tcq_gemm_w8': [P, P, P, P, P, I, I, I, P],
    'tcq_gemm_tcq_workspace': [I, I],
    'tcq_gemm_tcq': [P, P, P, P, P, P, I, I, I, I, I, P, SZ, P],
    'tcq_gemm_tcq_x': [P, P, P, I, P, P, P, I, I, I, I, I, P, SZ, P],
    'tcq_gemm_tcq_noalloc': [P, P, P, P, P, P, I, I, I, I, I, P],
    'tcq_gemm_tcq_noalloc_max_elements': [],
    'tcq_gemm_tcq_tc_workspace': [I, I],
    'tcq_gemm_tcq_tc': [P, P, P, P, P, P, I, I, I, I, I, P, SZ, P],
    'tcq_int_mm': [P, P, P, I, I, I, P],
    'tcq_int8_gemm': [P, P, P, P, P, I, I, I, I, P],
    'tcq_int8_gemm_bias': [P, P, P, P, P, P, P, I, I, I, P],
    'tcq_gemmf_tcq': [P, P, P, P, P, I, I, I, I, I, I, P],
    'tcq_gemmf_w8': [P, P, P, P, I, I, I, I, P],
    'tcq_add_norm': [P, P, P, P, P, P, I, P, P, I, I, F, I, I, I, P],
    'tcq_rope': [P, P, P, P, I, I, I, I, I, I, P],
    'tcq_chain': [P, I, P, P, P, P, I, I, P, P, P, P, P, P, I, P, P, I, I, F, I, P, P, P, P, I, I, I, P],
    'tcq_selftest_wait_expiry': [ctypes.c_uint, P],
    'tcq_device_error': [I],
}
RESTYPES = {'tcq_status_string': ctypes.c_char_p, 'tcq_gemm_tcq_workspace': SZ, 'tcq_gemm_tcq_tc_workspace': SZ, 'tcq_gemm_tcq_noalloc_max_elements': SZ}


def _load():
    if not LIB_PATH.exists():
        raise ImportError(f'{LIB_PATH} is missing: build it with `python -m yanlongvla_b200.build` (nvcc, sm_100a)')
    lib = ctypes.CDLL(str(LIB_PATH))
    for name, args in SIGNATURES.items():
        f = getattr(lib, name)
        f.argtypes = args
        f.restype = RESTYPES.get(name, ctypes.c_int)
    return lib


lib = _load()

DT_BF16, DT_F32, DT_F16, DT_I32 = 0, 1, 2, 3


class TcqError(RuntimeError):
    pass


def check(status, what):
    if status != 0:
        raise TcqError(f'{what}: {lib.tcq_status_string(status).decode()} (status {status})')
