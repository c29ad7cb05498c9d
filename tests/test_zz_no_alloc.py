"""The no-allocation fused decode-GEMV (tcq_gemm_tcq_noalloc) against the workspace entry point (tcq_gemm_tcq).

tcq_gemm_tcq_noalloc serves callers that cannot allocate device memory themselves, such as a real-time control loop
(cudaMalloc may synchronize the device at an arbitrary moment) or a plugin host that owns every device buffer. It
takes the same inputs and outputs as tcq_gemm_tcq and keeps its scratch in a fixed array inside the library. Both
entry points are called here through the C ABI; their FP32 outputs must agree bit for bit (the tolerance of every
other decode-GEMV test), on two calls in a row, so that the shared scratch is shown to be left clean.

This file is named to be collected last: if it fails, every other test has already run.
"""
import ctypes

import numpy as np
import pytest
import torch

import cases
import tcq_oracle as O

pytestmark = pytest.mark.gpu


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr())


@pytest.fixture(scope='module')
def lib():
    if not torch.cuda.is_available():
        pytest.skip('no CUDA device')
    from yanlongvla_b200 import _lib
    return _lib


# (16, 32768, 256) fills the scratch array exactly: M * N partial sums plus N / 16 arrival counters end at its last
# element.
@pytest.mark.parametrize('M,N,K', [(1, 4096, 4096), (5, 1536, 1152), (16, 2048, 2048), (16, 32768, 256)])
def test_noalloc_matches_workspace_entry(lib, M, N, K):
    dev = torch.device('cuda')
    tens, _ = cases.layer_tensors(f'noalloc{N}x{K}', N, K)
    ref = O.Layer(tens['bits'], tens['tlut'], tens['row_scale'], tens['su'], tens['sv'])
    x = cases.activations(f'noalloc{N}x{K}', M, K, 'bf16')
    q, s = O.pre(x, 'bf16', ref.su)
    bits = torch.from_numpy(tens['bits'].view(np.int16).copy()).to(dev)
    t8 = torch.from_numpy(ref.t8).to(dev)
    rs = torch.from_numpy(ref.rs).to(dev)
    q4 = torch.from_numpy(O.q4_words(q)).to(dev)
    sd = torch.from_numpy(s).to(dev)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    big = 1 << 30

    ws_bytes = int(lib.lib.tcq_gemm_tcq_workspace(M, N))
    ws = torch.zeros(ws_bytes // 4 + 1, dtype=torch.int32, device=dev)      # the test allocates; the entry point does not
    z_ws = torch.full((M, N), float('nan'), dtype=torch.float32, device=dev)
    lib.check(lib.lib.tcq_gemm_tcq(_ptr(bits), _ptr(t8), _ptr(q4), _ptr(sd), _ptr(rs), _ptr(z_ws), M, N, K, big, big, _ptr(ws),
                                   ws.numel() * 4, stream), 'tcq_gemm_tcq')
    expect = z_ws.cpu().numpy()
    for call in range(2):
        z = torch.full((M, N), float('nan'), dtype=torch.float32, device=dev)
        lib.check(lib.lib.tcq_gemm_tcq_noalloc(_ptr(bits), _ptr(t8), _ptr(q4), _ptr(sd), _ptr(rs), _ptr(z), M, N, K, big, big, stream),
                  'tcq_gemm_tcq_noalloc')
        torch.cuda.synchronize()
        got = z.cpu().numpy()
        assert np.array_equal(got.view(np.uint32), expect.view(np.uint32)), f'call {call}: {int((got != expect).sum())} outputs differ'
    assert np.array_equal(expect, O.gemm_z(q, ref.w8_reference(), s, ref.rs))


def test_noalloc_rejects_oversize(lib):
    limit = int(lib.lib.tcq_gemm_tcq_noalloc_max_elements())
    assert limit == 16 * 32768
    a = ctypes.c_void_p(1 << 20)
    assert lib.lib.tcq_gemm_tcq_noalloc(a, a, a, a, a, a, 16, 65536, 64, 1 << 30, 1 << 30, None) == 1      # N too large
    assert lib.lib.tcq_gemm_tcq_noalloc(a, a, a, a, a, a, 1, 32768 + 16, 64, 1 << 30, 1 << 30, None) == 1  # one tile row past the limit
    assert lib.lib.tcq_gemm_tcq_noalloc(a, a, a, a, a, a, 17, 1024, 64, 1 << 30, 1 << 30, None) == 1       # M > 16
