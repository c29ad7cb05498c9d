"""W8A8 INT8 GEMM on tcgen05 (through the C ABI) against the CPU oracle: exact INT32 accumulators and bit-exact
scale epilogues, including shapes whose K and N are not multiples of the 128-wide tiles (TMA zero fill)."""
import numpy as np
import pytest
import torch

import cases
import golden
import tcq_oracle as O
from gpu_util import n, t

pytestmark = pytest.mark.gpu


@pytest.fixture(scope='module')
def K():
    if not torch.cuda.is_available():
        pytest.skip('no CUDA device')
    from yanlongvla_b200 import kernels
    kernels.device_error(reset=True)
    yield kernels
    assert kernels.device_error(reset=True) == 0, 'a kernel pipeline wait expired'


def _rand(M, Kd, N, seed):
    r = cases.rng('i8', M, Kd, N, seed)
    q = r.integers(-127, 128, size=(M, Kd), dtype=np.int32).astype(np.int8)
    w = r.integers(-127, 128, size=(N, Kd), dtype=np.int32).astype(np.int8)
    return q, w


@pytest.mark.parametrize('M,Kd,N', [(1, 128, 128), (3, 80, 48), (17, 1152, 320), (64, 2048, 2048), (100, 4304, 1152),
                                    (160, 2048, 2048), (160, 8192, 2048), (512, 1152, 1152), (256, 2048, 6144),
                                    (300, 1536, 1536), (513, 2048, 384), (1024, 8192, 2048)])
def test_int_mm_exact(K, M, Kd, N):
    q, w = _rand(M, Kd, N, 0)
    acc = K.int_mm(t(q), t(w))
    torch.cuda.synchronize()
    ref = O.int_matmul(q, w)
    assert np.array_equal(n(acc), ref), f'{int((n(acc) != ref).sum())} mismatches'


@pytest.mark.parametrize('M,Kd,N', [(2304, 1024, 2304), (2300, 1040, 2320), (4096, 512, 4608), (1024, 256, 6144), (1000, 272, 6128)])
def test_int_mm_two_sm_tiles(K, M, Kd, N):
    """Products large enough for the two-SM 256 x 256 tiles, including M, N and K that are not tile multiples and a
    partly filled last round of SM pairs, in all three epilogues (INT32, FP32 and BF16 with the scales)."""
    q, w = _rand(M, Kd, N, 1)
    ref = O.int_matmul(q, w)
    assert np.array_equal(n(K.int_mm(t(q), t(w))), ref)
    r = np.random.default_rng(2)
    s_tok = (r.random(M).astype(np.float32) + 0.5) * 1e-2
    s_ch = (r.random(N).astype(np.float32) + 0.5) * 1e-3
    z = O.scale_acc(ref, s_tok, s_ch)
    assert np.array_equal(n(K.int8_gemm(t(q), t(w), t(s_tok), t(s_ch), out_dtype=torch.float32)), z)
    assert np.array_equal(n(K.int8_gemm(t(q), t(w), t(s_tok), t(s_ch))), O.f32_to_bf16(z))
    assert K.device_error() == 0


def test_int_mm_extremes(K):
    """All-(-127) and all-127 operands: the largest magnitudes the int8 path sees (no saturation, exact INT32)."""
    M, Kd, N = 40, 8192, 256
    q = np.full((M, Kd), -127, dtype=np.int8)
    w = np.full((N, Kd), 127, dtype=np.int8)
    w[::2] = -127
    acc = n(K.int_mm(t(q), t(w)))
    assert np.array_equal(acc, O.int_matmul(q, w))


@pytest.mark.parametrize('M,Kd,N', cases.GEMMS)
def test_int8_gemm_config3_golden(K, M, Kd, N):
    """benchmark config 3 end to end: per-token quantizer kernel + tcgen05 GEMM + scale epilogue == the reference."""
    a, w, sc = cases.gemm_inputs(M, Kd, N)
    qd, sd = K.quantize(t(a, 'bf16'))
    golden.check(f'gemm/{M}x{Kd}x{N}/q', n(qd))
    golden.check(f'gemm/{M}x{Kd}x{N}/scale', n(sd))
    q, s = O.quantize_tokens(O.bf16_to_f32(a))
    out = K.int8_gemm(t(q), t(w), t(s[:, 0].copy()), t(sc))
    golden.check(f'gemm/{M}x{Kd}x{N}/out', n(out))
    acc = K.int_mm(t(q), t(w))
    golden.check(f'gemm/{M}x{Kd}x{N}/acc', n(acc))
    z = K.int8_gemm(t(q), t(w), t(s[:, 0].copy()), t(sc), out_dtype=torch.float32)
    assert np.array_equal(n(z), O.scale_acc(O.int_matmul(q, w), s[:, 0], sc))


def test_int_mm_repeated_and_graph(K):
    """Persistent tile loop across calls, and capture into a CUDA graph."""
    M, Kd, N = 512, 2048, 2048
    q, w = _rand(M, Kd, N, 1)
    qd, wd = t(q), t(w)
    ref = O.int_matmul(q, w)
    out = torch.empty(M, N, dtype=torch.int32, device='cuda')
    for _ in range(5):
        K.int_mm(qd, wd, out=out)
    assert np.array_equal(n(out), ref)
    st = torch.cuda.Stream()
    st.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(st):
        K.int_mm(qd, wd, out=out)
    torch.cuda.current_stream().wait_stream(st)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        K.int_mm(qd, wd, out=out)
    out.zero_()
    g.replay()
    torch.cuda.synchronize()
    assert np.array_equal(n(out), ref)


@pytest.mark.parametrize('M', [1, 3, 17, 33, 64, 100, 160, 256])
@pytest.mark.parametrize('N,Kd', [(1536, 1536), (256, 4304), (2048, 2048)])
def test_gemm_tcq_tc_exact(K, M, N, Kd):
    """Trellis decode fused into the tcgen05 product: bit-exact z against the oracle, twice (workspace left clean)."""
    from gpu_util import DevLayer
    L = DevLayer(f'tc{N}x{Kd}', N, Kd, False)
    x = cases.activations(f'tc{N}x{Kd}', M, Kd, 'bf16')
    q, s = O.pre(x, 'bf16', L.ref.su)
    zr = O.gemm_z(q, L.ref.w8_reference(), s, L.ref.rs)
    z = torch.empty(M, N, dtype=torch.float32, device='cuda')
    for _ in range(2):
        z.fill_(float('nan'))
        K.gemm_tcq_tc(L.bits, L.t8, t(q), t(s), L.rs, z, Kd)
        got = n(z)
        assert np.array_equal(got, zr), f'{int((got != zr).sum())} of {zr.size} differ'


def test_gemm_tcq_tc_three_layers(K):
    """q / k / v (2048 + 512 + 512 rows) with their own tables, 160 tokens (the policy's LLM prefix)."""
    from gpu_util import DevLayer
    Ls = [DevLayer(f'tcqkv{i}', m, 2048, False) for i, m in enumerate((2048, 512, 512))]
    M = 160
    x = cases.activations('tcqkv', M, 2048, 'bf16')
    q, s = O.pre(x, 'bf16', Ls[0].ref.su)
    bits = torch.cat([L.bits for L in Ls]).contiguous()
    t8 = torch.cat([L.t8.reshape(-1) for L in Ls]).contiguous()
    rs = torch.cat([L.rs for L in Ls]).contiguous()
    z = torch.empty(M, 3072, dtype=torch.float32, device='cuda')
    K.gemm_tcq_tc(bits, t8, t(q), t(s), rs, z, 2048, bounds=(128, 160))
    zr = np.concatenate([O.gemm_z(q, L.ref.w8_reference(), s, L.ref.rs) for L in Ls], 1)
    assert np.array_equal(n(z), zr)


@pytest.mark.parametrize('M,Kd,N', [(512, 1152, 1152), (512, 1152, 4304), (512, 4304, 1152), (2048, 1152, 1152)])
def test_int8_gemm_vision_shapes(K, M, Kd, N):
    """The vision tower's W8A8 products (BF16 scaled epilogue) at the policy's token counts."""
    r = cases.rng('vit', M, Kd, N)
    a = (r.standard_normal((M, Kd)) * 2).astype(np.float32)
    w = r.integers(-127, 128, size=(N, Kd), dtype=np.int32).astype(np.int8)
    sc = r.uniform(1e-4, 1e-3, N).astype(np.float32)
    q, s = O.quantize_tokens(a)
    out = K.int8_gemm(t(q), t(w), t(s[:, 0].copy()), t(sc))
    assert np.array_equal(n(out), O.int8_gemm_scaled(q, w, s[:, 0], sc))


@pytest.mark.parametrize('act', [None, 'gelu'])
@pytest.mark.parametrize('M,Kd,N', [(7, 1152, 1152), (40, 1152, 4304), (512, 1152, 4304), (2048, 1152, 1152)])
def test_int8_gemm_bias_act_equals_torch_ops(K, M, Kd, N, act):
    """The vision Linear's epilogue: act(BF16(BF16(z) + bias)) in the GEMM equals int8_gemm, then the PyTorch BF16
    bias add, then the PyTorch activation, bit for bit (small-M tiles, split tiles and the two-SM path)."""
    r = cases.rng('vitb', M, Kd, N)
    a = (r.standard_normal((M, Kd)) * 2).astype(np.float32)
    w = r.integers(-127, 128, size=(N, Kd), dtype=np.int32).astype(np.int8)
    sc = r.uniform(1e-4, 1e-3, N).astype(np.float32)
    q, s = O.quantize_tokens(a)
    bias = torch.from_numpy((r.standard_normal(N) * 0.5).astype(np.float32)).cuda().bfloat16()
    want = K.int8_gemm(t(q), t(w), t(s[:, 0].copy()), t(sc)) + bias
    if act == 'gelu':
        want = torch.nn.functional.gelu(want, approximate='tanh')
    got = K.int8_gemm_bias(t(q), t(w), t(s[:, 0].copy()), t(sc), bias=bias, act=act)
    assert torch.equal(got, want)
    plain = K.int8_gemm_bias(t(q), t(w), t(s[:, 0].copy()), t(sc))
    assert torch.equal(plain, K.int8_gemm(t(q), t(w), t(s[:, 0].copy()), t(sc)))


def test_bounded_wait_expires_and_reports(K):
    """The failure path of the bounded waits, without a fault: a wait on a barrier nothing arrives at gives up after
    10 ms and raises the device error flag; the flag clears and the context keeps working."""
    assert K.device_error(reset=True) == 0
    assert K.selftest_wait_expiry(10000) == 1
    assert K.device_error() == 0
    q, w = _rand(64, 256, 128, 5)
    assert np.array_equal(n(K.int_mm(t(q), t(w))), O.int_matmul(q, w))
