"""Parity of the sm_100a kernels (through the C ABI) with the CPU oracle, bit for bit, and with the reference's golden
outputs. Requires a B200."""
import numpy as np
import pytest
import torch

import cases
import golden
import tcq_oracle as O
from gpu_util import DevLayer, n, t, x_dev

pytestmark = pytest.mark.gpu

K_ = None


@pytest.fixture(scope='module')
def K():
    if not torch.cuda.is_available():
        pytest.skip('no CUDA device')
    from yanlongvla_b200 import kernels
    return kernels


LAYERS = [c for c in cases.LAYERS]


def _eq(a, b, what):
    a, b = np.asarray(a), np.asarray(b)
    assert a.shape == b.shape, (what, a.shape, b.shape)
    bad = np.flatnonzero(a.reshape(-1) != b.reshape(-1))
    assert bad.size == 0, f'{what}: {bad.size} of {a.size} differ, first {bad[:8]}'


@pytest.mark.parametrize('spec', LAYERS, ids=[c[0] for c in LAYERS])
def test_decode(K, spec):
    name, m, nn, _, _, b = spec
    L = DevLayer(name, m, nn, b)
    out = torch.empty(m, nn, dtype=torch.int8, device='cuda')
    K.decode(L.bits, L.t8, out)
    w8 = n(out)
    golden.check(f'{name}/w8', w8)
    tb = t(O.decode_bf16_table(L.ref.t8).reshape(512, 2), 'bf16')
    ob = torch.empty(m, nn, dtype=torch.bfloat16, device='cuda')
    K.decode_bf16(L.bits, tb, ob)
    _eq(n(ob), O.decode_bf16(L.ref), 'decode_bf16')


@pytest.mark.parametrize('spec', LAYERS, ids=[c[0] for c in LAYERS])
def test_pre_post_linear(K, spec):
    """pre -> INT8 product (oracle) -> post reproduces reference_linear (golden y), resident and fused paths."""
    name, m, nn, tokens, dt, b = spec
    L = DevLayer(name, m, nn, b)
    w8 = L.ref.w8_reference()
    for M in tokens:
        x = cases.activations(name, M, nn, dt)
        xd = x_dev(x, dt)
        q = torch.empty(M, nn, dtype=torch.int8, device='cuda')
        q4 = torch.empty(nn // 4, M, dtype=torch.int32, device='cuda')
        s = torch.empty(M, dtype=torch.float32, device='cuda')
        K.pre(xd, L.su, q=q, q4=q4, scale=s)
        golden.check(f'{name}/M{M}/q', n(q))
        golden.check(f'{name}/M{M}/scale', n(s))
        _eq(n(q4), O.q4_words(n(q)), 'q4')
        acc = O.int_matmul(n(q), w8)
        y = torch.empty(M, m, dtype=torch.bfloat16, device='cuda')
        K.post(t(acc), s, L.rs, L.sv, L.bias, y)
        golden.check(f'{name}/M{M}/y', n(y))
        if M <= 16:
            z = torch.empty(M, m, dtype=torch.float32, device='cuda')
            K.gemm_tcq(L.bits, L.t8, q4, s, L.rs, z, nn)
            golden.check(f'{name}/M{M}/z', n(z))
            y2 = torch.empty_like(y)
            K.post(z, None, None, L.sv, L.bias, y2)
            golden.check(f'{name}/M{M}/y', n(y2))
            if m * nn <= 1536 * 1536:
                W = torch.empty(m, nn, dtype=torch.int8, device='cuda')
                K.decode(L.bits, L.t8, W)
                z3 = torch.empty_like(z)
                K.gemm_w8(W, q4, s, L.rs, z3)
                golden.check(f'{name}/M{M}/z', n(z3))


@pytest.mark.parametrize('M', list(range(1, 17)))
def test_gemm_tcq_every_m(K, M):
    """Every token count 1..16 (the templates pad to 1, 2, 4, 8, 16), odd widths, bit-exact z."""
    L = DevLayer('odd', 48, 80, False)
    x = cases.activations('gemm_m', M, 80, 'bf16')
    q, s = O.pre(x, 'bf16', L.ref.su)
    zr = O.gemm_z(q, L.ref.w8_reference(), s, L.ref.rs)
    z = torch.empty(M, 48, dtype=torch.float32, device='cuda')
    K.gemm_tcq(L.bits, L.t8, t(O.q4_words(q)), t(s), L.rs, z, 80)
    _eq(n(z), zr, f'gemm_tcq M={M}')
    W = torch.empty(48, 80, dtype=torch.int8, device='cuda')
    K.decode(L.bits, L.t8, W)
    z2 = torch.empty_like(z)
    K.gemm_w8(W, t(O.q4_words(q)), t(s), L.rs, z2)
    _eq(n(z2), zr, f'gemm_w8 M={M}')


@pytest.mark.parametrize('M,N,Kd', [(1, 4096, 4096), (3, 2048, 8192), (10, 1536, 6144), (16, 512, 16384), (2, 6144, 1152),
                                    (1, 4112, 4080), (1, 2048, 8192), (1, 8192, 2048)])
def test_gemm_tcq_shapes(K, M, N, Kd):
    """Stream-K split across warps / CTAs at policy shapes; repeated calls keep the workspace clean."""
    L = DevLayer(f'shape{N}x{Kd}', N, Kd, False)
    x = cases.activations(f'shape{N}x{Kd}', M, Kd, 'bf16')
    q, s = O.pre(x, 'bf16', L.ref.su)
    zr = O.gemm_z(q, L.ref.w8_reference(), s, L.ref.rs)
    z = torch.empty(M, N, dtype=torch.float32, device='cuda')
    for _ in range(3):
        z.zero_()
        K.gemm_tcq(L.bits, L.t8, t(O.q4_words(q)), t(s), L.rs, z, Kd)
        _eq(n(z), zr, f'gemm_tcq {M}x{N}x{Kd}')


def test_gemm_tcq_one_token_unaligned_activations(K):
    """M = 1 with activation words that do not start on a 16-byte boundary (scalar activation loads), on a layer large
    enough for one lane per tile whose last unit of each tile row is partial (4112 x 4080)."""
    L = DevLayer('g1u4112x4080', 4112, 4080, False)
    x = cases.activations('g1u4112x4080', 1, 4080, 'bf16')
    q, s = O.pre(x, 'bf16', L.ref.su)
    zr = O.gemm_z(q, L.ref.w8_reference(), s, L.ref.rs)
    words = t(O.q4_words(q))
    buf = torch.zeros(words.numel() + 1, dtype=torch.int32, device='cuda')
    buf[1:] = words.reshape(-1)
    q4 = buf[1:].view(words.shape)
    assert q4.data_ptr() % 16 != 0
    z = torch.empty(1, 4112, dtype=torch.float32, device='cuda')
    K.gemm_tcq(L.bits, L.t8, q4, t(s), L.rs, z, 4080)
    _eq(n(z), zr, 'gemm_tcq one token, unaligned activations')


@pytest.mark.parametrize('M,N,Kd,dt', [(1, 4096, 4096, 'bf16'), (1, 512, 1152, 'f16'), (2, 2048, 8192, 'f32'),
                                       (3, 1536, 1536, 'bf16'), (4, 6144, 1152, 'bf16'), (1, 8192, 8192, 'bf16'),
                                       (4, 48, 80, 'f32'), (1, 2048, 1024, 'f16'), (1, 1536, 2048, 'f32'),
                                       (1, 4112, 4096, 'bf16'), (2, 4096, 4096, 'f16')])
def test_gemm_tcq_x_fused_pre(K, M, N, Kd, dt):
    """pre fused into the decode-GEMV (tcq_gemm_tcq_x): z equals the oracle's pre + product bit for bit."""
    L = DevLayer(f'gx{N}x{Kd}', N, Kd, False)
    x = cases.activations(f'gx{N}x{Kd}', M, Kd, dt)
    q, s = O.pre(x, dt, L.ref.su)
    zr = O.gemm_z(q, L.ref.w8_reference(), s, L.ref.rs)
    z = torch.empty(M, N, dtype=torch.float32, device='cuda')
    for _ in range(2):
        z.zero_()
        K.gemm_tcq_x(L.bits, L.t8, x_dev(x, dt), L.su, L.rs, z, Kd)
        _eq(n(z), zr, f'gemm_tcq_x {M}x{N}x{Kd} {dt}')


def test_gemm_tcq_x_three_layers_and_limits(K):
    Ls = [DevLayer(f'gxq{i}', m, 1152, False) for i, m in enumerate((128, 64, 64))]
    M = 4
    x = cases.activations('gxqkv', M, 1152, 'bf16')
    q, s = O.pre(x, 'bf16', Ls[0].ref.su)
    bits = torch.cat([L.bits for L in Ls]).contiguous()
    t8 = torch.cat([L.t8.reshape(-1) for L in Ls]).contiguous()
    rs = torch.cat([L.rs for L in Ls]).contiguous()
    z = torch.empty(M, 256, dtype=torch.float32, device='cuda')
    K.gemm_tcq_x(bits, t8, x_dev(x, 'bf16'), Ls[0].su, rs, z, 1152, bounds=(128 // 16, 192 // 16))
    zr = np.concatenate([O.gemm_z(q, L.ref.w8_reference(), s, L.ref.rs) for L in Ls], 1)
    _eq(n(z), zr, 'gemm_tcq_x qkv')
    with pytest.raises(K.TcqError):                 # more than 4 tokens: not this entry point
        K.gemm_tcq_x(Ls[0].bits, Ls[0].t8, torch.zeros(5, 1152, device='cuda').bfloat16(), Ls[0].su, Ls[0].rs,
                     torch.empty(5, 128, device='cuda'), 1152)


def test_gemm_tcq_three_layers(K):
    """q / k / v concatenated along the rows with their own tables (bounds in tile rows)."""
    Ls = [DevLayer(f'qkv{i}', m, 1152, False) for i, m in enumerate((128, 64, 64))]
    M = 5
    x = cases.activations('qkv', M, 1152, 'bf16')
    q, s = O.pre(x, 'bf16', Ls[0].ref.su)
    bits = torch.cat([L.bits for L in Ls]).contiguous()
    t8 = torch.cat([L.t8.reshape(-1) for L in Ls]).contiguous()
    rs = torch.cat([L.rs for L in Ls]).contiguous()
    z = torch.empty(M, 256, dtype=torch.float32, device='cuda')
    K.gemm_tcq(bits, t8, t(O.q4_words(q)), t(s), rs, z, 1152, bounds=(128 // 16, 192 // 16))
    zr = np.concatenate([O.gemm_z(q, L.ref.w8_reference(), s, L.ref.rs) for L in Ls], 1)
    _eq(n(z), zr, 'gemm_tcq qkv')


@pytest.mark.parametrize('T,D', cases.ROTATIONS)
def test_rotate(K, T, D):
    x, sg = cases.rotation_input(T, D)
    y = K.rotate(t(x, 'bf16'), t(sg))
    golden.check(f'rot/{T}x{D}/fwd', n(y))
    back = K.rotate(y, t(sg), inverse=True)
    golden.check(f'rot/{T}x{D}/inv', n(back))
    yb = K.rotate(t(x, 'bf16'), t(sg), out_dtype=torch.bfloat16)
    _eq(n(yb), O.f32_to_bf16(O.rotate(x, sg, 'bf16')), 'rotate bf16 out')


def test_bf16_rounding_special_values(K):
    """BF16 outputs follow the reference's scalar rounding for every FP32 input class: overflow to infinity,
    infinities, NaN (-> 0x7fc0, whatever NaN the arithmetic produced), subnormals and signed zeros."""
    D = 64
    sg = np.where(cases.rng('special.sg', D).random(D) < 0.5, -1, 1).astype(np.int8)
    x = cases.rng('special.x', D).standard_normal((6, D)).astype(np.float32)
    x[1, 5] = np.nan
    x[2, 7] = np.inf
    x[3, :] = 3.0e38                                   # butterflies overflow to +-inf, inf - inf gives NaN
    x[4, :] *= np.float32(1e-39)                       # subnormal sums and outputs
    x[5, :] = 0.0
    x[5, ::3] = -0.0
    for inverse in (False, True):
        y = K.rotate(t(x), t(sg), inverse=inverse, out_dtype=torch.bfloat16)
        with np.errstate(all='ignore'):
            want = O.f32_to_bf16(O.rotate(x, sg, 'f32', inverse=inverse))
        _eq(n(y), want, f'rotate bf16 special values (inverse={inverse})')


@pytest.mark.parametrize('dt', ['bf16', 'f16', 'f32'])
@pytest.mark.parametrize('Kd', [16, 48, 1152, 1536, 2048, 4304, 6144, 12288, 16384])
def test_pre_dtypes_and_widths(K, dt, Kd):
    M = 6
    x = cases.activations(f'pre{Kd}', M, Kd, dt)
    su = np.where(cases.rng('su', Kd).random(Kd) < 0.5, -1, 1).astype(np.int8)
    qr, sr = O.pre(x, dt, su)
    q = torch.empty(M, Kd, dtype=torch.int8, device='cuda')
    s = torch.empty(M, dtype=torch.float32, device='cuda')
    K.pre(x_dev(x, dt), t(su), q=q, scale=s)
    _eq(n(q), qr, 'q')
    _eq(n(s), sr, 'scale')
    h = torch.empty(M, Kd, dtype=torch.bfloat16, device='cuda')
    hT = torch.empty(Kd, M, dtype=torch.bfloat16, device='cuda')
    K.pre_h(x_dev(x, dt), t(su), h=h, hT=hT)
    hr = O.pre_h(x, dt, su)
    _eq(n(h), hr, 'pre_h h')
    _eq(n(hT), np.ascontiguousarray(hr.T), 'pre_h hT')


@pytest.mark.parametrize('acc_dt', ['i32', 'f32', 'bf16'])
@pytest.mark.parametrize('N', [16, 80, 1536, 2048, 4304, 6144, 16384])
def test_post_acc_types(K, acc_dt, N):
    M = 3
    r = cases.rng('post', N, acc_dt)
    sv = np.where(r.random(N) < 0.5, -1, 1).astype(np.int8)
    rs = r.uniform(1e-5, 1e-4, N).astype(np.float32)
    s = r.uniform(0.01, 0.1, M).astype(np.float32)
    bias = (r.standard_normal(N) * 0.1).astype(np.float32)
    col0 = 16
    lda = N + 32
    if acc_dt == 'i32':
        acc = r.integers(-2 ** 22, 2 ** 22, size=(M, lda), dtype=np.int64).astype(np.int32)
        accd = t(acc)
    elif acc_dt == 'f32':
        acc = r.standard_normal((M, lda)).astype(np.float32)
        accd = t(acc)
    else:
        acc = cases.f32_to_bf16_bits(r.standard_normal((M, lda)).astype(np.float32) * 100)
        accd = t(acc, 'bf16')
    yr = O.post_acc(acc[:, col0:col0 + N], acc_dt, s, rs, sv, bias)
    y = torch.empty(M, N, dtype=torch.bfloat16, device='cuda')
    K.post(accd, t(s), t(rs), t(sv), t(bias), y, col0=col0)
    _eq(n(y), yr, f'post {acc_dt}')


def _mlp_inputs(M, N, seed):
    r = cases.rng('mlp', M, N, seed)
    acc = r.integers(-2 ** 20, 2 ** 20, size=(M, 2 * N), dtype=np.int64).astype(np.int32)
    s = r.uniform(0.5, 1.5, M).astype(np.float32)
    rs = (r.uniform(1e-6, 3e-6, 2 * N)).astype(np.float32)
    sv = np.where(r.random(2 * N) < 0.5, -1, 1).astype(np.int8)
    su = np.where(r.random(N) < 0.5, -1, 1).astype(np.int8)
    bias = (r.standard_normal(2 * N) * 0.1).astype(np.float32)
    return acc, s, rs, sv, su, bias


@pytest.mark.parametrize('act', ['gelu', 'silu'])
@pytest.mark.parametrize('M,N', [(10, 4096), (3, 4304), (17, 1536), (2, 16384), (5, 8192), (2, 12288), (160, 8192), (17, 6144),
                                 (1, 3072), (400, 2048)])
def test_mlp_middles(K, act, M, N):
    acc, s, rs, sv, su, bias = _mlp_inputs(M, N, 0)
    lut = n(K.act_table(act))
    z = O.scale_acc(acc, s, rs)
    # gated middle, fused and split (postg + pre2)
    qr, sr = O.mid2(z, sv, lut, su)
    q = torch.empty(M, N, dtype=torch.int8, device='cuda')
    sc = torch.empty(M, dtype=torch.float32, device='cuda')
    K.mid2(t(acc), t(s), t(rs), t(sv), t(su), q=q, scale=sc, act=act)
    _eq(n(q), qr, 'mid2 q')
    _eq(n(sc), sr, 'mid2 scale')
    g = torch.empty(M, N, dtype=torch.bfloat16, device='cuda')
    u = torch.empty_like(g)
    K.postg(t(z), None, None, t(sv), None, [g, u], gelu0=True, act=act)
    gr, ur = O.postg(z, sv, None, [N, N], lut, act0=True)
    _eq(n(g), gr, 'postg g')
    _eq(n(u), ur, 'postg u')
    q2 = torch.empty_like(q)
    sc2 = torch.empty_like(sc)
    q42 = torch.empty(N // 4, M, dtype=torch.int32, device='cuda')
    K.pre2(g, u, t(su), q=q2, q4=q42, scale=sc2)
    _eq(n(q2), qr, 'pre2 q')
    _eq(n(sc2), sr, 'pre2 scale')
    _eq(n(q42), O.q4_words(qr), 'pre2 q4')
    # plain middle
    q1r, s1r = O.mid1(z[:, :N], sv[:N], bias[:N], lut, su)
    q1 = torch.empty(M, N, dtype=torch.int8, device='cuda')
    s1 = torch.empty(M, dtype=torch.float32, device='cuda')
    K.mid1(t(np.ascontiguousarray(acc[:, :N])), t(s), t(rs[:N].copy()), t(sv[:N].copy()), t(bias[:N].copy()), t(su), q=q1, scale=s1,
           act=act)
    _eq(n(q1), q1r, 'mid1 q')
    _eq(n(s1), s1r, 'mid1 scale')


@pytest.mark.parametrize('M', [1, 7, 33])
def test_post3(K, M):
    ns = (2048, 512, 512)
    r = cases.rng('post3', M)
    Nt = sum(ns)
    acc = r.integers(-2 ** 22, 2 ** 22, size=(M, Nt), dtype=np.int64).astype(np.int32)
    s = r.uniform(0.01, 0.1, M).astype(np.float32)
    rs = r.uniform(1e-5, 1e-4, Nt).astype(np.float32)
    sv = np.where(r.random(Nt) < 0.5, -1, 1).astype(np.int8)
    bias = (r.standard_normal(Nt) * 0.1).astype(np.float32)
    ys = [torch.empty(M, k, dtype=torch.bfloat16, device='cuda') for k in ns]
    K.post3(t(acc), t(s), t(rs), t(sv), t(bias), ys)
    z = O.scale_acc(acc, s, rs)
    for y, yr in zip(ys, O.postg(z, sv, bias, list(ns))):
        _eq(n(y), yr, 'post3')
    ys2 = [torch.empty_like(y) for y in ys]
    K.postg(t(acc), t(s), t(rs), t(sv), t(bias), ys2)
    for y, y2 in zip(ys, ys2):
        _eq(n(y2), n(y), 'postg == post3')


def test_config1_fused_linear(K):
    """benchmark config 1: 4096 x 4096 layer, x fp16 [1, 4096]: pre -> fused decode-GEMV -> post == reference y."""
    L = DevLayer('config1', 4096, 4096, False)
    x = cases.activations('config1', 1, 4096, 'f16')
    q4 = torch.empty(1024, 1, dtype=torch.int32, device='cuda')
    s = torch.empty(1, dtype=torch.float32, device='cuda')
    K.pre(t(x), L.su, q4=q4, scale=s)
    z = torch.empty(1, 4096, dtype=torch.float32, device='cuda')
    K.gemm_tcq(L.bits, L.t8, q4, s, L.rs, z, 4096)
    y = torch.empty(1, 4096, dtype=torch.bfloat16, device='cuda')
    K.post(z, None, None, L.sv, None, y)
    golden.check('config1/M1/z', n(z))
    golden.check('config1/M1/y', n(y))


def test_graph_capture(K):
    """The whole small-M chain replays from a CUDA graph with identical results."""
    L = DevLayer('dit', 1536, 1536, False)
    M = 10
    x = t(cases.activations('dit', M, 1536, 'bf16'), 'bf16')
    q4 = torch.empty(384, M, dtype=torch.int32, device='cuda')
    s = torch.empty(M, dtype=torch.float32, device='cuda')
    z = torch.empty(M, 1536, dtype=torch.float32, device='cuda')
    y = torch.empty(M, 1536, dtype=torch.bfloat16, device='cuda')

    def chain():
        K.pre(x, L.su, q4=q4, scale=s)
        K.gemm_tcq(L.bits, L.t8, q4, s, L.rs, z, 1536)
        K.post(z, None, None, L.sv, None, y)

    chain()
    torch.cuda.synchronize()
    ref = n(y).copy()
    st = torch.cuda.Stream()
    st.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(st):
        chain()
    torch.cuda.current_stream().wait_stream(st)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        chain()
    y.zero_()
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    _eq(n(y), ref, 'graph replay')
    golden.check(f'dit/M{M}/y', n(y))


def test_quantizer_ties_and_tiny_scales(K):
    """The per-token quantizer at its edge cases (the division-free path falls back to the IEEE quotient near
    half-integers): exact halves with s = 1, quotients a rounding away from halves, a denormal scale whose reciprocal
    overflows, and an all-zero row; against the oracle's true division."""
    Kd = 256
    x = np.zeros((6, Kd), dtype=np.float32)
    x[0, :-1] = np.arange(-127, 128, dtype=np.float32)[:Kd - 1] + 0.5
    x[0, -1] = 127.0                                           # amax 127: s = 1, every quotient an exact half
    s1 = np.float32(0.0123)
    x[1, :-1] = ((np.arange(Kd - 1, dtype=np.float32) - 127.0) + np.float32(0.5)) * s1
    x[1, -1] = np.float32(127.0) * s1
    r = np.random.default_rng(3)
    x[2] = r.standard_normal(Kd).astype(np.float32) * 7
    x[3] = r.standard_normal(Kd).astype(np.float32) * np.float32(1e-40)   # denormal amax: 1/s overflows
    # quotients one to four ulps either side of a half-integer (inside and just outside the guard band)
    s5 = np.float32(0.0371)
    halves = ((np.arange(Kd - 1) % 254) - 127 + 0.5).astype(np.float32) * s5
    steps = (np.arange(Kd - 1) % 9 - 4).astype(np.int32)
    x[5, :-1] = (halves.view(np.int32) + steps).view(np.float32)
    x[5, -1] = np.float32(127.0) * s5
    qd, sd = K.quantize(t(x))
    qo, so = O.quantize_tokens(x)
    assert np.array_equal(n(qd), qo) and np.array_equal(n(sd), so[:, 0])
