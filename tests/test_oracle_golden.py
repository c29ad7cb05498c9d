"""The CPU oracle against the reference's own outputs (golden fixtures), bit for bit. No GPU."""
import numpy as np
import pytest

import cases
import golden
import tcq_oracle as O


def _layer(name, m, n, has_bias):
    t, b = cases.layer_tensors(name, m, n, has_bias)
    return O.Layer(t['bits'], t['tlut'], t['row_scale'], t['su'], t['sv'], bias=b)


@pytest.mark.parametrize('spec', cases.LAYERS, ids=[c[0] for c in cases.LAYERS])
def test_layer_decode_and_linear(spec):
    name, m, n, tokens, dt, has_bias = spec
    L = _layer(name, m, n, has_bias)
    golden.check(f'{name}/t8', L.t8)
    golden.check(f'{name}/rs', L.rs)
    golden.check(f'{name}/states', L.states().astype(np.int32))
    w8 = L.w8_reference()
    golden.check(f'{name}/w8', w8)
    if m * n <= 64 * 1152:
        golden.check(f'{name}/dense_fp16', L.dense('fp16'))
        golden.check(f'{name}/dense_int8', L.dense('int8'))
    for M in tokens:
        x = cases.activations(name, M, n, dt)
        h = O.fwht(O.to_f32(x, dt) * L.su.astype(np.float32))
        golden.check(f'{name}/M{M}/h', h)
        q, s = O.pre(x, dt, L.su)
        golden.check(f'{name}/M{M}/q', q)
        golden.check(f'{name}/M{M}/scale', s)
        acc = O.int_matmul(q, w8)
        golden.check(f'{name}/M{M}/acc', acc)
        z = O.scale_acc(acc, s, L.rs)
        golden.check(f'{name}/M{M}/z', z)
        golden.check(f'{name}/M{M}/y', O.reference_linear(x, dt, L, w8=w8))
        golden.check(f'{name}/M{M}/y', O.post_acc(acc, 'i32', s, L.rs, L.sv, L.bias))
        if m * n <= 1536 * 1536:
            golden.check(f'{name}/M{M}/y_a16', O.reference_linear(x, dt, L, a8=False, w8=w8))
            golden.check(f'{name}/M{M}/y_fp16table', O.reference_linear(x, dt, L, table='fp16'))
            golden.check(f'{name}/M{M}/y_fp16table_a16', O.reference_linear(x, dt, L, a8=False, table='fp16'))


@pytest.mark.parametrize('T,D', cases.ROTATIONS)
def test_rotation(T, D):
    x, s = cases.rotation_input(T, D)
    fwd = O.rotate(x, s, 'bf16')
    golden.check(f'rot/{T}x{D}/fwd', fwd)
    inv = O.rotate(fwd, s, 'f32', inverse=True)
    golden.check(f'rot/{T}x{D}/inv', inv)
    assert np.abs(inv - O.bf16_to_f32(x)).max() <= 1e-5 * max(1.0, float(np.abs(O.bf16_to_f32(x)).max()))


@pytest.mark.parametrize('M,K,N', cases.GEMMS)
def test_w8a8_gemm(M, K, N):
    a, w, sc = cases.gemm_inputs(M, K, N)
    q, s = O.quantize_tokens(O.bf16_to_f32(a))
    golden.check(f'gemm/{M}x{K}x{N}/q', q)
    golden.check(f'gemm/{M}x{K}x{N}/scale', s[:, 0])
    acc = O.int_matmul(q, w)
    golden.check(f'gemm/{M}x{K}x{N}/acc', acc)
    golden.check(f'gemm/{M}x{K}x{N}/out', O.int8_gemm_scaled(q, w, s[:, 0], sc))


@pytest.mark.parametrize('i', range(cases.SNAP_TABLES))
def test_snap(i):
    tlut, rsc = cases.snap_inputs(i)
    t8, rs, g = O.snap(tlut, rsc)
    golden.check(f'snap/{i}/t8', t8)
    golden.check(f'snap/{i}/rs', rs)
    golden.check(f'snap/{i}/gain', np.float32(g).reshape(1))


def test_q4_layout():
    q = np.arange(-60, 60, dtype=np.int8).reshape(3, 40)
    w = O.q4_words(q)
    assert w.shape == (10, 3)
    for tok in range(3):
        for j in range(10):
            b = np.array([w[j, tok]], dtype=np.int32).view(np.int8)
            assert np.array_equal(b, q[tok, 4 * j:4 * j + 4])


def test_bf16_rounding_matches_torch():
    import torch
    x = np.array([1.0, 1.00390625, 1.01171875, -2.0, np.inf, -np.inf, np.nan, 3.3895314e38, 3.4e38, 0.0, -0.0, 1e-40],
                 dtype=np.float32)
    x = np.concatenate([x, np.random.default_rng(0).standard_normal(100000).astype(np.float32) * 1e3])
    b = O.f32_to_bf16(x)
    assert b[0] == 0x3f80 and b[1] == 0x3f80 and b[2] == 0x3f82          # ties to even
    t = torch.from_numpy(x).bfloat16().view(torch.int16).numpy().view(np.uint16)
    finite = ~np.isnan(x)                      # NaN: the kernels write 0x7fc0 (c10 scalar rule); torch's CPU vector path 0xffff
    assert np.array_equal(b[finite], t[finite]) and b[6] == 0x7fc0


def test_quantizer_zero_row_and_ties():
    h = np.zeros((2, 8), dtype=np.float32)
    h[1] = [127.0, 0.5, 1.5, 2.5, -0.5, -1.5, 63.5, -127.0]
    q, s = O.quantize_tokens(h)
    assert s[0, 0] == 1.0 and np.all(q[0] == 0)
    assert s[1, 0] == 1.0 and list(q[1]) == [127, 0, 2, 2, 0, -2, 64, -127]
