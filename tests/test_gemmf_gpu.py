"""W2 float-activation path (the reference's operating point a8=False): kernels.gemmf_tcq / gemmf_w8 against the
oracle's float64 product, and install(a8=False) against the oracle's reference_linear(a8=False).

The kernels accumulate in FP32 in their own fixed order, so they are held to tolerances: the products to
|z - z64| <= 1e-4 * max|z64| (FP32 sums of K terms), the BF16 layer outputs to max(1e-2 x output RMS, 2 BF16 ulps)
per element and cosine >= 0.9995 (the kernel path also rounds the rotated activations to BF16, by design). Repeated
runs must give identical bits."""
import numpy as np
import pytest
import torch

import cases
import tcq_oracle as O
from gpu_util import DevLayer, n, t

pytestmark = pytest.mark.gpu


@pytest.fixture(scope='module')
def K():
    if not torch.cuda.is_available():
        pytest.skip('no CUDA device')
    from yanlongvla_b200 import kernels
    return kernels


def _hT(M, k, seed):
    rng = np.random.default_rng(seed)
    h = O.f32_to_bf16(rng.standard_normal((M, k)).astype(np.float32))
    return h, np.ascontiguousarray(h.T)


def _close(z, ref, rtol=1e-4):
    err = np.abs(z.astype(np.float64) - ref.astype(np.float64)).max()
    assert err <= rtol * np.abs(ref).max(), f'max error {err:.3g} vs scale {np.abs(ref).max():.3g}'


@pytest.mark.parametrize('M', [1, 3, 16, 21])
@pytest.mark.parametrize('m,k', [(256, 1152), (512, 512)])
def test_gemmf_matches_float64(K, M, m, k):
    L = DevLayer(f'gemmf.{m}.{k}', m, k)
    w8 = L.ref.w8_reference()
    h, hT = _hT(M, k, m + k + M)
    zref = O.gemmf_z(h, w8, L.ref.rs)
    z = torch.empty(M, m, device='cuda')
    K.gemmf_tcq(L.bits, L.t8, t(hT, 'bf16'), L.rs, z, k)
    _close(n(z), zref)
    z2 = torch.empty_like(z)
    K.gemmf_tcq(L.bits, L.t8, t(hT, 'bf16'), L.rs, z2, k)
    assert torch.equal(z, z2)                          # fixed sum order: reproducible
    zw = torch.empty_like(z)
    K.gemmf_w8(t(w8), t(hT, 'bf16'), L.rs, zw)
    _close(n(zw), zref)


def test_gemmf_tcq_multi_layer_bounds(K):
    """Three layers of one group in one launch: per-layer tables selected by tile-row bounds."""
    k, ms = 512, (128, 256, 64)
    parts = [DevLayer(f'gemmf.grp.{i}', m, k) for i, m in enumerate(ms)]
    M = 5
    h, hT = _hT(M, k, 99)
    bits = torch.cat([p.bits for p in parts]).contiguous()
    t8 = torch.cat([p.t8.reshape(-1) for p in parts]).contiguous()
    rs = torch.cat([p.rs for p in parts]).contiguous()
    z = torch.empty(M, sum(ms), device='cuda')
    K.gemmf_tcq(bits, t8, t(hT, 'bf16'), rs, z, k, (ms[0] // 16, (ms[0] + ms[1]) // 16))
    c = 0
    for p, m in zip(parts, ms):
        _close(n(z)[:, c:c + m], O.gemmf_z(h, p.ref.w8_reference(), p.ref.rs))
        c += m


class _Block(torch.nn.Module):
    def __init__(self, d, f):
        super().__init__()
        self.attn = torch.nn.Module()
        for name, (o, i) in dict(q_proj=(d, d), k_proj=(d // 4, d), v_proj=(d // 4, d)).items():
            setattr(self.attn, name, torch.nn.Linear(i, o, bias=False))
        self.ffn = torch.nn.Module()
        self.ffn.fc1 = torch.nn.Linear(d, f)

    def forward(self, x):
        return self.attn.q_proj(x), self.attn.k_proj(x), self.attn.v_proj(x), self.ffn.fc1(x)


def _within_tolerance(got, ref):
    """Per element within max(1e-2 x output RMS, 2 BF16 ulps of the reference value) — a BF16 output of a few times
    the RMS moves by one ulp (2^-7 relative) when the BF16-rounded activations shift its last bit — and cosine
    >= 0.9995 over the layer."""
    g, r = got.astype(np.float64), ref.astype(np.float64)
    rms = np.sqrt((r ** 2).mean())
    ulp = np.ldexp(1.0, np.frexp(r)[1] - 8)
    cos = (g * r).sum() / np.sqrt((g ** 2).sum() * (r ** 2).sum())
    bound = np.maximum(1e-2 * rms, 2 * ulp)
    assert (np.abs(g - r) <= bound).all() and cos >= 0.9995, (float((np.abs(g - r) / bound).max()), cos)


@pytest.mark.parametrize('runtime', ['fly', 'resident', 'hybrid', 'reference'])
@pytest.mark.parametrize('M', [1, 16, 17, 200])
def test_install_w2_float_path(K, runtime, M):
    from yanlongvla_b200 import modules
    from yanlongvla_b200.tcq_format import Layer
    D, F = 256, 1152
    shapes = {'attn.q_proj': (D, D), 'attn.k_proj': (D // 4, D), 'attn.v_proj': (D // 4, D), 'ffn.fc1': (F, D)}
    layers, refs, su = {}, {}, None
    for name, (m, k) in shapes.items():
        tens, b = cases.layer_tensors('w2.' + name, m, k, bias=name.startswith('ffn'))
        su = tens['su'] if su is None else su
        tens['su'] = su
        tt = {key: torch.from_numpy(tens[key].view(np.int16).copy() if key == 'bits' else tens[key])
              for key in ('bits', 'tlut', 'row_scale', 'su', 'sv')}
        layers[name] = Layer(name, tt, bias=None if b is None else torch.from_numpy(b), device='cuda')
        refs[name] = O.Layer(tens['bits'], tens['tlut'], tens['row_scale'], tens['su'], tens['sv'], bias=b)
    model = _Block(D, F).cuda()
    info = modules.install(model, layers, runtime=runtime, chunk_parts=('attn',), a8=False)
    assert info['a8'] is False
    if runtime == 'hybrid':
        modules.decode_chunk(model)
    x = cases.activations('w2', M, D, 'bf16')
    outs = model(t(x, 'bf16'))
    torch.cuda.synchronize()
    for (name, ref), got in zip(refs.items(), outs):
        want = O.bf16_to_f32(O.reference_linear(x, 'bf16', ref, a8=False))
        _within_tolerance(n(got.float()), want)
