"""Policy glue kernels (tcq_add_norm, tcq_rope) against PyTorch FP32 restatements of the same ops.

The residual add and the rotary embedding are elementwise with one rounding per operation, so they must match PyTorch
bit for bit. The norms reduce over the row in the kernel's own fixed order and use the hardware reciprocal square
root, so they are held to BF16 rounding: every output within 2 BF16 ulps of the FP32 restatement, and a run twice
gives identical bits."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope='module')
def K():
    if not torch.cuda.is_available():
        pytest.skip('no CUDA device')
    from yanlongvla_b200 import kernels
    return kernels


def _ref_norm(h, kind, w, b, eps, mod=None, mod_rows=1):
    hf = h.float()
    if kind == 'rms':
        n = hf * torch.rsqrt(hf.pow(2).mean(-1, keepdim=True) + eps)
    else:
        mu = hf.mean(-1, keepdim=True)
        n = (hf - mu) * torch.rsqrt((hf - mu).pow(2).mean(-1, keepdim=True) + eps)
    if w is not None:
        n = n * w
    if b is not None:
        n = n + b
    if mod is not None:
        ms, mh = mod
        ms = ms.float().repeat_interleave(mod_rows, 0)
        mh = mh.float().repeat_interleave(mod_rows, 0)
        n = n * (1 + ms) + mh
    return n


def _close_bf16(n, ref, ulps=2):
    """|n - ref| within `ulps` BF16 ulps of ref (ulp = 2^(exponent(ref) - 7)), plus a tiny absolute floor."""
    r = ref.float()
    ulp = torch.ldexp(torch.ones_like(r), torch.frexp(r)[1] - 8)
    err = (n.float() - r).abs()
    return bool((err <= ulps * ulp + 1e-30).all()), float((err / ulp.clamp_min(1e-30)).max())


@pytest.mark.parametrize('M,D', [(1, 2048), (17, 1536), (160, 2048), (64, 1152), (5, 4608), (3, 16384), (2, 32768)])
@pytest.mark.parametrize('kind', ['rms', 'ln'])
def test_add_norm_matches_fp32(K, M, D, kind):
    g = torch.Generator(device='cuda').manual_seed(M * 7 + D)
    x = (torch.randn(M, D, device='cuda', generator=g) * 3).bfloat16()
    y = (torch.randn(M, D, device='cuda', generator=g) * 0.5).bfloat16()
    w = torch.rand(D, device='cuda', generator=g) + 0.5
    b = torch.randn(D, device='cuda', generator=g) * 0.1 if kind == 'ln' else None
    eps = 1e-6 if kind == 'rms' else 1e-5
    h, n = K.add_norm(x, y, w, b, eps, kind)
    assert torch.equal(h, x + y)                       # the BF16 residual add, bit for bit
    ok, worst = _close_bf16(n, _ref_norm(h, kind, w, b, eps))
    assert ok, f'worst error {worst:.2f} ulps'
    _, n2 = K.add_norm(x, y, w, b, eps, kind)
    assert torch.equal(n, n2)                          # fixed reduction order: reproducible


@pytest.mark.parametrize('kind', ['rms', 'ln'])
def test_add_norm_bf16_params(K, kind):
    """Parameters of a model cast to BF16 (the policy's): weight / bias read as BF16."""
    g = torch.Generator(device='cuda').manual_seed(9)
    x = torch.randn(33, 1152, device='cuda', generator=g).bfloat16()
    w = (torch.rand(1152, device='cuda', generator=g) + 0.5).bfloat16()
    b = (torch.randn(1152, device='cuda', generator=g) * 0.1).bfloat16() if kind == 'ln' else None
    _, n = K.add_norm(x, None, w, b, 1e-5, kind)
    ok, worst = _close_bf16(n, _ref_norm(x, kind, w.float(), None if b is None else b.float(), 1e-5))
    assert ok, worst


def test_add_norm_rejects_mismatched_params(K):
    x = torch.randn(4, 2048, device='cuda').bfloat16()
    with pytest.raises(K.TcqError):
        K.add_norm(x, None, torch.ones(2048, device='cuda'), torch.zeros(2048, device='cuda').bfloat16(), 1e-5, 'ln')
    with pytest.raises(K.TcqError):
        K.add_norm(x, None, torch.ones(1024, device='cuda'), None, 1e-6, 'rms')


def test_add_norm_plain_and_in_place(K):
    g = torch.Generator(device='cuda').manual_seed(3)
    x = torch.randn(40, 2048, device='cuda', generator=g).bfloat16()
    y = torch.randn(40, 2048, device='cuda', generator=g).bfloat16()
    h0 = x + y
    _, n_plain = K.add_norm(h0, None, None, None, 1e-6, 'rms')
    ok, worst = _close_bf16(n_plain, _ref_norm(h0, 'rms', None, None, 1e-6))
    assert ok, worst
    xi = x.clone()
    h, n = K.add_norm(xi, y, None, None, 1e-6, 'rms', h_out=xi)      # residual updated in place
    assert h.data_ptr() == xi.data_ptr() and torch.equal(xi, h0) and torch.equal(n, n_plain)


def test_add_norm_modulation(K):
    """The DiT's AdaLN: LayerNorm without affine, then n * (1 + scale) + shift per sample (scale / shift are views
    into one (B, 1, 2D) projection output)."""
    B, T, D = 3, 17, 1536
    g = torch.Generator(device='cuda').manual_seed(5)
    x = torch.randn(B, T, D, device='cuda', generator=g).bfloat16()
    mod = (torch.randn(B, 1, 2 * D, device='cuda', generator=g) * 0.3).bfloat16()
    scale, shift = mod[:, 0, :D], mod[:, 0, D:]
    _, n = K.add_norm(x, None, None, None, 1e-6, 'ln', mod=(scale, shift), mod_rows=T)
    ref = _ref_norm(x.view(B * T, D), 'ln', None, None, 1e-6, (scale, shift), T).view(B, T, D)
    ok, worst = _close_bf16(n, ref, ulps=3)
    assert ok, worst


@pytest.mark.parametrize('B,T,heads,D', [(1, 160, 32, 64), (2, 160, 8, 64), (1, 17, 16, 96)])
def test_rope_matches_torch_bit_exact(K, B, T, heads, D):
    g = torch.Generator(device='cuda').manual_seed(T + heads)
    x = torch.randn(B, T, heads * D, device='cuda', generator=g).bfloat16()
    inv = 1.0 / (10000 ** (torch.arange(0, D, 2, device='cuda', dtype=torch.float32) / D))
    ang = torch.arange(T, device='cuda').float()[:, None] * inv[None, :]
    cos, sin = ang.cos().contiguous(), ang.sin().contiguous()
    xh = x.view(B, T, heads, D).float()
    a, b = xh[..., :D // 2], xh[..., D // 2:]
    c, s = cos[None, :, None, :], sin[None, :, None, :]
    ref = torch.cat((a * c - b * s, a * s + b * c), -1).to(torch.bfloat16).view(B, T, heads * D)
    assert torch.equal(K.rope(x, cos, sin, heads), ref)
    xi = x.clone()
    K.rope(xi, cos, sin, heads, out=xi)                              # in place
    assert torch.equal(xi, ref)
