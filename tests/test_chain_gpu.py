"""tcq_chain (post -> residual add -> norm -> pre in one launch) against the three separate entry points.

Every stage of the chain is specified as the separate kernel's arithmetic (kernels.post, kernels.add_norm with the
same thread count and sum order, kernels.pre), so the fused outputs must equal the decomposition bit for bit: the new
residual h, the norm output n, the next layer's INT8 activations (q and q4 layouts) and their scales."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope='module')
def K():
    if not torch.cuda.is_available():
        pytest.skip('no CUDA device')
    from yanlongvla_b200 import kernels
    return kernels


def _signs(n, g):
    return (torch.randint(0, 2, (n,), device='cuda', generator=g) * 2 - 1).to(torch.int8)


def _case(M, N, at, g, lda_extra=0):
    lda = N + lda_extra
    if at == 'i32':
        acc = torch.randint(-2 ** 20, 2 ** 20, (M, lda), dtype=torch.int32, device='cuda', generator=g)
        s = torch.rand(M, device='cuda', generator=g) * 1e-3 + 1e-4
        rs = torch.rand(N, device='cuda', generator=g) * 1e-2 + 1e-3
    else:
        acc = torch.randn(M, lda, device='cuda', generator=g) * 2
        s = rs = None
    sv = _signs(N, g)
    return acc, s, rs, sv


@pytest.mark.parametrize('M,N', [(1, 2048), (3, 1536), (17, 1536), (160, 2048), (40, 1152), (9, 6144)])
@pytest.mark.parametrize('at', ['i32', 'f32'])
@pytest.mark.parametrize('kind', ['rms', 'ln'])
def test_chain_equals_post_addnorm_pre(K, M, N, at, kind):
    g = torch.Generator(device='cuda').manual_seed(M * 131 + N + (7 if at == 'f32' else 0) + (3 if kind == 'ln' else 0))
    col0 = 16 if at == 'i32' else 0
    acc, s, rs, sv = _case(M, N, at, g, lda_extra=col0 + 32)
    bias = torch.randn(N, device='cuda', generator=g) * 0.1 if kind == 'ln' else None
    x = torch.randn(M, N, device='cuda', generator=g).bfloat16()
    w = (torch.rand(N, device='cuda', generator=g) + 0.5).bfloat16()
    nb = (torch.randn(N, device='cuda', generator=g) * 0.1).bfloat16() if kind == 'ln' else None
    su = _signs(N, g)
    eps = 1e-6 if kind == 'rms' else 1e-5
    # decomposition: three launches
    y = torch.empty(M, N, dtype=torch.bfloat16, device='cuda')
    K.post(acc, s, None if rs is None else rs, sv, bias, y, col0=col0)
    h_ref, n_ref = K.add_norm(x, y, w, nb, eps, kind)
    q_ref = torch.empty(M, N, dtype=torch.int8, device='cuda')
    q4_ref = torch.empty(N // 4, M + 3, dtype=torch.int32, device='cuda')
    sc_ref = torch.empty(M, device='cuda')
    K.pre(n_ref, su, q=q_ref, q4=q4_ref, scale=sc_ref)
    # fused: one launch
    q = torch.empty_like(q_ref)
    q4 = torch.zeros_like(q4_ref)
    sc = torch.empty_like(sc_ref)
    q4_ref[:, M:] = 0
    h, n = K.chain(x, kind, w, nb, eps, acc=acc, s=s, rs=rs, sv=sv, bias=bias, col0=col0, su=su, q=q, q4=q4, scale=sc)
    assert torch.equal(h, h_ref)
    assert torch.equal(n, n_ref)
    assert torch.equal(q, q_ref) and torch.equal(q4, q4_ref) and torch.equal(sc, sc_ref)


def test_chain_with_tensor_add_and_modulation(K):
    """y from a BF16 tensor (a producer whose post already ran) and the DiT's AdaLN modulation, pre to q only."""
    B, T, N = 2, 17, 1536
    g = torch.Generator(device='cuda').manual_seed(21)
    x = torch.randn(B * T, N, device='cuda', generator=g).bfloat16()
    y = torch.randn(B * T, N, device='cuda', generator=g).bfloat16()
    mod = (torch.randn(B, 1, 2 * N, device='cuda', generator=g) * 0.3).bfloat16()
    ms, mh = mod[:, 0, :N], mod[:, 0, N:]
    su = _signs(N, g)
    h_ref, n_ref = K.add_norm(x, y, None, None, 1e-6, 'ln', mod=(ms, mh), mod_rows=T)
    q_ref = torch.empty(B * T, N, dtype=torch.int8, device='cuda')
    sc_ref = torch.empty(B * T, device='cuda')
    K.pre(n_ref, su, q=q_ref, scale=sc_ref)
    q = torch.empty_like(q_ref)
    sc = torch.empty_like(sc_ref)
    h, n = K.chain(x, 'ln', None, None, 1e-6, y=y, mod=(ms, mh), mod_rows=T, su=su, q=q, scale=sc, want_n=False)
    assert n is None and torch.equal(h, h_ref) and torch.equal(q, q_ref) and torch.equal(sc, sc_ref)


def test_chain_norm_pre_without_add(K):
    """The first block of a stack: no pending residual, norm + pre of x itself."""
    g = torch.Generator(device='cuda').manual_seed(22)
    x = torch.randn(160, 2048, device='cuda', generator=g).bfloat16()
    w = torch.rand(2048, device='cuda', generator=g).bfloat16() + 0.5
    su = _signs(2048, g)
    _, n_ref = K.add_norm(x, None, w, None, 1e-6, 'rms')
    q_ref = torch.empty(160, 2048, dtype=torch.int8, device='cuda')
    sc_ref = torch.empty(160, device='cuda')
    K.pre(n_ref, su, q=q_ref, scale=sc_ref)
    q, sc = torch.empty_like(q_ref), torch.empty_like(sc_ref)
    h, n = K.chain(x, 'rms', w, None, 1e-6, su=su, q=q, scale=sc)
    assert h.data_ptr() == x.data_ptr() and torch.equal(n, n_ref) and torch.equal(q, q_ref) and torch.equal(sc, sc_ref)


@pytest.mark.parametrize('kind', ['rms', 'ln'])
@pytest.mark.parametrize('N', [1152, 1536, 2048])
def test_rows_do_not_depend_on_launch_size(K, kind, N):
    """A few rows run with 4-element chunks per thread, many rows with 16 (more threads per row only while the launch
    is small); the norm's sum order is the same for both, so a row's results must not change with the row count."""
    g = torch.Generator(device='cuda').manual_seed(N + (1 if kind == 'ln' else 0))
    few, many = 5, 1200
    acc = torch.randint(-2 ** 20, 2 ** 20, (few, N), dtype=torch.int32, device='cuda', generator=g)
    s = torch.rand(few, device='cuda', generator=g) * 1e-3 + 1e-4
    rs = torch.rand(N, device='cuda', generator=g) * 1e-2 + 1e-3
    sv, su = _signs(N, g), _signs(N, g)
    x = torch.randn(few, N, device='cuda', generator=g).bfloat16()
    w = (torch.rand(N, device='cuda', generator=g) + 0.5).bfloat16()
    nb = (torch.randn(N, device='cuda', generator=g) * 0.1).bfloat16() if kind == 'ln' else None
    bias = torch.randn(N, device='cuda', generator=g) * 0.1
    eps = 1e-6 if kind == 'rms' else 1e-5
    rep = many // few

    def run(a, sc, xx):
        M = xx.shape[0]
        y = torch.empty(M, N, dtype=torch.bfloat16, device='cuda')
        K.post(a, sc, rs, sv, bias, y)
        h1, n1 = K.add_norm(xx, y, w, nb, eps, kind)
        q1 = torch.empty(M, N, dtype=torch.int8, device='cuda')
        sc1 = torch.empty(M, device='cuda')
        K.pre(n1, su, q=q1, scale=sc1)
        q2 = torch.empty_like(q1)
        sc2 = torch.empty_like(sc1)
        h2, n2 = K.chain(xx, kind, w, nb, eps, acc=a, s=sc, rs=rs, sv=sv, bias=bias, su=su, q=q2, scale=sc2)
        return [y, h1, n1, q1, sc1, h2, n2, q2, sc2]

    small = run(acc, s, x)
    large = run(acc.repeat(rep, 1), s.repeat(rep), x.repeat(rep, 1))
    for a, b in zip(small, large):
        assert torch.equal(a, b[:few])
    # the fused chain equals its decomposition at both sizes
    for out in (small, large):
        assert torch.equal(out[5], out[1]) and torch.equal(out[6], out[2])
        assert torch.equal(out[7], out[3]) and torch.equal(out[8], out[4])


@pytest.mark.parametrize('M,N', [(1, 1152), (128, 1152), (512, 1152), (7, 2048)])
@pytest.mark.parametrize('add', [False, True])
def test_chain_quantize_only_equals_addnorm_quantize(K, M, N, add):
    """No rotation (a W8A8 consumer, the vision tower's layer norms): q / q4 / scale are the plain per-token INT8
    quantization of the norm output, bit for bit kernels.add_norm followed by kernels.quantize."""
    g = torch.Generator(device='cuda').manual_seed(M * 7 + N + (1 if add else 0))
    x = torch.randn(M, N, device='cuda', generator=g).bfloat16()
    y = torch.randn(M, N, device='cuda', generator=g).bfloat16() if add else None
    w = (torch.rand(N, device='cuda', generator=g) + 0.5).bfloat16()
    nb = (torch.randn(N, device='cuda', generator=g) * 0.1).bfloat16()
    h_ref, n_ref = K.add_norm(x, y, w, nb, 1e-5, 'ln')
    q_ref, sc_ref = K.quantize(n_ref)
    q = torch.empty_like(q_ref)
    q4 = torch.zeros(N // 4, M, dtype=torch.int32, device='cuda')
    sc = torch.empty_like(sc_ref)
    kw = {'y': y} if add else {}
    h, n = K.chain(x, 'ln', w, nb, 1e-5, q=q, q4=q4, scale=sc, want_n=False, **kw)
    assert n is None and torch.equal(h, h_ref)
    assert torch.equal(q, q_ref) and torch.equal(sc, sc_ref)
    assert torch.equal(q4, q_ref.view(M, N // 4, 4).view(torch.int32).view(M, N // 4).t())
