"""Parity at the benchmark configurations' full sizes, where the float64 oracle would take minutes: exact,
size-independent properties plus oracle checks on sampled rows.

- config 3 (W8A8 GEMM), every M x (K, N) of the grid: the INT32 accumulator satisfies acc r = q (W^T r) exactly in
  int64 for random integer vectors r (a wrong element changes the product with overwhelming probability), and the
  BF16 epilogue of sampled rows equals the oracle's.
- configs 1 / 4 layer shapes up to 16384 x 16384: the fused decode-GEMV equals the dense decode followed by the exact
  INT8 GEMM and the same FP32 epilogue, bit for bit (two independent paths, each pinned to the oracle at small sizes).
- config 2 (rotation), T = 4096, D up to 16384: sampled rows equal the oracle's block Walsh bit for bit, and the
  inverse undoes the forward to FP32 rounding.
- config 4: in the full-size policy (27 / 24 / 16 layers) every quantized layer equals the PyTorch-ops definition bit
  for bit on its in-policy input, and the fly runtime's action chunk is within the task's tolerance of the
  reference runtime's."""
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


def _projection_check(acc, q, w, seed):
    r = np.random.default_rng(seed)
    for _ in range(2):
        v = r.integers(-1000, 1001, size=w.shape[0]).astype(np.int64)
        lhs = acc.astype(np.int64) @ v
        rhs = q.astype(np.int64) @ (w.astype(np.int64).T @ v)
        assert np.array_equal(lhs, rhs)


@pytest.mark.parametrize('M', [1, 16, 64, 256, 1024, 4096])
@pytest.mark.parametrize('Kd,N', [(2048, 2048), (2048, 6144), (2048, 8192), (8192, 2048)])
def test_config3_full_grid(K, M, Kd, N):
    a, w, sc = cases.gemm_inputs(M, Kd, N)
    qd, sd = K.quantize(t(a, 'bf16'))
    q, s = n(qd), n(sd)
    acc = n(K.int_mm(qd, t(w)))
    _projection_check(acc, q, w, M + Kd + N)
    rows = np.unique(np.linspace(0, M - 1, 8).astype(int))
    qo, so = O.quantize_tokens(O.bf16_to_f32(a[rows]))
    assert np.array_equal(q[rows], qo) and np.array_equal(s[rows], so[:, 0])
    out = n(K.int8_gemm(qd, t(w), sd, t(sc)))
    assert np.array_equal(out[rows], O.int8_gemm_scaled(qo, w, so[:, 0], sc))


@pytest.mark.parametrize('N,Kd,M', [(4096, 4096, 1), (16384, 16384, 1), (16384, 4096, 3), (8192, 16384, 16),
                                     (6144, 1536, 4), (2048, 8192, 8)])
def test_fused_gemv_equals_decode_plus_gemm(K, N, Kd, M):
    L = DevLayer(f'full{N}x{Kd}', N, Kd, False)
    g = torch.Generator(device='cuda').manual_seed(N + Kd + M)
    x = torch.randn(M, Kd, device='cuda', generator=g).bfloat16()
    q4 = torch.empty(Kd // 4, M, dtype=torch.int32, device='cuda')
    q = torch.empty(M, Kd, dtype=torch.int8, device='cuda')
    s = torch.empty(M, device='cuda')
    K.pre(x, L.su, q=q, q4=q4, scale=s)
    z = torch.empty(M, N, device='cuda')
    K.gemm_tcq(L.bits, L.t8, q4, s, L.rs, z, Kd)
    W = torch.empty(N, Kd, dtype=torch.int8, device='cuda')
    K.decode(L.bits, L.t8, W)
    zz = K.int8_gemm(q, W, s, L.rs, out_dtype=torch.float32)
    assert torch.equal(z, zz)
    if M <= 4 and Kd <= 8192:                          # the pre-fused entry point on the same input
        zx = torch.empty_like(z)
        K.gemm_tcq_x(L.bits, L.t8, x, L.su, L.rs, zx, Kd)
        assert torch.equal(zx, z)


@pytest.mark.parametrize('D', [4096, 16384])
def test_config2_full_rotation(K, D):
    T = 4096
    g = torch.Generator(device='cuda').manual_seed(D)
    x = torch.randn(T, D, device='cuda', generator=g).bfloat16()
    sg = (torch.randint(0, 2, (D,), device='cuda', generator=g) * 2 - 1).to(torch.int8)
    y = K.rotate(x, sg)
    rows = [0, 1, 777, 2048, T - 1]
    yo = O.rotate(n(x)[rows], n(sg), 'bf16')
    assert np.array_equal(n(y)[rows], yo)
    back = K.rotate(y, sg, inverse=True)
    err = (back - x.float()).abs().max().item()
    assert err <= 1e-5 * max(1.0, x.float().abs().max().item())


def test_config4_full_policy_every_layer_and_chunk(K):
    """Config 4 at full depth, B = 1: all 442 quantized layers (280 W2A8, 162 W8A8) reproduce the definition's
    intermediates bit for bit on the inputs they receive in the reference-runtime policy; three of the decodes are
    also checked against the CPU oracle; the fly chunk is within the task's tolerance of the reference chunk, and equal
    to it bit for bit."""
    import policy_parity as PP
    from yanlongvla_b200 import policy as P
    c = P.PolicyConfig()
    ref, layers, _ = P.build_policy('cuda', 'reference', c)
    obs = P.synthetic_observations(1, c)
    seen, a_ref = PP.capture_inputs(ref, obs)
    assert len(seen) == 442
    rec = PP.layer_records(seen, layers)
    assert not PP.failures(rec), PP.failures(rec)
    assert sum(r['kind'] == 'w2a8' for r in rec.values()) == 280
    for name in ('llm.5.mlp.down_proj', 'dit.3.attn1.q_proj', 'dit.0.adaln'):
        L = layers[name]
        ref_layer = O.Layer(n(L.bits).view(np.uint16), n(L.tlut), n(L.row_scale), n(L.su), n(L.sv))
        assert np.array_equal(n(seen[name][0].w8), ref_layer.w8_reference()), name
    del seen, ref
    torch.cuda.empty_cache()
    fly, _, info = P.build_policy('cuda', 'fly', c, layers=layers)
    assert info['chains'] == 2 * (c.llm_layers + c.dit_layers + c.vit_layers)
    with torch.no_grad():
        a = fly(*obs)
    torch.cuda.synchronize()
    ok, max_rel, cos = PP.within_tolerance(a, a_ref)
    assert torch.isfinite(a).all() and ok, f'max-abs / RMS {max_rel.tolist()}, cosine {cos.tolist()}'
    assert torch.equal(a, a_ref), f'within tolerance but not bit-exact: max-abs / RMS {max_rel.tolist()}'
