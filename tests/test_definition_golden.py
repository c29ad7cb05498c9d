"""The PyTorch-ops definition (`yanlongvla_b200.definition`, the policy's 'reference' runtime) against the reference's
own outputs (golden fixtures), bit for bit, on the CPU. The definition calls nothing of the kernel library, so the
GPU tests that compare the kernels with it compare them with an independently pinned statement of the arithmetic."""
import numpy as np
import pytest
import torch

import cases
import golden
import tcq_oracle as O
from yanlongvla_b200 import definition as D


class _L:
    """The fields of a layer the definition reads: su, sv, rs, bias, m."""
    def __init__(self, name, m, n, has_bias):
        t, b = cases.layer_tensors(name, m, n, has_bias)
        ref = O.Layer(t['bits'], t['tlut'], t['row_scale'], t['su'], t['sv'], bias=b)
        self.m, self.n = m, n
        self.bits = torch.from_numpy(t['bits'].view(np.int16).copy())
        self.t8 = torch.from_numpy(ref.t8)
        self.rs = torch.from_numpy(ref.rs)
        self.su = torch.from_numpy(t['su'])
        self.sv = torch.from_numpy(t['sv'])
        self.bias = None if b is None else torch.from_numpy(b)


def _x(a, dt):
    if dt == 'bf16':
        return torch.from_numpy(a.view(np.int16).copy()).view(torch.bfloat16)
    return torch.from_numpy(a.copy())


def _bf16(t):
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


@pytest.mark.parametrize('spec', cases.LAYERS, ids=[c[0] for c in cases.LAYERS])
def test_definition_decode_and_linear(spec):
    name, m, n, tokens, dt, has_bias = spec
    L = _L(name, m, n, has_bias)
    golden.check(f'{name}/states', D.trellis_states(L.bits, m, n).numpy().astype(np.int32))
    w8 = D.decode_w8(L.bits, L.t8, m, n)
    golden.check(f'{name}/w8', w8.numpy())
    for M in tokens:
        x = _x(cases.activations(name, M, n, dt), dt)
        h = D.walsh(x.float() * L.su.float())
        golden.check(f'{name}/M{M}/h', h.numpy())
        q, s = D.quantize_tokens(h)
        golden.check(f'{name}/M{M}/q', q.numpy())
        golden.check(f'{name}/M{M}/scale', s[:, 0].numpy())
        golden.check(f'{name}/M{M}/acc', D.int_matmul(q, w8).numpy())
        golden.check(f'{name}/M{M}/y', _bf16(D.linear(x, L, w8)))
        if m * n <= 1536 * 1536:
            golden.check(f'{name}/M{M}/y_a16', _bf16(D.linear(x, L, w8, a8=False)))


@pytest.mark.parametrize('T,Dw', cases.ROTATIONS)
def test_definition_rotation(T, Dw):
    x, s = cases.rotation_input(T, Dw)
    xs = torch.from_numpy(x.view(np.int16).copy()).view(torch.bfloat16).float() * torch.from_numpy(s).float()
    fwd = D.walsh(xs)
    golden.check(f'rot/{T}x{Dw}/fwd', fwd.numpy())
    golden.check(f'rot/{T}x{Dw}/inv', (D.walsh(fwd) * torch.from_numpy(s).float()).numpy())


@pytest.mark.parametrize('M,K,N', cases.GEMMS)
def test_definition_w8a8(M, K, N):
    a, w, sc = cases.gemm_inputs(M, K, N)
    x = torch.from_numpy(a.view(np.int16).copy()).view(torch.bfloat16)
    golden.check(f'gemm/{M}x{K}x{N}/out', _bf16(D.w8a8_linear(x, torch.from_numpy(w), torch.from_numpy(sc))))


def test_block_widths():
    assert D.block_widths(4304) == [4096, 128, 64, 16]
    assert D.block_widths(1152) == [1024, 128]
    assert D.block_widths(16384) == [16384]
    assert all(sum(D.block_widths(w)) == w for w in range(1, 2000))


def test_norms_and_rope_shapes():
    """The glue ops keep shapes and dtypes; RMSNorm of a constant row is the weight (up to one BF16 rounding)."""
    x = torch.full((3, 64), 2.0, dtype=torch.bfloat16)
    w = torch.linspace(0.5, 1.5, 64).bfloat16()
    h, nrm = D.add_norm(x, None, w, None, 1e-6, 'rms')
    assert h is x and nrm.dtype == torch.bfloat16 and torch.allclose(nrm.float(), w.float().expand(3, 64), rtol=1e-2)
    _, ln = D.add_norm(x, x, None, None, 1e-5, 'ln', mod=(torch.ones(1, 64).bfloat16(), torch.full((1, 64), 0.5).bfloat16()),
                       mod_rows=3)
    assert torch.equal(ln.float(), torch.full((3, 64), 0.5))          # centred constant row: 0 * 2 + 0.5
    q = torch.randn(2, 5, 4 * 16).bfloat16()
    cos, sin = torch.ones(5, 8), torch.zeros(5, 8)
    assert torch.equal(D.rope(q, cos, sin, 4), q)                       # angle 0 is the identity
