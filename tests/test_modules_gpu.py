"""Module-level operator API (install / KLinear / KGatedMLP / KPlainMLP / RefLinear / decode_chunk) against the CPU
oracle: every runtime reproduces the reference definition bit for bit, for few tokens (fused decode-GEMV path) and
many tokens (tcgen05 INT8 GEMM path)."""
import numpy as np
import pytest
import torch

import cases
import tcq_oracle as O
from gpu_util import n, t

pytestmark = pytest.mark.gpu


class Block(torch.nn.Module):
    """A minimal transformer-shaped block: q/k/v/o attention projections, a gated MLP and a plain MLP."""
    def __init__(self, d, f):
        super().__init__()
        self.attn = torch.nn.Module()
        for name, (o, i) in dict(q_proj=(d, d), k_proj=(d // 4, d), v_proj=(d // 4, d), o_proj=(d, d)).items():
            setattr(self.attn, name, torch.nn.Linear(i, o, bias=False))
        self.mlp = torch.nn.Module()
        self.mlp.gate_proj = torch.nn.Linear(d, f, bias=False)
        self.mlp.up_proj = torch.nn.Linear(d, f, bias=False)
        self.mlp.down_proj = torch.nn.Linear(f, d, bias=False)
        self.ffn = torch.nn.Module()
        self.ffn.fc1 = torch.nn.Linear(d, f)
        self.ffn.fc2 = torch.nn.Linear(f, d)

    def forward(self, x):
        q, k, v = self.attn.q_proj(x), self.attn.k_proj(x), self.attn.v_proj(x)
        return q, k, v, self.attn.o_proj(q), self.mlp(x), self.ffn(x)


def _mlp_forward(self, x):
    return self.down_proj(torch.nn.functional.silu(self.gate_proj(x)) * self.up_proj(x))


D, F = 256, 1152


def make_layers(dev):
    from yanlongvla_b200.tcq_format import Layer
    shapes = {'attn.q_proj': (D, D), 'attn.k_proj': (D // 4, D), 'attn.v_proj': (D // 4, D), 'attn.o_proj': (D, D),
              'mlp.gate_proj': (F, D), 'mlp.up_proj': (F, D), 'mlp.down_proj': (D, F), 'ffn.fc1': (F, D), 'ffn.fc2': (D, F)}
    su_by_width = {}
    layers, refs = {}, {}
    for name, (m, k) in shapes.items():
        tens, b = cases.layer_tensors('mod.' + name, m, k, bias=name.startswith('ffn'))
        if k not in su_by_width:
            su_by_width[k] = tens['su']
        tens['su'] = su_by_width[k]                           # layers reading the same input share their input signs
        tt = dict(bits=torch.from_numpy(tens['bits'].view(np.int16).copy()), tlut=torch.from_numpy(tens['tlut']),
                  row_scale=torch.from_numpy(tens['row_scale']), su=torch.from_numpy(tens['su']), sv=torch.from_numpy(tens['sv']))
        layers[name] = Layer(name, tt, bias=None if b is None else torch.from_numpy(b), device=dev)
        refs[name] = O.Layer(tens['bits'], tens['tlut'], tens['row_scale'], tens['su'], tens['sv'], bias=b)
    return layers, refs


def oracle_outputs(refs, x, lut_silu, lut_gelu):
    lin = lambda name, xx, dt='bf16': O.reference_linear(xx, dt, refs[name])
    q, k, v = lin('attn.q_proj', x), lin('attn.k_proj', x), lin('attn.v_proj', x)
    o = lin('attn.o_proj', q)
    g = O.act_lut(lut_silu, lin('mlp.gate_proj', x))
    mlp = lin('mlp.down_proj', O.bf16_mul(g, lin('mlp.up_proj', x)))
    ffn = lin('ffn.fc2', O.act_lut(lut_gelu, lin('ffn.fc1', x)))
    return [q, k, v, o, mlp, ffn]


@pytest.fixture(scope='module')
def env():
    if not torch.cuda.is_available():
        pytest.skip('no CUDA device')
    from yanlongvla_b200 import kernels as K
    dev = torch.device('cuda')
    layers, refs = make_layers(dev)
    return K, dev, layers, refs, n(K.act_table('silu')), n(K.act_table('gelu'))


@pytest.mark.parametrize('runtime', ['fly', 'resident', 'hybrid', 'reference'])
@pytest.mark.parametrize('M', [1, 7, 16, 17, 200])
def test_install_runtimes(env, runtime, M):
    from yanlongvla_b200 import modules
    K, dev, layers, refs, lut_silu, lut_gelu = env
    model = Block(D, F).to(dev)
    model.mlp.forward = _mlp_forward.__get__(model.mlp)
    info = modules.install(model, layers, runtime=runtime, chunk_parts=('mlp',),
                           mlp_acts={'mlp': 'silu', 'ffn': 'gelu'} if runtime != 'reference' else None)
    if runtime == 'reference':
        model.ffn.forward = lambda x: model.ffn.fc2(torch.nn.functional.gelu(model.ffn.fc1(x), approximate='tanh'))
    else:
        assert info['groups'] == 6 and info['shared_rotations'] == 3 and info['fused_mlps'] == 2
    if runtime == 'hybrid':
        assert modules.decode_chunk(model) == 3
    x = cases.activations('mod', M, D, 'bf16')
    outs = model(t(x, 'bf16'))
    torch.cuda.synchronize()
    want = oracle_outputs(refs, x, lut_silu, lut_gelu)
    for i, (got, ref) in enumerate(zip(outs, want)):
        assert np.array_equal(n(got), ref), f'output {i} ({runtime}, M={M}): {int((n(got) != ref).sum())} differ'


def test_tcq_format_roundtrip(env, tmp_path):
    from yanlongvla_b200 import tcq_format as TF
    K, dev, layers, refs, _, _ = env
    packed = {name: dict(bits=L.bits, tlut=L.tlut, row_scale=L.row_scale, su=L.su, sv=L.sv) for name, L in layers.items()}
    p = tmp_path / 'packed.safetensors'
    TF.save(p, packed)
    back = TF.load(p, device=dev)
    for name, L in layers.items():
        B = back[name]
        assert torch.equal(B.bits, L.bits) and torch.equal(B.t8, L.t8) and torch.equal(B.rs, L.rs)
        assert np.array_equal(n(B.w8()), refs[name].w8_reference())
    dense = layers['attn.q_proj'].dense()
    ref = refs['attn.q_proj'].dense('int8')
    assert np.abs(n(dense) - ref).max() <= 1e-6 * max(1.0, np.abs(ref).max())
