"""The GR00T-style quantized policy: every kernel runtime reproduces the reference runtime (the
W2A8 / W8A8 definition in PyTorch ops) bit for bit on whole action chunks, and single layers inside the policy match
the CPU oracle on the inputs they see there."""
import numpy as np
import pytest
import torch

import tcq_oracle as O
from gpu_util import n

pytestmark = pytest.mark.gpu


@pytest.fixture(scope='module')
def built():
    if not torch.cuda.is_available():
        pytest.skip('no CUDA device')
    from yanlongvla_b200 import policy as P
    c = P.PolicyConfig(vit_layers=4, llm_layers=4, dit_layers=4)
    ref, layers, _ = P.build_policy('cuda', 'reference', c)
    obs = P.synthetic_observations(2, c)
    with torch.no_grad():
        a_ref = ref(*obs)
    torch.cuda.synchronize()
    return P, c, layers, obs, a_ref


@pytest.mark.parametrize('runtime', ['fly', 'resident', 'hybrid'])
def test_policy_runtimes_match_reference(built, runtime):
    from yanlongvla_b200 import modules
    P, c, layers, obs, a_ref = built
    model, _, info = P.build_policy('cuda', runtime, c, layers=layers)
    assert info['fused_mlps'] == c.llm_layers + c.dit_layers
    assert info['chains'] == 2 * (c.llm_layers + c.dit_layers + c.vit_layers)   # every block boundary fused
    with torch.no_grad():
        if runtime == 'hybrid':
            modules.decode_chunk(model)
        a = model(*obs)
    torch.cuda.synchronize()
    assert torch.isfinite(a).all()
    assert torch.equal(a, a_ref), f'max |da| = {float((a - a_ref).abs().max())}'


def test_policy_layers_match_oracle(built):
    """Hook two quantized layers (LLM q/k/v group member, DiT AdaLN at M = batch) and check them against the oracle."""
    from yanlongvla_b200 import modules
    P, c, layers, obs, _ = built
    modules.FUSE['chain'] = False                  # the hooks read each layer's input as a tensor
    try:
        model, _, info = P.build_policy('cuda', 'fly', c, layers=layers)
    finally:
        modules.FUSE['chain'] = True
    assert info['chains'] == 0
    seen = {}

    def hook(name):
        def f(mod, inp, out):
            if name not in seen:
                seen[name] = (inp[0].detach().clone(), out.detach().clone())
        return f
    names = ['llm.1.self_attn.k_proj', 'dit.2.adaln', 'dit.0.attn1.v_proj']
    hs = [model.get_submodule(nm).register_forward_hook(hook(nm)) for nm in names]
    with torch.no_grad():
        model(*obs)
    for h in hs:
        h.remove()
    for nm in names:
        L = layers[nm]
        x, y = seen[nm]
        ref = O.Layer(n(L.bits).view(np.uint16), n(L.tlut), n(L.row_scale), n(L.su), n(L.sv))
        yr = O.reference_linear(n(x.reshape(-1, L.n)), 'bf16', ref)
        assert np.array_equal(n(y.reshape(-1, L.m)), yr), nm
