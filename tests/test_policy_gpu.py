"""The GR00T-style quantized policy (benchmark configs 4 and 5) at reduced depth, against its 'reference' runtime: the
W2A8 / W8A8 definition with norms and rotary embedding in PyTorch ops (`yanlongvla_b200.definition`), which runs
nothing of the kernel library.

  * every quantized layer, on the input it receives inside the reference policy, reproduces the definition's
    intermediates bit for bit through the kernels (tests/policy_parity.py; the reference's parity.py:22-73);
  * whole action chunks of every kernel runtime are within the task's tolerance of the reference chunk, per
    observation (max-abs <= 1e-2 x RMS, cosine >= 0.9995), at B = 1 and B = 8, and in fact bit for bit: the
    reference runtime's norms sum their rows in the kernels' fixed order (`definition.row_sum`);
  * the kernel runtimes agree with one another bit for bit, and the fused block-boundary chains equal the separate
    post / add-norm / pre kernels bit for bit.
"""
import pytest
import torch

import policy_parity as PP

pytestmark = pytest.mark.gpu


@pytest.fixture(scope='module')
def small():
    if not torch.cuda.is_available():
        pytest.skip('no CUDA device')
    from yanlongvla_b200 import policy as P
    c = P.PolicyConfig(vit_layers=2, llm_layers=2, dit_layers=2)
    ref, layers, info = P.build_policy('cuda', 'reference', c)
    return P, c, ref, layers, info


@pytest.mark.parametrize('B', [1, 8])
def test_every_layer_matches_definition(small, B):
    P, c, ref, layers, _ = small
    obs = P.synthetic_observations(B, c, seed=10 + B)
    seen, _ = PP.capture_inputs(ref, obs)
    assert len(seen) == 6 * c.vit_layers + 7 * (c.llm_layers + c.dit_layers)
    rec = PP.layer_records(seen, layers)
    assert not PP.failures(rec), PP.failures(rec)
    kinds = {(r['kind'], r['tokens']) for r in rec.values()}
    assert ('w2a8', B * c.prefix_tokens) in kinds and ('w2a8', B * (c.chunk + 1)) in kinds and ('w2a8', B) in kinds


@pytest.mark.parametrize('B', [1, 8])
@pytest.mark.parametrize('runtime', ['fly', 'resident', 'hybrid'])
def test_chunk_within_tolerance(small, runtime, B):
    from yanlongvla_b200 import modules
    P, c, ref, layers, _ = small
    obs = P.synthetic_observations(B, c, seed=20 + B)
    with torch.no_grad():
        a_ref = ref(*obs)
    model, _, info = P.build_policy('cuda', runtime, c, layers=layers)
    assert info['fused_mlps'] == c.llm_layers + c.dit_layers
    assert info['chains'] == 2 * (c.llm_layers + c.dit_layers + c.vit_layers)   # every block boundary fused
    with torch.no_grad():
        if runtime == 'hybrid':
            modules.decode_chunk(model)
        a = model(*obs)
    torch.cuda.synchronize()
    assert torch.isfinite(a).all()
    ok, max_rel, cos = PP.within_tolerance(a, a_ref)
    assert ok, f'max-abs / RMS {max_rel.tolist()}, cosine {cos.tolist()}'
    assert torch.equal(a, a_ref), f'within tolerance but not bit-exact: max-abs / RMS {max_rel.tolist()}'


def test_kernel_runtimes_agree_and_chains_equal_unfused(small):
    from yanlongvla_b200 import modules
    P, c, _, layers, _ = small
    obs = P.synthetic_observations(3, c, seed=30)
    outs = {}
    for runtime in ('fly', 'resident', 'hybrid'):
        model, _, _ = P.build_policy('cuda', runtime, c, layers=layers)
        with torch.no_grad():
            if runtime == 'hybrid':
                modules.decode_chunk(model)
            outs[runtime] = model(*obs)
    modules.FUSE['chain'] = False
    try:
        model, _, info = P.build_policy('cuda', 'fly', c, layers=layers)
    finally:
        modules.FUSE['chain'] = True
    assert info['chains'] == 0
    with torch.no_grad():
        outs['unfused'] = model(*obs)
    torch.cuda.synchronize()
    for k, v in outs.items():
        assert torch.equal(v, outs['fly']), k
