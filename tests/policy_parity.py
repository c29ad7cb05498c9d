"""Layer-by-layer and chunk-level parity of the quantized policy against its 'reference' runtime (the definition in
PyTorch ops, `yanlongvla_b200.definition`, which runs none of the kernel library), in the manner of the reference's
deploy/tcq_kernels/parity.py:22-102:

  layer_records  runs the reference-runtime policy once with a forward hook on every quantized layer (the W2A8
                 RefLinear of the LLM / DiT and the W8A8 layers of the vision tower), then replays each layer's first
                 call through the kernels on the same input and compares every intermediate bit for bit: decoded INT8
                 weights, INT8 activations, token scales, INT32 accumulators (tcgen05 INT8 GEMM, and the fused
                 products' FP32 scaled accumulators: SIMT decode-GEMV for M <= 16, tensor-core decode-GEMM for
                 M <= 256), BF16 outputs.
  chunk_error    per-observation error of an action chunk against the reference chunk: max-abs over the output RMS
                 and the cosine similarity (the task's tolerance: max-abs <= 1e-2 x RMS, cosine >= 0.9995).
"""
import torch
import torch.nn.functional as F

MAX_ABS_OVER_RMS = 1e-2
MIN_COSINE = 0.9995


def capture_inputs(model, obs):
    """Forward the reference-runtime `model` on `obs` with hooks on every quantized layer; returns
    {name: (module, input, kwargs, output)} of each layer's first call and the action chunk."""
    from yanlongvla_b200 import modules, policy as P
    seen, handles = {}, []

    def hook(name):
        def f(mod, args, kwargs, out):
            if name not in seen:
                seen[name] = (mod, args[0].detach().clone(), dict(kwargs), out.detach().clone())
        return f
    for name, m in model.named_modules():
        if isinstance(m, (modules.RefLinear, P.W8A8Linear)):
            handles.append(m.register_forward_hook(hook(name), with_kwargs=True))
    with torch.no_grad():
        actions = model(*obs)
    for h in handles:
        h.remove()
    torch.cuda.synchronize()
    return seen, actions


def _w2a8_record(K, D, L, mod, x, y_ref):
    """Kernel paths of one W2A8 layer on input x against the definition's intermediates."""
    x2 = x.reshape(-1, L.n).contiguous()
    M = x2.shape[0]
    dev = x2.device
    rec = dict(kind='w2a8', tokens=M, shape=[L.m, L.n])
    w8 = L.w8()                                                    # sm_100a decode kernel
    rec['decode'] = bool(torch.equal(w8, mod.w8))                  # PyTorch-ops decode of the definition
    h = D.walsh(x2.float() * L.su.float())
    q_ref, s_ref = D.quantize_tokens(h)
    acc_ref = D.int_matmul(q_ref, mod.w8)                          # cuBLASLt (torch._int_mm)
    z_ref = (acc_ref.float() * s_ref) * L.rs[None, :]
    q = torch.empty(M, L.n, dtype=torch.int8, device=dev)
    s = torch.empty(M, dtype=torch.float32, device=dev)
    q4 = torch.empty(L.n // 4, M, dtype=torch.int32, device=dev) if M <= 16 else None
    K.pre(x2, L.su, q=q, q4=q4, scale=s)
    rec['activations'] = bool(torch.equal(q, q_ref))
    rec['scales'] = bool(torch.equal(s, s_ref[:, 0]))
    acc = K.int_mm(q, w8)
    rec['accumulator'] = bool(torch.equal(acc, acc_ref))
    if q4 is not None:
        z = torch.empty(M, L.m, dtype=torch.float32, device=dev)
        K.gemm_tcq(L.bits, L.t8, q4, s, L.rs, z, L.n)
        rec['accumulator_gemv'] = bool(torch.equal(z, z_ref))
    if M <= 256:
        z = torch.empty(M, L.m, dtype=torch.float32, device=dev)
        K.gemm_tcq_tc(L.bits, L.t8, q, s, L.rs, z, L.n)
        rec['accumulator_tc'] = bool(torch.equal(z, z_ref))
    y = torch.empty(M, L.m, dtype=torch.bfloat16, device=dev)
    K.post(acc, s, L.rs, L.sv, L.bias, y)
    rec['output'] = bool(torch.equal(y, y_ref.reshape(M, L.m)))
    return rec


def _w8a8_record(K, D, mod, x, kwargs, y_ref):
    x2 = x.reshape(-1, mod.in_features).contiguous()
    M = x2.shape[0]
    rec = dict(kind='w8a8', tokens=M, shape=[mod.out_features, mod.in_features])
    q_ref, s_ref = D.quantize_tokens(x2.float())
    q, s = K.quantize(x2)
    rec['activations'] = bool(torch.equal(q, q_ref))
    rec['scales'] = bool(torch.equal(s, s_ref[:, 0]))
    rec['accumulator'] = bool(torch.equal(K.int_mm(q, mod.W), D.int_matmul(q_ref, mod.W)))
    y = K.int8_gemm_bias(q, mod.W, s, mod.s_ch, bias=mod.bias)
    if kwargs.get('act') == 'gelu':
        y = F.gelu(y, approximate='tanh')
    rec['output'] = bool(torch.equal(y, y_ref.reshape(M, -1)))
    return rec


def layer_records(seen, layers):
    """Bit-exactness record of every hooked layer (see the module docstring)."""
    from yanlongvla_b200 import definition as D
    from yanlongvla_b200 import kernels as K
    from yanlongvla_b200 import modules
    out = {}
    with torch.no_grad():
        for name, (mod, x, kwargs, y_ref) in seen.items():
            if isinstance(mod, modules.RefLinear):
                out[name] = _w2a8_record(K, D, layers[name], mod, x, y_ref)
            else:
                out[name] = _w8a8_record(K, D, mod, x, kwargs, y_ref)
    torch.cuda.synchronize()
    return out


def failures(records):
    return {name: [k for k, v in r.items() if v is False] for name, r in records.items()
            if any(v is False for v in r.values())}


def chunk_error(a, a_ref):
    """Per observation: (max |a - a_ref| / RMS(a_ref), cosine(a, a_ref)) over the flattened chunk."""
    d = (a.double() - a_ref.double()).flatten(1)
    r = a_ref.double().flatten(1)
    rms = r.pow(2).mean(dim=1).sqrt()
    max_rel = d.abs().amax(dim=1) / rms
    cos = F.cosine_similarity(a.double().flatten(1), r, dim=1)
    return max_rel, cos


def within_tolerance(a, a_ref):
    max_rel, cos = chunk_error(a, a_ref)
    return bool((max_rel <= MAX_ABS_OVER_RMS).all() and (cos >= MIN_COSINE).all()), max_rel, cos
