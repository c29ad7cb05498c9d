"""Model integration: quantized nn.Linear replacements backed by the sm_100a kernels.

Mirrors deploy/tcq_kernels/modules.py of the reference (ForeverBlue816/yanlongvla): the same classes and runtimes,
without its pi0.5-specific loader. `install(model, layers, runtime)` swaps every nn.Linear named in `layers`
({name: tcq_format.Layer}) for a kernel-backed module.

Runtimes (modules.py:3-8):
  reference  the W2A8 definition in PyTorch ops on the device (RefLinear), for comparisons only
  resident   operating point (i): every layer decoded once at install, weights held as INT8
  fly        operating point (ii): the 2-bit stream is decoded on every call (fused into the product for few tokens)
  hybrid     operating point (iii): layers whose name matches `chunk_parts` are decoded once per action chunk
             (decode_chunk), the rest on the fly

Token-count dispatch. The reference chooses the product by model part (action expert = few tokens). Here the group
chooses per call, from B200 measurements of the three products: M <= SIMT_MAX_M tokens run the SIMT products on q4
words (fused trellis decode-GEMV, or the INT8-resident GEMV), FP32 scaled output; M <= TC_MAX_M tokens with the
2-bit stream run the tensor-core fused decode-GEMM (FP32 scaled output); larger M, or INT8-resident weights, run the
tcgen05 INT8 GEMM (INT32 accumulators) on resident or freshly decoded INT8 weights. All give bit-identical results.

Layers that read the same tensor with identical input signs share one rotation + quantization and one product
(q / k / v; gate / up): the group runs on the first member's call and the others return their slice (modules.py:10-12).
"""
import math

import torch

from . import kernels as K

RUNTIMES = ('reference', 'resident', 'fly', 'hybrid')
GROUPS = (('q_proj', 'k_proj', 'v_proj'), ('gate_proj', 'up_proj'))
STATS = dict(group_runs=0, regroup_misses=0, fused_mlps=0)
FUSE = dict(post3=True, mlp=True, split=True, chain=True, pre_gemv=True)
SIMT_MAX_M = 4
TC_MAX_M = 32
FLOAT_MAX_M = 16            # W2 float path: fused FP32 products up to this many tokens, BF16 GEMM above


class Deferred:
    """Output of a single-layer group (or fused MLP) whose post has not run yet, for a consumer that fuses it with
    what follows (the policy's residual add + norm + next pre, kernels.chain). `tensor()` runs the post instead."""
    def __init__(self, group, acc, b, in_shape):
        self.group, self.acc, self.b, self.in_shape = group, acc, b, in_shape

    def post_args(self):
        g, small = self.group, self.acc.dtype == torch.float32
        return dict(acc=self.acc, s=None if small else self.b['scale'], rs=None if small else g.rs, sv=g.sv, bias=g.bias)

    def tensor(self):
        return self.group.posts(self.acc, self.b, self.in_shape)[0]


class QAct:
    """A group input already rotated and quantized into the group's buffers (q or q4, scale) by a fused chain: the
    group skips its own pre. `shape` is the shape of the activation it stands for."""
    def __init__(self, b, shape):
        self.b, self.shape = b, shape


class Group:
    """One or more layers sharing the input (and its signs): one rotation + quantization, one product.
    a8=False: the W2 float operating point (BF16 activations in the rotated space, FP32 / BF16 products)."""
    def __init__(self, layers, mode, act='gelu', a8=True):
        self.layers, self.mode, self.act, self.a8 = layers, mode, act, a8
        self.K = layers[0].n
        for L in layers:
            if L.n != self.K or not torch.equal(L.su, layers[0].su):
                raise ValueError(f'layers {[x.name for x in layers]} do not share their input signs')
        self.su = layers[0].su
        self.N = [L.m for L in layers]
        self.col0 = [sum(self.N[:i]) for i in range(len(layers))]
        self.Ntot = sum(self.N)
        dev = self.su.device
        self.rs = torch.cat([L.rs for L in layers]).contiguous()
        self.sv = torch.cat([L.sv for L in layers]).contiguous()
        self.bias = torch.cat([L.bias for L in layers]).contiguous() if layers[0].bias is not None else None
        self.t8 = torch.cat([L.t8.reshape(-1) for L in layers]).contiguous()
        self.bits = torch.cat([L.bits for L in layers]).contiguous() if mode != 'resident' else None
        self.bounds = [c // 16 for c in self.col0[1:]] + [1 << 30] * (3 - len(layers))
        self.tc_ok = all(b % 8 == 0 for b in self.bounds[:len(layers) - 1])   # layer bounds on 128-row tiles
        self.W = None
        if mode in ('resident', 'chunk'):
            self.W = torch.empty(self.Ntot, self.K, dtype=torch.int8, device=dev)
            self.decode()
        if not a8:
            self.tb = [L.t8.to(torch.bfloat16).contiguous() for L in layers]   # BF16 values of the INT8 tables
        self.x = self.outs = None
        self.served = 0
        self.defer = False          # single-layer groups: return a Deferred instead of running the post

    def decode(self, W=None):
        """Dense INT8 weights of the group (rotated basis) into W (Ntot, K)."""
        W = self.W if W is None else W
        for L, c in zip(self.layers, self.col0):
            K.decode(L.bits, L.t8, W[c:c + L.m])
        return W

    def prep(self, x):
        x2 = x.reshape(-1, self.K)
        if not x2.is_contiguous():
            x2 = x2.contiguous()
        if x2.dtype not in (torch.bfloat16, torch.float16, torch.float32):
            x2 = x2.float()
        return x2

    def buffers(self, M, dev):
        """Quantized-activation buffer in the layout of this group's product, and the per-token scales."""
        s = torch.empty(M, dtype=torch.float32, device=dev)
        if M <= SIMT_MAX_M:
            return dict(q4=torch.empty(self.K // 4, M, dtype=torch.int32, device=dev), scale=s)
        return dict(q=torch.empty(M, self.K, dtype=torch.int8, device=dev), scale=s)

    def quantize(self, x2):
        b = self.buffers(x2.shape[0], x2.device)
        K.pre(x2, self.su, **b)
        return b

    def product(self, b):
        """INT8 activations -> FP32 z = ((float)acc * s) * rs (M, Ntot) on the fused paths, INT32 acc (M, Ntot) on the
        tcgen05 INT8 GEMM path."""
        if 'q' in b:
            M = b['q'].shape[0]
            if self.W is None and M <= TC_MAX_M and self.tc_ok:
                z = torch.empty(M, self.Ntot, dtype=torch.float32, device=b['q'].device)
                K.gemm_tcq_tc(self.bits, self.t8, b['q'], b['scale'], self.rs, z, self.K, self.bounds)
                return z
            W = self.W if self.W is not None else self.decode(torch.empty(self.Ntot, self.K, dtype=torch.int8, device=b['q'].device))
            return K.int_mm(b['q'], W)
        M = b['q4'].shape[1]
        z = torch.empty(M, self.Ntot, dtype=torch.float32, device=b['q4'].device)
        if self.W is not None:
            K.gemm_w8(self.W, b['q4'], b['scale'], self.rs, z)
        else:
            K.gemm_tcq(self.bits, self.t8, b['q4'], b['scale'], self.rs, z, self.K, self.bounds)
        return z

    def posts(self, acc, b, shape):
        M, dev = acc.shape[0], acc.device
        ys = [torch.empty(M, n, dtype=torch.bfloat16, device=dev) for n in self.N]
        small = acc.dtype == torch.float32
        s, rs = (None, None) if small else (b['scale'], self.rs)
        if len(ys) == 3 and small and FUSE['split']:
            K.postg(acc, s, rs, self.sv, self.bias, ys)            # few tokens: the three layers on different SMs at once
        elif len(ys) == 3 and FUSE['post3']:
            K.post3(acc, s, rs, self.sv, self.bias, ys)
        else:
            for L, c, y in zip(self.layers, self.col0, ys):
                K.post(acc, s, None if rs is None else L.rs, L.sv, L.bias, y, col0=c)
        return [y.reshape(*shape[:-1], n) for y, n in zip(ys, self.N)]

    def input(self, x):
        """Quantized input buffers: a QAct's as they are, a tensor rotated + quantized here."""
        return x.b if isinstance(x, QAct) else self.quantize(self.prep(x))

    def run_float(self, x2, shape):
        """W2 (modules.py:117-145 of the reference): rotated activations rounded to BF16, INT8-table weights. Few
        tokens: the fused FP32-accumulating products on hT; more: BF16 decode + BF16 tensor-core product (cuBLAS) with
        FP32 output (the reference rounds this accumulator to BF16; keeping FP32 stays closer to the definition)."""
        M, dev, outs = x2.shape[0], x2.device, []
        if M > FLOAT_MAX_M:
            h = torch.empty(M, self.K, dtype=torch.bfloat16, device=dev)
            K.pre_h(x2, self.su, h=h)
            W = torch.empty(self.Ntot, self.K, dtype=torch.bfloat16, device=dev)
            for L, c, tb in zip(self.layers, self.col0, self.tb):
                K.decode_bf16(L.bits, tb, W[c:c + L.m])
            z = torch.mm(h, W.t(), out_dtype=torch.float32) * self.rs[None, :]
            for L, c in zip(self.layers, self.col0):
                y = torch.empty(M, L.m, dtype=torch.bfloat16, device=dev)
                K.post(z, None, None, L.sv, L.bias, y, col0=c)
                outs.append(y.reshape(*shape[:-1], L.m))
        else:
            hT = torch.empty(self.K, M, dtype=torch.bfloat16, device=dev)
            K.pre_h(x2, self.su, hT=hT)
            z = torch.empty(M, self.Ntot, dtype=torch.float32, device=dev)
            if self.W is not None:
                K.gemmf_w8(self.W, hT, self.rs, z)
            else:
                K.gemmf_tcq(self.bits, self.t8, hT, self.rs, z, self.K, self.bounds)
            for L, c in zip(self.layers, self.col0):
                y = torch.empty(M, L.m, dtype=torch.bfloat16, device=dev)
                K.post(z, None, None, L.sv, L.bias, y, col0=c)
                outs.append(y.reshape(*shape[:-1], L.m))
        STATS['group_runs'] += 1
        return outs

    def acc(self, x):
        """Accumulator of the group's product and its quantized-input buffers. A tensor input of at most
        kernels.GEMV_X_MAX_M tokens on the 2-bit stream takes the decode-GEMV with the pre fused (one launch)."""
        if (FUSE['pre_gemv'] and not isinstance(x, QAct) and self.W is None and self.K <= K.GEMV_X_MAX_K):
            x2 = self.prep(x)
            M = x2.shape[0]
            if M <= min(SIMT_MAX_M, K.GEMV_X_MAX_M):
                z = torch.empty(M, self.Ntot, dtype=torch.float32, device=x2.device)
                K.gemm_tcq_x(self.bits, self.t8, x2, self.su, self.rs, z, self.K, self.bounds)
                return z, dict(scale=None)
        b = self.input(x)
        return self.product(b), b

    def run(self, x):
        if not self.a8:
            return self.run_float(self.prep(x), x.shape)
        acc, b = self.acc(x)
        STATS['group_runs'] += 1
        if self.defer:
            return [Deferred(self, acc, b, x.shape)]
        return self.posts(acc, b, x.shape)

    def get(self, x, index):
        if self.x is not x:
            if self.x is not None:
                STATS['regroup_misses'] += 1
            self.outs = self.run(x)
            self.x = x
            self.served = 0
        out = self.outs[index]
        self.served += 1
        if self.served == len(self.layers):
            self.x = self.outs = None
        return out


class KLinear(torch.nn.Module):
    """Kernel-backed replacement of one quantized nn.Linear (modules.py:158-167)."""
    def __init__(self, group, index):
        super().__init__()
        self.group, self.index = [group], index                 # list: keep the group out of the module tree
        L = group.layers[index]
        self.in_features, self.out_features, self.layer_name = L.n, L.m, L.name
        self.register_buffer('weight', torch.empty(0, dtype=torch.bfloat16, device=L.su.device), persistent=False)

    def forward(self, x):
        return self.group[0].get(x, self.index)


class KGatedMLP(torch.nn.Module):
    """down(act(gate(x)) * up(x)) with the middle fused (modules.py:170-189): rotate+quantize, product, middle, product,
    scale+rotate. act = 'gelu' (tanh, Gemma) or 'silu' (SwiGLU)."""
    def __init__(self, gate_up, down, act='gelu'):
        super().__init__()
        self.groups = [gate_up, down]
        self.act = act
        self.defer = False
        self.gate_proj, self.up_proj, self.down_proj = KLinear(gate_up, 0), KLinear(gate_up, 1), KLinear(down, 0)

    def forward(self, x):
        gu, down = self.groups
        acc, b = gu.acc(x)
        M = acc.shape[0]
        b2 = down.buffers(M, acc.device)
        small = acc.dtype == torch.float32
        if small and FUSE['split']:                              # few tokens: gate and up in parallel blocks
            g = torch.empty(M, gu.N[0], dtype=torch.bfloat16, device=acc.device)
            u = torch.empty_like(g)
            K.postg(acc, None, None, gu.sv, None, [g, u], gelu0=True, act=self.act)
            K.pre2(g, u, down.su, **b2)
        else:
            K.mid2(acc, None if small else b['scale'], None if small else gu.rs, gu.sv, down.su, act=self.act, **b2)
        STATS['fused_mlps'] += 1
        acc2 = down.product(b2)
        return Deferred(down, acc2, b2, x.shape) if self.defer else down.posts(acc2, b2, x.shape)[0]


class KPlainMLP(torch.nn.Module):
    """fc2(act(fc1(x))) with the middle fused (modules.py:192-206)."""
    def __init__(self, fc1, fc2, act='gelu'):
        super().__init__()
        self.groups = [fc1, fc2]
        self.act = act
        self.defer = False
        self.fc1, self.fc2 = KLinear(fc1, 0), KLinear(fc2, 0)

    def forward(self, x):
        g1, g2 = self.groups
        acc, b = g1.acc(x)
        small = acc.dtype == torch.float32
        b2 = g2.buffers(acc.shape[0], acc.device)
        K.mid1(acc, None if small else b['scale'], None if small else g1.rs, g1.sv, g1.bias, g2.su, act=self.act, **b2)
        STATS['fused_mlps'] += 1
        acc2 = g2.product(b2)
        return Deferred(g2, acc2, b2, x.shape) if self.defer else g2.posts(acc2, b2, x.shape)[0]


# ------------------------------------------------------------------------------------------------ definition runtime
def _fwht(x):
    """Block Walsh of the reference definition in PyTorch ops (tcq_format.py:44-55), FP32."""
    outs, off = [], 0
    for w in _widths(x.shape[-1]):
        y, h = x[..., off:off + w], 1
        while h < w:
            y = y.reshape(*y.shape[:-1], w // (2 * h), 2, h)
            y = torch.stack((y[..., 0, :] + y[..., 1, :], y[..., 0, :] - y[..., 1, :]), dim=-2).reshape(*y.shape[:-3], w)
            h *= 2
        outs.append(y * _scale(w, x.device))
        off += w
    return torch.cat(outs, -1) if len(outs) > 1 else outs[0]


_SCALES = {}


def _scale(w, device):
    """FP32 constant 1 / sqrt(w) on the device, created once (tcq_format.py:36-41)."""
    key = (w, str(device))
    if key not in _SCALES:
        _SCALES[key] = torch.tensor(1.0 / math.sqrt(w), dtype=torch.float32, device=device)
    return _SCALES[key]


def _widths(width):
    out = []
    while width:
        b = 1 << (width.bit_length() - 1)
        out.append(b)
        width -= b
    return out


class RefLinear(torch.nn.Module):
    """W2A8 by definition in PyTorch ops on the device (modules.py:209-219): the 'reference' runtime, used only to
    compare against; the kernel runtimes never call it. Weights decoded once by the decode kernel. a8=False: the same
    INT8-table weights with FP32 activations (tcq_format.py:137-138), product in float64."""
    def __init__(self, layer, a8=True):
        super().__init__()
        self.a8 = a8
        self.layer = [layer]
        self.w8 = layer.w8()
        self.in_features, self.out_features, self.layer_name = layer.n, layer.m, layer.name
        self.register_buffer('weight', torch.empty(0, dtype=torch.bfloat16, device=layer.su.device), persistent=False)

    def forward(self, x):
        L = self.layer[0]
        shape = x.shape
        h = _fwht(x.float().reshape(-1, shape[-1]) * L.su.float())
        if not self.a8:
            y = _fwht((h.double() @ self.w8.double().t()).float() * L.rs[None, :]) * L.sv.float()
            if L.bias is not None:
                y = y + L.bias
            return y.to(torch.bfloat16).reshape(*shape[:-1], -1)
        amax = h.abs().amax(dim=1, keepdim=True)
        s = torch.where(amax > 0, amax / torch.full_like(amax, 127.0), torch.ones_like(amax))
        q = torch.clamp(torch.round(h / s), -127, 127).to(torch.int8)
        acc = K.int_mm(q, self.w8)
        y = _fwht((acc.float() * s) * L.rs[None, :]) * L.sv.float()
        if L.bias is not None:
            y = y + L.bias
        return y.to(torch.bfloat16).reshape(*shape[:-1], -1)


# ------------------------------------------------------------------------------------------------ policy surgery
def set_submodule(model, name, module):
    parent, _, leaf = name.rpartition('.')
    setattr(model.get_submodule(parent) if parent else model, leaf, module)


def install(model, layers, runtime='fly', chunk_parts=('action_head',), mlp_acts=None, a8=True):
    """Swap the nn.Linear modules named in `layers` ({name: tcq_format.Layer}) for kernel modules (modules.py:246-311).
    a8=False installs the W2 float operating point (BF16 rotated activations; MLP middles stay unfused).

    mlp_acts: {mlp module name: 'gelu' | 'silu'} of the MLPs whose middles are fused (gate_proj/up_proj/down_proj or
    fc1/fc2 children); MLPs not listed keep their own forward and call the KLinear members one by one.
    Returns an info dict (groups, shared rotations, fused MLPs)."""
    if runtime not in RUNTIMES:
        raise ValueError(runtime)
    names = list(layers)
    for name in names:
        m = model.get_submodule(name)
        if not hasattr(m, 'in_features') or not hasattr(m, 'out_features'):
            raise TypeError(f'{name} is {type(m).__name__}, not a Linear')
    info = dict(runtime=runtime, layers=len(names))
    info['a8'] = a8
    if runtime == 'reference':
        for name in names:
            set_submodule(model, name, RefLinear(layers[name], a8=a8))
        return info
    groups, done = [], set()
    for name in names:
        if name in done:
            continue
        parent, _, leaf = name.rpartition('.')
        members = [name]
        for g in GROUPS:
            if leaf in g:
                cand = [f'{parent}.{x}' if parent else x for x in g]
                if all(c in layers for c in cand) and all(layers[c].n == layers[cand[0]].n and torch.equal(layers[c].su, layers[cand[0]].su)
                                                          for c in cand):
                    members = cand
        chunk = runtime == 'hybrid' and any(p in name for p in chunk_parts)
        mode = 'resident' if runtime == 'resident' else 'chunk' if chunk else 'fly'
        group = Group([layers[n] for n in members], mode, a8=a8)
        for i, n in enumerate(members):
            set_submodule(model, n, KLinear(group, i))
            done.add(n)
        groups.append(group)
    fused = 0
    if FUSE['mlp'] and mlp_acts and a8:
        by_name = {g.layers[0].name: g for g in groups}
        for mlp, act in mlp_acts.items():
            p = f'{mlp}.' if mlp else ''
            if f'{p}gate_proj' in by_name and len(by_name[f'{p}gate_proj'].layers) == 2 and f'{p}down_proj' in by_name:
                set_submodule(model, mlp, KGatedMLP(by_name[f'{p}gate_proj'], by_name[f'{p}down_proj'], act))
                fused += 1
            elif f'{p}fc1' in by_name and f'{p}fc2' in by_name:
                set_submodule(model, mlp, KPlainMLP(by_name[f'{p}fc1'], by_name[f'{p}fc2'], act))
                fused += 1
    model._tcq_groups = groups
    info.update(groups=len(groups), shared_rotations=sum(len(g.layers) - 1 for g in groups), fused_mlps=fused,
                modes={m: sum(1 for g in groups if g.mode == m) for m in ('resident', 'fly', 'chunk')})
    return info


def decode_chunk(model):
    """Operating point (iii): decode the chunk-mode layers once per action chunk (modules.py:314-320)."""
    n = 0
    for g in getattr(model, '_tcq_groups', ()):
        if g.mode == 'chunk':
            g.decode()
            n += len(g.layers)
    return n
