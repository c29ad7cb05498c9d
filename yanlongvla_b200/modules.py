"""Quantized nn.Linear replacements backed by the sm_100a kernels: the reference's module-level operator API.

Public surface (ForeverBlue816/yanlongvla, deploy/tcq_kernels/modules.py:3-12, 158-320): `install(model, layers,
runtime)` puts a kernel module in place of every nn.Linear named in `layers` ({name: tcq_format.Layer}); `KLinear`,
`KGatedMLP`, `KPlainMLP` and `RefLinear` are those modules; `decode_chunk(model)` re-decodes the per-chunk layers.
The reference's pi0.5 checkpoint loader is not part of it: callers pass their layers.

Runtimes:
  reference  the definition in PyTorch ops (`definition.linear`), independent of this library: for comparisons only
  resident   operating point (i): every layer decoded once at install and held as INT8
  fly        operating point (ii): the 2-bit stream decoded inside every product
  hybrid     operating point (iii): layers whose name contains one of `chunk_parts` are decoded once per action
             chunk by decode_chunk, the others run on the fly

Layers that read one tensor with one set of input signs (q / k / v, gate / up) form a Group: one rotation +
quantization and one product serve all of them, and each member module returns its column slice.

Product dispatch is per call, by token count M (the reference decides by model part instead), from B200 timings of
the products, which all give the same bits:
  M <= SIMT_MAX_M                      SIMT products on q4 words: the fused trellis decode-GEMV, or the INT8-resident
                                       GEMV; FP32 scaled output
  M <= TC_MAX_M, 2-bit stream          tcgen05 decode-GEMM with the trellis decode fused; FP32 scaled output (also up
                                       to TC_WIDE_MAX_M tokens on products of at most TC_WIDE_MAX_TILES channel tiles)
  otherwise                            tcgen05 INT8 GEMM on resident INT8 weights, or on weights decoded just before
                                       into a temporary; INT32 accumulators, scaled by the post
"""
import torch

from . import definition
from . import kernels as K

RUNTIMES = ('reference', 'resident', 'fly', 'hybrid')
GROUPS = (('q_proj', 'k_proj', 'v_proj'), ('gate_proj', 'up_proj'))
STATS = dict(group_runs=0, regroup_misses=0, fused_mlps=0)
FUSE = dict(post3=True, mlp=True, split=True, chain=True, pre_gemv=True)
SIMT_MAX_M = 4
TC_MAX_M = 32               # 2-bit stream: the tensor-core decode-GEMM for up to this many tokens,
TC_WIDE_MAX_M = 160         # and for up to this many when the product has at most TC_WIDE_MAX_TILES 128-channel tiles
TC_WIDE_MAX_TILES = 24      # (enough K splits per tile to spread the decode over the SMs)
FLOAT_MAX_M = 16            # W2 float path: fused FP32 products up to this many tokens, BF16 GEMM above
_NO_BOUND = 1 << 30         # layer-boundary slot of a group with fewer than three members


class Deferred:
    """A product whose post (scale epilogue, output rotation, signs, bias) has not run: the policy's block boundary
    fuses it with the residual add, the norm and the next layer's pre (kernels.chain). `tensor()` runs the post
    instead and returns the BF16 output."""
    def __init__(self, group, acc, b, in_shape):
        self.group, self.acc, self.b, self.in_shape = group, acc, b, in_shape

    def post_args(self):
        """Keyword arguments of kernels.chain that describe the pending post."""
        g = self.group
        if self.acc.dtype == torch.float32:                   # fused products: scales already applied
            return dict(acc=self.acc, s=None, rs=None, sv=g.sv, bias=g.bias)
        return dict(acc=self.acc, s=self.b['scale'], rs=g.rs, sv=g.sv, bias=g.bias)

    def tensor(self):
        return self.group.posts(self.acc, self.b, self.in_shape)[0]


class QAct:
    """A group input that a fused chain already rotated and quantized into the group's buffers (q or q4, scale): the
    group skips its own pre. `shape` is the shape of the activation it stands for."""
    def __init__(self, b, shape):
        self.b, self.shape = b, shape


def _concat(tensors):
    return torch.cat(list(tensors)).contiguous()


class Group:
    """Layers sharing their input and input signs: one rotation + quantization, one product over the concatenated
    output rows, then one post per member (or one launch for all three of q / k / v).

    mode: 'fly' (2-bit stream in the products), 'resident' (INT8 decoded at construction) or 'chunk' (INT8 decoded
    at construction and again by decode()). a8=False: the W2 float operating point (BF16 activations in the rotated
    space, FP32 accumulation)."""
    def __init__(self, layers, mode, act='gelu', a8=True):
        lead = layers[0]
        odd = [L.name for L in layers if L.n != lead.n or not torch.equal(L.su, lead.su)]
        if odd:
            raise ValueError(f'layers {odd} do not share the input width and signs of {lead.name}')
        self.layers, self.mode, self.act, self.a8 = list(layers), mode, act, a8
        self.K, self.su = lead.n, lead.su
        self.N = [L.m for L in layers]
        edges = [0]
        for m in self.N:
            edges.append(edges[-1] + m)
        self.col0, self.Ntot = edges[:-1], edges[-1]
        self.rs = _concat(L.rs for L in layers)
        self.sv = _concat(L.sv for L in layers)
        self.bias = _concat(L.bias for L in layers) if lead.bias is not None else None
        self.t8 = _concat(L.t8.reshape(-1) for L in layers)
        self.bits = _concat(L.bits for L in layers) if mode != 'resident' else None
        # tile rows where the next member's table starts (the kernels take two boundaries)
        inner = [e // 16 for e in edges[1:-1]]
        self.bounds = (inner + [_NO_BOUND, _NO_BOUND])[:2]
        # the tensor-core decode-GEMM switches tables only at its 128-row tiles
        self.tc_ok = all(e % 8 == 0 for e in inner)
        self.W = None
        if mode in ('resident', 'chunk'):
            self.W = self.decode(torch.empty(self.Ntot, self.K, dtype=torch.int8, device=lead.su.device))
        if not a8:
            self.tb = [L.t8.to(torch.bfloat16).contiguous() for L in layers]   # BF16 values of the INT8 tables
        self.defer = False          # single-layer groups: return a Deferred instead of running the post
        self._share = None          # (input, outputs, members not yet handed their output)

    # ---------------------------------------------------------------------------------------- weights and inputs
    def decode(self, W=None):
        """Decode every member's stream into its rows of W (Ntot, K) int8 (the group's resident copy when W is None)."""
        if W is None:
            W = self.W
        for L, c in zip(self.layers, self.col0):
            K.decode(L.bits, L.t8, W.narrow(0, c, L.m))
        return W

    def prep(self, x):
        """x (..., K) -> a contiguous (M, K) BF16 / F16 / F32 matrix for the pre."""
        x2 = x.reshape(-1, self.K)
        if x2.dtype not in (torch.bfloat16, torch.float16, torch.float32):
            x2 = x2.float()
        return x2.contiguous()

    def buffers(self, M, dev):
        """Quantized-activation buffers in the layout this group's product reads for M tokens: q4 words (K/4, M) for
        the SIMT products, q (M, K) for the tensor-core ones; scale (M,) either way."""
        b = dict(scale=torch.empty(M, dtype=torch.float32, device=dev))
        if M <= SIMT_MAX_M:
            b['q4'] = torch.empty(self.K // 4, M, dtype=torch.int32, device=dev)
        else:
            b['q'] = torch.empty(M, self.K, dtype=torch.int8, device=dev)
        return b

    def quantize(self, x2):
        b = self.buffers(x2.shape[0], x2.device)
        K.pre(x2, self.su, **b)
        return b

    def input(self, x):
        """Quantized input buffers: those of a QAct as they are, a tensor rotated + quantized here."""
        return x.b if isinstance(x, QAct) else self.quantize(self.prep(x))

    # ---------------------------------------------------------------------------------------- products
    def _fp32_out(self, M, dev):
        return torch.empty(M, self.Ntot, dtype=torch.float32, device=dev)

    def product(self, b):
        """Product of quantized inputs b: FP32 z = ((float)acc * s) * rs (M, Ntot) from the fused products, INT32
        accumulators (M, Ntot) from the INT8 GEMM."""
        if 'q4' in b:
            q4 = b['q4']
            z = self._fp32_out(q4.shape[1], q4.device)
            if self.W is None:
                K.gemm_tcq(self.bits, self.t8, q4, b['scale'], self.rs, z, self.K, self.bounds)
            else:
                K.gemm_w8(self.W, q4, b['scale'], self.rs, z)
            return z
        q = b['q']
        M = q.shape[0]
        if self.W is None and self.tc_ok and (M <= TC_MAX_M or (M <= TC_WIDE_MAX_M and -(-self.Ntot // 128) <= TC_WIDE_MAX_TILES)):
            z = self._fp32_out(q.shape[0], q.device)
            K.gemm_tcq_tc(self.bits, self.t8, q, b['scale'], self.rs, z, self.K, self.bounds)
            return z
        W = self.W
        if W is None:                                          # fly, many tokens: decode into a temporary first
            W = self.decode(torch.empty(self.Ntot, self.K, dtype=torch.int8, device=q.device))
        return K.int_mm(q, W)

    def acc(self, x):
        """(accumulator, quantized-input buffers) of the group's product on x. A tensor of at most
        kernels.GEMV_X_MAX_M tokens on the 2-bit stream takes the decode-GEMV with the pre fused (one launch)."""
        if FUSE['pre_gemv'] and not isinstance(x, QAct) and self.W is None and self.K <= K.GEMV_X_MAX_K:
            x2 = self.prep(x)
            M = x2.shape[0]
            if M <= min(SIMT_MAX_M, K.GEMV_X_MAX_M):
                z = self._fp32_out(M, x2.device)
                K.gemm_tcq_x(self.bits, self.t8, x2, self.su, self.rs, z, self.K, self.bounds)
                return z, dict(scale=None)
        b = self.input(x)
        return self.product(b), b

    # ---------------------------------------------------------------------------------------- posts
    def posts(self, acc, b, shape):
        """BF16 outputs of every member from the product's accumulators, shaped like the input with each member's
        width. FP32 z already carries the scales; INT32 accumulators take the token and row scales here."""
        M = acc.shape[0]
        fused = acc.dtype == torch.float32
        s = None if fused else b['scale']
        ys = [torch.empty(M, n, dtype=torch.bfloat16, device=acc.device) for n in self.N]
        if len(ys) == 3 and (FUSE['split'] and fused or FUSE['post3']):
            # q / k / v in one launch: for few tokens one block per (token, layer), else one block per token
            launch = K.postg if (FUSE['split'] and fused) else K.post3
            launch(acc, s, None if fused else self.rs, self.sv, self.bias, ys)
        else:
            for L, c, y in zip(self.layers, self.col0, ys):
                K.post(acc, s, None if fused else L.rs, L.sv, L.bias, y, col0=c)
        lead = tuple(shape[:-1])
        return [y.view(*lead, y.shape[1]) for y in ys]

    def run_float(self, x2, shape):
        """W2 (the reference's modules.py:117-145): rotated activations rounded to BF16, INT8-table weights. Few
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

    def run(self, x):
        """Outputs of every member on input x (a list; one Deferred for a deferring single-layer group)."""
        if not self.a8:
            return self.run_float(self.prep(x), x.shape)
        acc, b = self.acc(x)
        STATS['group_runs'] += 1
        return [Deferred(self, acc, b, x.shape)] if self.defer else self.posts(acc, b, x.shape)

    def get(self, x, index):
        """Member `index`'s output on x. The first member to ask runs the whole group; the run is kept until every
        member has taken its output, and an input other than the kept one before then counts as a regroup miss."""
        share = self._share
        if share is None or share[0] is not x:
            if share is not None:
                STATS['regroup_misses'] += 1
            share = self._share = (x, self.run(x), set(range(len(self.layers))))
        _, outs, owed = share
        owed.discard(index)
        if not owed:
            self._share = None
        return outs[index]


class KLinear(torch.nn.Module):
    """Replacement of one quantized nn.Linear (the reference's modules.py:158-167): forwards to its Group, `shared`,
    which is a plain object and so stays out of the module tree."""
    def __init__(self, group, index):
        super().__init__()
        L = group.layers[index]
        self.shared, self.index = group, index
        self.in_features, self.out_features, self.layer_name = L.n, L.m, L.name
        # callers that probe `module.weight.dtype` see BF16; the tensor itself holds nothing
        self.register_buffer('weight', torch.empty(0, dtype=torch.bfloat16, device=L.su.device), persistent=False)

    def forward(self, x):
        return self.shared.get(x, self.index)


class KGatedMLP(torch.nn.Module):
    """down(act(gate(x)) * up(x)) with its middle fused (the reference's modules.py:170-189); act = 'gelu' (tanh
    form) or 'silu' (SwiGLU). Launches: pre (or a fused chain), gate|up product, middle (posts + activation + product +
    the down projection's pre), down product, post (or a deferred post)."""
    def __init__(self, gate_up, down, act='gelu'):
        super().__init__()
        self.groups, self.act, self.defer = [gate_up, down], act, False
        self.gate_proj, self.up_proj, self.down_proj = KLinear(gate_up, 0), KLinear(gate_up, 1), KLinear(down, 0)

    def forward(self, x):
        first, second = self.groups
        acc, b = first.acc(x)
        M, dev = acc.shape[0], acc.device
        nxt = second.buffers(M, dev)
        fused = acc.dtype == torch.float32
        if fused and FUSE['split']:
            # few tokens: the gate and up posts as parallel blocks (activation on the gate), then the product and
            # the down projection's pre
            gate = torch.empty(M, first.N[0], dtype=torch.bfloat16, device=dev)
            up = torch.empty_like(gate)
            K.postg(acc, None, None, first.sv, None, [gate, up], gelu0=True, act=self.act)
            K.pre2(gate, up, second.su, **nxt)
        else:
            K.mid2(acc, None if fused else b['scale'], None if fused else first.rs, first.sv, second.su, act=self.act, **nxt)
        STATS['fused_mlps'] += 1
        acc2 = second.product(nxt)
        if self.defer:
            return Deferred(second, acc2, nxt, x.shape)
        return second.posts(acc2, nxt, x.shape)[0]


class KPlainMLP(torch.nn.Module):
    """fc2(act(fc1(x))) with its middle fused (the reference's modules.py:192-206)."""
    def __init__(self, fc1, fc2, act='gelu'):
        super().__init__()
        self.groups, self.act, self.defer = [fc1, fc2], act, False
        self.fc1, self.fc2 = KLinear(fc1, 0), KLinear(fc2, 0)

    def forward(self, x):
        first, second = self.groups
        acc, b = first.acc(x)
        fused = acc.dtype == torch.float32
        nxt = second.buffers(acc.shape[0], acc.device)
        K.mid1(acc, None if fused else b['scale'], None if fused else first.rs, first.sv, first.bias, second.su,
               act=self.act, **nxt)
        STATS['fused_mlps'] += 1
        acc2 = second.product(nxt)
        if self.defer:
            return Deferred(second, acc2, nxt, x.shape)
        return second.posts(acc2, nxt, x.shape)[0]


class RefLinear(torch.nn.Module):
    """The W2A8 layer by definition in PyTorch ops (`definition.linear`, the reference's modules.py:209-219): the
    'reference' runtime, used to compare against; it calls nothing of the kernel library. The INT8 weights are
    decoded once at construction by the PyTorch-ops decoder, or given (w8, e.g. decoded by an independent checker).
    a8=False: FP32 activations in the rotated space with the same weights, product in float64."""
    def __init__(self, layer, a8=True, w8=None):
        super().__init__()
        self.a8 = a8
        self.layer = [layer]        # a list: the layer object stays out of the module tree
        self.w8 = definition.decode_w8(layer.bits, layer.t8, layer.m, layer.n) if w8 is None else w8
        self.in_features, self.out_features, self.layer_name = layer.n, layer.m, layer.name
        self.register_buffer('weight', torch.empty(0, dtype=torch.bfloat16, device=layer.su.device), persistent=False)

    def forward(self, x):
        return definition.linear(x, self.layer[0], self.w8, a8=self.a8)


# ------------------------------------------------------------------------------------------------ policy surgery
def set_submodule(model, name, module):
    """Replace the submodule at dotted path `name` by `module`."""
    owner, _, attr = name.rpartition('.')
    setattr(model.get_submodule(owner) if owner else model, attr, module)


def _plan_groups(layers):
    """Partition the layer names into groups: within one parent module, the members of a GROUPS pattern that are all
    present with one input width and one set of input signs form a group; every other layer is alone. Returns
    lists of names, each in pattern order."""
    by_parent = {}
    for name in layers:
        owner, _, leaf = name.rpartition('.')
        by_parent.setdefault(owner, {})[leaf] = name
    plans = []
    for owner, leaves in by_parent.items():
        claimed = set()
        for pattern in GROUPS:
            if not all(leaf in leaves for leaf in pattern):
                continue
            first = layers[leaves[pattern[0]]]
            if all(layers[leaves[leaf]].n == first.n and torch.equal(layers[leaves[leaf]].su, first.su) for leaf in pattern):
                plans.append([leaves[leaf] for leaf in pattern])
                claimed.update(pattern)
        plans.extend([name] for leaf, name in leaves.items() if leaf not in claimed)
    return plans


def install(model, layers, runtime='fly', chunk_parts=('action_head',), mlp_acts=None, a8=True, ref_w8=None):
    """Put kernel modules in place of the nn.Linear modules named in `layers` ({name: tcq_format.Layer}) (the
    reference's modules.py:246-311). a8=False installs the W2 float operating point (BF16 rotated activations; MLP
    middles stay unfused). mlp_acts: {MLP module name: 'gelu' | 'silu'} of the MLPs whose middles are fused (children
    gate_proj / up_proj / down_proj, or fc1 / fc2); MLPs not listed keep their own forward and call their KLinear
    members one by one. ref_w8 (runtime 'reference' only): {name: decoded INT8 weights} to use instead of the
    PyTorch-ops decode. Returns an info dict (groups, shared rotations, fused MLPs)."""
    if runtime not in RUNTIMES:
        raise ValueError(f'runtime {runtime!r} is not one of {RUNTIMES}')
    for name in layers:
        m = model.get_submodule(name)
        if not (hasattr(m, 'in_features') and hasattr(m, 'out_features')):
            raise TypeError(f'{name} is {type(m).__name__}, not a Linear')
    info = dict(runtime=runtime, layers=len(layers), a8=a8)
    if runtime == 'reference':
        for name, L in layers.items():
            set_submodule(model, name, RefLinear(L, a8=a8, w8=(ref_w8 or {}).get(name)))
        return info
    groups = []
    for names in _plan_groups(layers):
        per_chunk = runtime == 'hybrid' and any(part in names[0] for part in chunk_parts)
        mode = {'resident': 'resident'}.get(runtime, 'chunk' if per_chunk else 'fly')
        group = Group([layers[n] for n in names], mode, a8=a8)
        for i, n in enumerate(names):
            set_submodule(model, n, KLinear(group, i))
        groups.append(group)
    fused = 0
    if FUSE['mlp'] and mlp_acts and a8:
        lead_of = {g.layers[0].name: g for g in groups}
        for mlp, act in mlp_acts.items():
            pre = f'{mlp}.' if mlp else ''
            gate, down = lead_of.get(f'{pre}gate_proj'), lead_of.get(f'{pre}down_proj')
            fc1, fc2 = lead_of.get(f'{pre}fc1'), lead_of.get(f'{pre}fc2')
            if gate is not None and len(gate.layers) == 2 and down is not None:
                set_submodule(model, mlp, KGatedMLP(gate, down, act))
            elif fc1 is not None and fc2 is not None:
                set_submodule(model, mlp, KPlainMLP(fc1, fc2, act))
            else:
                continue
            fused += 1
    model._tcq_groups = groups
    modes = {m: sum(g.mode == m for g in groups) for m in ('resident', 'fly', 'chunk')}
    info.update(groups=len(groups), shared_rotations=len(layers) - len(groups), fused_mlps=fused, modes=modes)
    return info


def decode_chunk(model):
    """Operating point (iii), once per action chunk: decode the per-chunk groups into their INT8 weights (the
    reference's modules.py:314-320). Returns the number of layers decoded."""
    chunk = [g for g in getattr(model, '_tcq_groups', ()) if g.mode == 'chunk']
    for g in chunk:
        g.decode()
    return sum(len(g.layers) for g in chunk)
