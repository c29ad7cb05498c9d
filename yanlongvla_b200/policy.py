"""A GR00T-style vision-language-action policy with the W2A8 trellis path in every LLM and DiT Linear (benchmark
config 4) and W8A8 INT8 in the vision tower, random-initialised (no checkpoints travel).

Shape (benchmark config 4): ViT of 27 layers (hidden 1152, 16 heads, MLP 4304) on 2 camera images of 224 x 224 x 3
uint8 with 14 x 14 patches, pixel-shuffled to 64 tokens each; a 24-layer LLM (hidden 2048, 32 query / 8 KV heads,
SwiGLU FFN 8192) over 128 image tokens + 32 language tokens (vocab 49152); a 16-block DiT action head (hidden 1536,
32 heads, FFN 6144) alternating cross-attention to the backbone features (even blocks) and self-attention (odd
blocks), AdaLN conditioned on the flow timestep, 4 flow-matching Euler steps producing a 16 x 32 action chunk from a
64-dim state. Attention, norms, embeddings and the small input / output projections are PyTorch BF16; the quantized
Linears are `modules.KLinear` / `KGatedMLP` / `KPlainMLP` (2-bit trellis, W2A8) and `W8A8Linear` (vision).

Oracle for the whole policy: the same model with runtime='reference', as the reference does with its RefLinear
runtime (modules.py:209-219): every quantized Linear is the W2A8 / W8A8 definition in PyTorch ops (`definition`:
PyTorch-ops trellis decode, cuBLASLt INT8 products through torch._int_mm), and the norms and the rotary embedding
are PyTorch ops too. Nothing of the kernel library runs in it.
"""
import math
from dataclasses import dataclass

import torch
import torch.nn.functional as F

from . import definition
from . import kernels as K
from . import modules
from .tcq_format import Layer


@dataclass
class PolicyConfig:
    image: int = 224
    patch: int = 14
    cameras: int = 2
    vit_layers: int = 27
    vit_hidden: int = 1152
    vit_heads: int = 16
    vit_mlp: int = 4304
    shuffle: int = 2
    llm_layers: int = 24
    llm_hidden: int = 2048
    llm_heads: int = 32
    llm_kv_heads: int = 8
    llm_ffn: int = 8192
    vocab: int = 49152
    lang_tokens: int = 32
    dit_layers: int = 16
    dit_hidden: int = 1536
    dit_heads: int = 32
    dit_ffn: int = 6144
    flow_steps: int = 4
    chunk: int = 16
    action_dim: int = 32
    state_dim: int = 64

    @property
    def patches(self):
        return (self.image // self.patch) ** 2

    @property
    def image_tokens(self):
        return self.patches // (self.shuffle ** 2)

    @property
    def prefix_tokens(self):
        return self.cameras * self.image_tokens + self.lang_tokens


class LinearSlot(torch.nn.Module):
    """Placeholder of a quantized Linear: shapes only; replaced by `quantize` before the first forward."""
    def __init__(self, n_in, n_out, bias=False):
        super().__init__()
        self.in_features, self.out_features, self.has_bias = n_in, n_out, bias

    def forward(self, x):
        raise RuntimeError('quantized Linear slot used before quantize()')


class W8Act:
    """A W8A8 layer's input already quantized per token by the producing norm (kernels.chain with q but no su):
    q (M, K) int8, s (M,) FP32, shape the activation's shape."""
    def __init__(self, q, s, shape):
        self.q, self.s, self.shape = q, s, shape


class W8A8Linear(torch.nn.Module):
    """W8A8 Linear of the vision tower: per-token INT8 activations (no rotation), INT8 weights (N, K) with per-channel
    FP32 scales, exact INT32 product, y = BF16(((float)acc * s_tok) * s_ch) + bias (benchmark config 3)."""
    def __init__(self, W, s_ch, bias=None, reference=False):
        super().__init__()
        self.W, self.s_ch, self.bias, self.reference = W, s_ch, bias, reference
        self.in_features, self.out_features = W.shape[1], W.shape[0]

    def forward(self, x, act=None):
        """y = act(BF16 product + bias); act None or 'gelu' (tanh approximation). The kernel runtimes add the bias in
        the GEMM's epilogue (kernels.int8_gemm_bias, the same rounding as the PyTorch add of the reference runtime);
        the activation stays PyTorch's elementwise op (as a table lookup in the epilogue it costs more than it saves:
        the 128 KB table does not stay in L1 beside the GEMM's shared-memory stages)."""
        if isinstance(x, W8Act):
            shape = x.shape
            y = K.int8_gemm_bias(x.q, self.W, x.s, self.s_ch, bias=self.bias)
            if act == 'gelu':
                y = F.gelu(y, approximate='tanh')
            return y.reshape(*shape[:-1], -1)
        shape = x.shape
        x2 = x.reshape(-1, shape[-1]).contiguous()
        if self.reference:                                     # the definition in PyTorch ops (tcq_format.py:119-135)
            y = definition.w8a8_linear(x2, self.W, self.s_ch, self.bias)
            if act == 'gelu':
                y = F.gelu(y, approximate='tanh')
        else:
            q, s = K.quantize(x2)
            y = K.int8_gemm_bias(q, self.W, s, self.s_ch, bias=self.bias)
            if act == 'gelu':
                y = F.gelu(y, approximate='tanh')
        return y.reshape(*shape[:-1], -1)


class W8A8Group(torch.nn.Module):
    """W8A8 layers that read the same input (the vision tower's q / k / v): one GEMM over the concatenated weights,
    per-channel scales and biases; returns the layers' outputs as column views of its output. Every output element is
    computed exactly as by the layer alone."""
    def __init__(self, parts):
        super().__init__()
        self.W = torch.cat([m.W for m in parts]).contiguous()
        self.s_ch = torch.cat([m.s_ch for m in parts]).contiguous()
        self.bias = torch.cat([m.bias for m in parts]).contiguous() if parts[0].bias is not None else None
        self.sizes = [m.out_features for m in parts]

    def forward(self, x):
        shape = x.shape
        if isinstance(x, W8Act):
            y = K.int8_gemm_bias(x.q, self.W, x.s, self.s_ch, bias=self.bias)
        else:
            q, s = K.quantize(x.reshape(-1, shape[-1]).contiguous())
            y = K.int8_gemm_bias(q, self.W, s, self.s_ch, bias=self.bias)
        y = y.view(*shape[:-1], -1)
        return tuple(torch.split(y, self.sizes, dim=-1))


def _attention(q, k, v, heads, kv_heads=None, causal=False):
    """q (B, Tq, H*D), k / v (B, Tk, Hk*D) BF16 -> (B, Tq, H*D). Grouped-query heads share their K / V inside the
    attention kernel (no repeated copies)."""
    B, Tq, _ = q.shape
    Tk = k.shape[1]
    kv_heads = kv_heads or heads
    D = q.shape[-1] // heads
    q = q.view(B, Tq, heads, D).transpose(1, 2)
    k = k.view(B, Tk, kv_heads, D).transpose(1, 2)
    v = v.view(B, Tk, kv_heads, D).transpose(1, 2)
    o = F.scaled_dot_product_attention(q, k, v, is_causal=causal, enable_gqa=kv_heads != heads)
    return o.transpose(1, 2).reshape(B, Tq, heads * D)


def rope_tables(T, D, device):
    """cos / sin (T, D/2) FP32 of the half-split rotary embedding at positions 0..T-1 (computed once per forward)."""
    inv = 1.0 / (10000 ** (torch.arange(0, D, 2, device=device, dtype=torch.float32) / D))
    ang = torch.arange(T, device=device).float()[:, None] * inv[None, :]
    return ang.cos().contiguous(), ang.sin().contiguous()


def _norm(norm, kind, x, delta, weight, bias, eps, mod=None, mod_rows=1):
    """Residual add + norm of a block boundary. delta: None, a BF16 tensor, or a modules.Deferred (the producing
    layer's post not yet run). With a consumer group wired to the norm (`norm.consumer`), the next layer's rotation +
    quantization runs in the same kernel and the normed activation is returned as a modules.QAct for that group.
    Returns (x + delta, normed activation). The reference runtime's norms (`torch_ops`) are PyTorch ops."""
    if getattr(norm, 'torch_ops', False):
        return definition.add_norm(x, delta, weight, bias, eps, kind, mod=mod, mod_rows=mod_rows)
    consumer = getattr(norm, 'consumer', None)
    if getattr(norm, 'w8_consumer', False) and not isinstance(delta, modules.Deferred) and mod is None:
        # W8A8 consumers: the norm quantizes its output per token in the same kernel (no rotation)
        shape = x.shape
        x2 = x.reshape(-1, shape[-1])
        q = torch.empty(x2.shape, dtype=torch.int8, device=x.device)
        s = torch.empty(x2.shape[0], dtype=torch.float32, device=x.device)
        kw = {} if delta is None else {'y': delta.reshape(x2.shape)}
        h, _ = K.chain(x2, kind, weight, bias, eps, q=q, scale=s, want_n=False, **kw)
        return h.view(shape), W8Act(q, s, shape)
    if consumer is None and not isinstance(delta, modules.Deferred):
        return K.add_norm(x, delta, weight, bias, eps, kind, mod=mod, mod_rows=mod_rows)
    shape = x.shape
    x2 = x.reshape(-1, shape[-1])
    kw = dict(mod=mod, mod_rows=mod_rows)
    if isinstance(delta, modules.Deferred):
        kw.update(delta.post_args())
    elif delta is not None:
        kw['y'] = delta.reshape(x2.shape)
    if consumer is None:
        h, n = K.chain(x2, kind, weight, bias, eps, **kw)
        return h.view(shape), n.view(shape)
    b = consumer.buffers(x2.shape[0], x2.device)
    h, _ = K.chain(x2, kind, weight, bias, eps, su=consumer.su, q=b.get('q'), q4=b.get('q4'), scale=b['scale'],
                   want_n=False, **kw)
    return h.view(shape), modules.QAct(b, shape)


class RMSNorm(torch.nn.Module):
    """RMSNorm, eps 1e-6; `forward(x, delta)` first adds the pending residual delta (one kernel) and returns
    (x + delta, norm(x + delta)); see _norm for the fused forms."""
    def __init__(self, d):
        super().__init__()
        self.weight = torch.nn.Parameter(torch.ones(d))

    def forward(self, x, delta=None):
        return _norm(self, 'rms', x, delta, self.weight, None, 1e-6)


class LayerNorm(torch.nn.Module):
    """LayerNorm (eps 1e-5 as torch's default, weight / bias when affine); `forward(x, delta, mod)` as RMSNorm's,
    with the optional AdaLN modulation (scale, shift) per sample."""
    def __init__(self, d, elementwise_affine=True, eps=1e-5):
        super().__init__()
        self.eps = eps
        if elementwise_affine:
            self.weight = torch.nn.Parameter(torch.ones(d))
            self.bias = torch.nn.Parameter(torch.zeros(d))
        else:
            self.weight = self.bias = None

    def forward(self, x, delta=None, mod=None, mod_rows=1):
        return _norm(self, 'ln', x, delta, self.weight, self.bias, self.eps, mod, mod_rows)


# Blocks take the residual stream x and the pending residual delta of the previous block (None for the first): the
# add is folded into the block's first norm. They return (x, delta) for the next block.
class VitBlock(torch.nn.Module):
    def __init__(self, c):
        super().__init__()
        d = c.vit_hidden
        self.heads = c.vit_heads
        self.layer_norm1 = LayerNorm(d)
        self.layer_norm2 = LayerNorm(d)
        self.self_attn = torch.nn.Module()
        for n in ('q_proj', 'k_proj', 'v_proj', 'out_proj'):
            setattr(self.self_attn, n, LinearSlot(d, d, bias=True))
        self.mlp = torch.nn.Module()
        self.mlp.fc1 = LinearSlot(d, c.vit_mlp, bias=True)
        self.mlp.fc2 = LinearSlot(c.vit_mlp, d, bias=True)

    def forward(self, x, delta=None):
        x, h = self.layer_norm1(x, delta)
        a = self.self_attn
        qkv = a.qkv(h) if hasattr(a, 'qkv') else (a.q_proj(h), a.k_proj(h), a.v_proj(h))
        o = _attention(*qkv, self.heads)
        x, h = self.layer_norm2(x, a.out_proj(o))
        return x, self.mlp.fc2(self.mlp.fc1(h, act='gelu'))


class LlmBlock(torch.nn.Module):
    def __init__(self, c):
        super().__init__()
        d = c.llm_hidden
        self.heads, self.kv_heads = c.llm_heads, c.llm_kv_heads
        kv = d // c.llm_heads * c.llm_kv_heads
        self.input_layernorm = RMSNorm(d)
        self.post_attention_layernorm = RMSNorm(d)
        self.self_attn = torch.nn.Module()
        self.self_attn.q_proj = LinearSlot(d, d)
        self.self_attn.k_proj = LinearSlot(d, kv)
        self.self_attn.v_proj = LinearSlot(d, kv)
        self.self_attn.o_proj = LinearSlot(d, d)
        self.mlp = torch.nn.Module()
        self.mlp.gate_proj = LinearSlot(d, c.llm_ffn)
        self.mlp.up_proj = LinearSlot(d, c.llm_ffn)
        self.mlp.down_proj = LinearSlot(c.llm_ffn, d)
        self.mlp.forward = lambda x: self.mlp.down_proj(F.silu(self.mlp.gate_proj(x)) * self.mlp.up_proj(x))

    def forward(self, x, delta, rope):
        x, h = self.input_layernorm(x, delta)
        a = self.self_attn
        q, k, v = a.q_proj(h), a.k_proj(h), a.v_proj(h)
        cos, sin = rope
        if getattr(self, 'torch_ops', False):
            q, k = definition.rope(q, cos, sin, self.heads), definition.rope(k, cos, sin, self.kv_heads)
        else:
            q, k = K.rope(q, cos, sin, self.heads, out=q), K.rope(k, cos, sin, self.kv_heads, out=k)
        o = _attention(q, k, v, self.heads, self.kv_heads, causal=True)
        x, h = self.post_attention_layernorm(x, a.o_proj(o))
        return x, self.mlp(h)


class DitBlock(torch.nn.Module):
    def __init__(self, c, cross):
        super().__init__()
        d = c.dit_hidden
        self.heads, self.cross = c.dit_heads, cross
        self.norm1 = LayerNorm(d, elementwise_affine=False, eps=1e-6)
        self.norm3 = LayerNorm(d)
        self.adaln = LinearSlot(d, 2 * d)                      # timestep -> (scale, shift)
        self.attn1 = torch.nn.Module()
        self.attn1.q_proj = LinearSlot(d, d)
        self.attn1.k_proj = LinearSlot(c.llm_hidden if cross else d, d)
        self.attn1.v_proj = LinearSlot(c.llm_hidden if cross else d, d)
        self.attn1.o_proj = LinearSlot(d, d)
        self.ff = torch.nn.Module()
        self.ff.fc1 = LinearSlot(d, c.dit_ffn)
        self.ff.fc2 = LinearSlot(c.dit_ffn, d)
        self.ff.forward = lambda x: self.ff.fc2(F.gelu(self.ff.fc1(x), approximate='tanh'))

    def kv(self, feats):
        """Cross-attention keys / values of the backbone features: computed once per action chunk."""
        return self.attn1.k_proj(feats), self.attn1.v_proj(feats)

    def forward(self, x, delta, silu_temb, kv=None):
        d = x.shape[-1]
        mod = self.adaln(silu_temb)                           # (B, 1, 2d): AdaLN scale, shift
        x, h = self.norm1(x, delta, mod=(mod[:, 0, :d], mod[:, 0, d:]), mod_rows=x.shape[1])
        a = self.attn1
        if self.cross:
            k, v = kv
            o = _attention(a.q_proj(h), k, v, self.heads)
        else:
            o = _attention(a.q_proj(h), a.k_proj(h), a.v_proj(h), self.heads)
        x, h = self.norm3(x, a.o_proj(o))
        return x, self.ff(h)


class GrootStylePolicy(torch.nn.Module):
    def __init__(self, c=PolicyConfig()):
        super().__init__()
        self.c = c
        dv, dl, dd = c.vit_hidden, c.llm_hidden, c.dit_hidden
        self.patch_embed = torch.nn.Linear(3 * c.patch * c.patch, dv)
        self.pos_embed = torch.nn.Parameter(torch.zeros(c.patches, dv))
        self.vit = torch.nn.ModuleList([VitBlock(c) for _ in range(c.vit_layers)])
        self.vit_norm = LayerNorm(dv)
        self.proj_norm = LayerNorm(dv * c.shuffle ** 2)
        self.proj1 = torch.nn.Linear(dv * c.shuffle ** 2, dl)
        self.proj2 = torch.nn.Linear(dl, dl)
        self.embed_tokens = torch.nn.Embedding(c.vocab, dl)
        self.llm = torch.nn.ModuleList([LlmBlock(c) for _ in range(c.llm_layers)])
        self.llm_norm = RMSNorm(dl)
        self.state_enc1 = torch.nn.Linear(c.state_dim, dd)
        self.state_enc2 = torch.nn.Linear(dd, dd)
        self.action_enc = torch.nn.Linear(c.action_dim, dd)
        self.time1 = torch.nn.Linear(256, dd)
        self.time2 = torch.nn.Linear(dd, dd)
        self.dit = torch.nn.ModuleList([DitBlock(c, cross=(i % 2 == 0)) for i in range(c.dit_layers)])
        self.out_norm = LayerNorm(dd)
        self.proj_out = torch.nn.Linear(dd, c.action_dim)

    # ---------------------------------------------------------------------------------------------------- stages
    def embed(self, images, lang_ids):
        """images (B, cams, H, W, 3) uint8, lang_ids (B, L) -> prefix embeddings (B, T, 2048) BF16."""
        c = self.c
        B = images.shape[0]
        x = images.to(torch.bfloat16) / 127.5 - 1.0
        g = c.image // c.patch
        x = x.view(B * c.cameras, g, c.patch, g, c.patch, 3).permute(0, 1, 3, 2, 4, 5).reshape(B * c.cameras, g * g, -1)
        h = self.patch_embed(x) + self.pos_embed.to(torch.bfloat16)
        d = None
        for blk in self.vit:
            h, d = blk(h, d)
        _, h = self.vit_norm(h, d)
        s = c.shuffle
        h = h.view(B * c.cameras, g // s, s, g // s, s, -1).permute(0, 1, 3, 2, 4, 5).reshape(B * c.cameras, (g // s) ** 2, -1)
        img = self.proj2(F.gelu(self.proj1(self.proj_norm(h)[1]), approximate='tanh'))
        img = img.view(B, c.cameras * c.image_tokens, -1)
        return torch.cat((img, self.embed_tokens(lang_ids)), 1)

    def backbone(self, prefix):
        c = self.c
        rope = rope_tables(prefix.shape[1], c.llm_hidden // c.llm_heads, prefix.device)
        x, d = prefix, None
        for blk in self.llm:
            x, d = blk(x, d, rope)
        return self.llm_norm(x, d)[1]

    def timestep(self, t, B, device):
        half = 128
        freqs = torch.exp(-math.log(10000.0) * torch.arange(half, device=device, dtype=torch.float32) / half)
        ang = (t * 1000.0) * freqs
        emb = torch.cat((ang.sin(), ang.cos()))[None, None, :].expand(B, 1, 256).to(torch.bfloat16)
        return self.time2(F.silu(self.time1(emb)))

    def action_head(self, feats, state, noise):
        """feats (B, T, 2048), state (B, 64), noise (B, chunk, action_dim) -> actions (B, chunk, action_dim)."""
        c = self.c
        B = feats.shape[0]
        kvs = [blk.kv(feats) if blk.cross else None for blk in self.dit]
        st = self.state_enc2(F.silu(self.state_enc1(state.to(torch.bfloat16))))[:, None, :]
        a = noise.float()
        dt = 1.0 / c.flow_steps
        ts = torch.arange(c.flow_steps, device=feats.device, dtype=torch.float32) * dt   # on device: graph-capturable
        for k in range(c.flow_steps):
            temb = self.timestep(ts[k], B, feats.device)
            x = torch.cat((st, self.action_enc(a.to(torch.bfloat16)) + temb), 1)
            silu_temb, d = F.silu(temb), None
            for blk, kv in zip(self.dit, kvs):
                x, d = blk(x, d, silu_temb, kv)
            v = self.proj_out(self.out_norm(x, d)[1][:, 1:])
            a = a + dt * v.float()
        return a

    def forward(self, images, lang_ids, state, noise):
        return self.action_head(self.backbone(self.embed(images, lang_ids)), state, noise)


# ---------------------------------------------------------------------------------------------------- weights
def _fp_init(model, seed):
    """Seeded random FP weights (every parameter drawn from one generator, so equal seeds give equal models)."""
    g = torch.Generator(device='cpu').manual_seed(seed)
    with torch.no_grad():
        model.pos_embed.copy_(torch.randn(model.pos_embed.shape, generator=g) * 0.02)
    for m in model.modules():
        if isinstance(m, torch.nn.Linear):
            with torch.no_grad():
                m.weight.copy_(torch.randn(m.weight.shape, generator=g) / math.sqrt(m.in_features))
                if m.bias is not None:
                    m.bias.zero_()
        elif isinstance(m, torch.nn.Embedding):
            with torch.no_grad():
                m.weight.copy_(torch.randn(m.weight.shape, generator=g))


def quantized_slots(model):
    return {name: m for name, m in model.named_modules() if isinstance(m, LinearSlot)}


def synthetic_layers(model, device, seed=0):
    """Random trellis-coded layers for every LLM / DiT slot: uniform 2-bit streams (valid codes of the tail-biting
    trellis), N(0, 0.968^2) FP16 tables, FP16 row scales sized so a layer keeps the activation scale, and one sign
    vector per input tensor (layers that read the same tensor share their input signs, as in the reference)."""
    g = torch.Generator(device=device).manual_seed(seed)
    layers, su_cache = {}, {}
    for name, m in quantized_slots(model).items():
        if name.startswith('vit.'):
            continue
        n, mm = m.in_features, m.out_features
        parent = name.rsplit('.', 1)[0]
        cross_kv = name.endswith(('k_proj', 'v_proj')) and getattr(model.get_submodule(parent.rsplit('.', 1)[0]), 'cross', False)
        key = (parent + (':kv' if cross_kv else ''), n)        # cross-attention k / v read the backbone features
        if key not in su_cache:
            su_cache[key] = (torch.randint(0, 2, (n,), device=device, generator=g) * 2 - 1).to(torch.int8)
        bits = torch.randint(-32768, 32768, ((mm // 16) * (n // 16), 32), dtype=torch.int32, device=device, generator=g).to(torch.int16)
        tens = dict(bits=bits, tlut=(torch.randn(512, 2, device=device, generator=g) * 0.968).half(),
                    row_scale=torch.full((mm,), 1.0 / math.sqrt(n), device=device).half(), su=su_cache[key],
                    sv=(torch.randint(0, 2, (mm,), device=device, generator=g) * 2 - 1).to(torch.int8))
        bias = torch.zeros(mm, device=device) if m.has_bias else None
        layers[name] = Layer(name, tens, bias=bias, device=device)
    return layers


def synthetic_w8a8(model, device, seed=1, reference=False):
    g = torch.Generator(device=device).manual_seed(seed)
    for name, m in quantized_slots(model).items():
        if not name.startswith('vit.'):
            continue
        W = torch.randint(-127, 128, (m.out_features, m.in_features), dtype=torch.int8, device=device, generator=g)
        s_ch = torch.full((m.out_features,), 1.0 / (73.3 * math.sqrt(m.in_features)), device=device)
        bias = (torch.randn(m.out_features, device=device, generator=g) * 0.02).bfloat16() if m.has_bias else None
        modules.set_submodule(model, name, W8A8Linear(W, s_ch, bias, reference=reference))


def build_policy(device='cuda', runtime='fly', c=PolicyConfig(), seed=0, layers=None, ref_w8=None):
    """The quantized policy on `device`. runtime: 'fly' (2-bit stream decoded inside the products), 'resident' (INT8
    decoded once), 'hybrid' (DiT decoded once per chunk via modules.decode_chunk) or 'reference' (the definition in
    PyTorch ops, with norms and rotary embedding in PyTorch ops; ref_w8 optionally gives its decoded weights).
    Returns (policy, trellis layers, install info)."""
    model = GrootStylePolicy(c)
    _fp_init(model, seed)
    model = model.to(device=device, dtype=torch.bfloat16)
    layers = synthetic_layers(model, device, seed) if layers is None else layers
    synthetic_w8a8(model, device, seed + 1, reference=(runtime == 'reference'))
    mlp_acts = {}
    for i in range(c.llm_layers):
        mlp_acts[f'llm.{i}.mlp'] = 'silu'
    for i in range(c.dit_layers):
        mlp_acts[f'dit.{i}.ff'] = 'gelu'
    info = modules.install(model, layers, runtime=runtime, chunk_parts=('dit.',), mlp_acts=mlp_acts, ref_w8=ref_w8)
    info['chains'] = wire_chains(model) if runtime != 'reference' and modules.FUSE['chain'] else 0
    if runtime == 'reference':
        for m in model.modules():
            if isinstance(m, (RMSNorm, LayerNorm, LlmBlock)):
                m.torch_ops = True
    model.eval()
    return model, layers, info


def wire_chains(model):
    """Fuse every 2-bit block boundary of the LLM and the DiT into one kernel (kernels.chain): the layer before the
    residual add (o_proj, the MLP's down / fc2) hands its accumulator over unposted, and the norm after it quantizes
    straight into the next group's buffers (q / k / v, or the MLP's first group). Returns the number of norms wired."""
    wired = 0

    def consume(norm, target):
        nonlocal wired
        group = target.shared if isinstance(target, modules.KLinear) else \
            target.groups[0] if isinstance(target, (modules.KGatedMLP, modules.KPlainMLP)) else None
        if group is not None:
            norm.consumer = group
            wired += 1

    def defer(producer):
        if isinstance(producer, modules.KLinear) and len(producer.shared.layers) == 1:
            producer.shared.defer = True
        elif isinstance(producer, (modules.KGatedMLP, modules.KPlainMLP)):
            producer.defer = True

    for blk in model.llm:
        consume(blk.input_layernorm, blk.self_attn.q_proj)
        consume(blk.post_attention_layernorm, blk.mlp)
        defer(blk.self_attn.o_proj)
        defer(blk.mlp)
    for blk in model.dit:
        consume(blk.norm1, blk.attn1.q_proj)
        consume(blk.norm3, blk.ff)
        defer(blk.attn1.o_proj)
        defer(blk.ff)
    for blk in model.vit:
        # W8A8 vision blocks: both norms quantize for their consumers, and q / k / v run as one GEMM (their weights
        # become views of the group's concatenation)
        a = blk.self_attn
        if all(isinstance(m, W8A8Linear) for m in (a.q_proj, a.k_proj, a.v_proj, blk.mlp.fc1)):
            a.qkv = W8A8Group([a.q_proj, a.k_proj, a.v_proj])
            off = 0
            for m in (a.q_proj, a.k_proj, a.v_proj):
                m.W, m.s_ch = a.qkv.W[off:off + m.out_features], a.qkv.s_ch[off:off + m.out_features]
                if m.bias is not None:
                    m.bias = a.qkv.bias[off:off + m.out_features]
                off += m.out_features
            blk.layer_norm1.w8_consumer = blk.layer_norm2.w8_consumer = True
            wired += 2
    return wired


def synthetic_observations(B, c=PolicyConfig(), device='cuda', seed=0):
    g = torch.Generator(device=device).manual_seed(seed)
    images = torch.randint(0, 256, (B, c.cameras, c.image, c.image, 3), dtype=torch.uint8, device=device, generator=g)
    lang = torch.randint(0, c.vocab, (B, c.lang_tokens), device=device, generator=g)
    state = torch.randn(B, c.state_dim, device=device, generator=g)
    noise = torch.randn(B, c.chunk, c.action_dim, device=device, generator=g)
    return images, lang, state, noise
