"""The W2A8 / W8A8 definition in plain PyTorch ops: the arithmetic the kernels are held to, as its own runtime.

This module is the 'reference' runtime of `modules.install` and `policy.build_policy`. It uses no entry point of the
sm_100a library, so a comparison against it checks the kernels against an independent statement of the definition
(the reference's `tcq_format.py`, ForeverBlue816/yanlongvla, deploy/tcq_kernels/tcq_format.py:36-148):

  walsh            block Walsh over the binary decomposition of the width, FP32, radix-2 stages h = 1, 2, 4, ... with
                   (a + b, a - b) pairs, then an FP32 multiply by FP32(1/sqrt(w)) per block        (tcq_format.py:44-55)
  trellis_states   state t of a 16 x 16 tile = bits [4t, 4t + 16) of its 512-bit stream, MSB first, tail-biting
                                                                                                    (tcq_format.py:58-63)
  decode_w8        hash lookup h = ((s + 1) s >> 6) & 511 into the INT8 table, first coordinate negated when bit 15
                   of (s + 1) s is set                                                              (tcq_format.py:66-71)
  quantize_tokens  per-token absmax, true FP32 division, round half to even, clamp +-127           (tcq_format.py:119-122)
  int_matmul       exact INT8 product: cuBLASLt (torch._int_mm, token rows padded to 32) on CUDA, float64 on the CPU
                                                                                                    (tcq_format.py:110-116)
  linear           the whole layer, y = BF16(walsh(((acc * s) * rs)) * sv + bias)                  (tcq_format.py:125-148)

and, for the policy's own glue between quantized layers, the residual add + RMSNorm / LayerNorm (+ AdaLN) and the
half-split rotary embedding in PyTorch ops. A norm's row sums are taken in one fixed order (`row_sum`), the one the
norm kernels use, so that the whole policy can be compared bit for bit.
"""
import math

import torch

_BLOCK_SCALE = {}


def block_widths(width):
    """Descending power-of-two blocks whose sum is `width` (tcq_format.py:26-30)."""
    return [1 << b for b in range(width.bit_length() - 1, -1, -1) if width >> b & 1]


def _block_scale(w, device):
    """FP32(1 / sqrt(w)) as a device scalar, made once per (w, device) so that graph captures copy nothing."""
    key = (w, str(device))
    t = _BLOCK_SCALE.get(key)
    if t is None:
        t = _BLOCK_SCALE[key] = torch.tensor(1.0 / math.sqrt(w), dtype=torch.float32, device=device)
    return t


def walsh(x):
    """Block Walsh of x (..., D) FP32 along its last dim (tcq_format.py:44-55). Stage h adds and subtracts the element
    pairs (i, i + h) inside every run of 2h elements, for h = 1, 2, 4, ..., w / 2 in each power-of-two block."""
    lead, D = x.shape[:-1], x.shape[-1]
    pieces, start = [], 0
    for w in block_widths(D):
        blk = x[..., start:start + w].reshape(-1, w)
        rows = blk.shape[0]
        h = 1
        while h < w:
            pair = blk.view(rows, w // (2 * h), 2, h)
            lo, hi = pair.select(2, 0), pair.select(2, 1)
            blk = torch.stack((lo + hi, lo - hi), dim=2).view(rows, w)
            h <<= 1
        pieces.append((blk * _block_scale(w, x.device)).view(*lead, w))
        start += w
    return pieces[0] if len(pieces) == 1 else torch.cat(pieces, dim=-1)


def trellis_states(bits, m, n):
    """(m/16 * n/16, 32) stream words -> (m, n/2) int64 states in weight order (tcq_format.py:58-63). Within a tile,
    state t = 8 * row + pair is the 16-bit window starting at bit 4t of the 512-bit stream (word t // 4, offset
    4 (t % 4)); the window of the last states wraps to word 0 (tail-biting)."""
    words = bits.to(torch.int64) & 0xFFFF                      # int16 view -> the uint16 words
    t = torch.arange(128, device=bits.device)
    first, second = words[:, t >> 2], words[:, ((t >> 2) + 1) & 31]
    window = (first << 16) | second                              # 32 bits starting at the window's word
    st = (window >> (16 - 4 * (t & 3))) & 0xFFFF
    return st.view(m // 16, n // 16, 16, 8).permute(0, 2, 1, 3).reshape(m, n // 2)


def decode_w8(bits, t8, m, n):
    """Dense INT8 weights (m, n) in the rotated basis from the trellis stream and the INT8 table (512, 2)
    (tcq_format.py:66-71, 97-98)."""
    s = trellis_states(bits, m, n)
    x = s * (s + 1)
    pair = t8.to(torch.int16)[(x >> 6) & 511]                   # (m, n/2, 2)
    first = torch.where((x >> 15) & 1 == 1, -pair[..., 0], pair[..., 0])
    return torch.stack((first, pair[..., 1]), dim=-1).reshape(m, n).to(torch.int8)


def quantize_tokens(h):
    """Per-token INT8 quantizer of h (M, K) FP32 (tcq_format.py:119-122): s = amax / 127 by a true FP32 division (a
    tensor divisor; 1 for an all-zero row), q = clamp(round-half-even(h / s), -127, 127). Returns q int8, s (M, 1)."""
    amax = h.abs().amax(dim=1, keepdim=True)
    s = torch.where(amax > 0, amax / torch.full_like(amax, 127.0), torch.ones_like(amax))
    return torch.clamp(torch.round(h / s), -127, 127).to(torch.int8), s


def int_matmul(q, w8):
    """Exact (M, K) int8 x (N, K) int8 -> (M, N) int32 (tcq_format.py:110-116): cuBLASLt through torch._int_mm on CUDA
    (which wants more than 16 rows: the token rows are zero-padded to 32), float64 dot products on the CPU."""
    if q.is_cuda:
        M = q.shape[0]
        if M < 32:
            q = torch.cat((q, q.new_zeros(32 - M, q.shape[1])), dim=0)
        return torch._int_mm(q, w8.t())[:M]
    return (q.double() @ w8.double().t()).to(torch.int32)


def linear(x, layer, w8, a8=True):
    """The W2A8 layer by definition (tcq_format.py:125-148): x (..., n) -> y (..., m) BF16. `layer` provides su, sv
    (int8 signs), rs (FP32 row scales) and bias (FP32 or None); w8 (m, n) int8 are its decoded weights. a8=False: the
    FP32 activations in the rotated space times the same weights, in float64 (tcq_format.py:137-138)."""
    shape = x.shape
    h = walsh(x.reshape(-1, shape[-1]).float() * layer.su.float())
    if a8:
        q, s = quantize_tokens(h)
        z = (int_matmul(q, w8).float() * s) * layer.rs[None, :]
    else:
        z = (h.double() @ w8.double().t()).float() * layer.rs[None, :]
    y = walsh(z) * layer.sv.float()
    if layer.bias is not None:
        y = y + layer.bias
    return y.to(torch.bfloat16).reshape(*shape[:-1], layer.m)


def w8a8_linear(x, W, s_ch, bias=None):
    """W8A8 layer (benchmark config 3, the vision tower): per-token INT8 activations without rotation, exact product,
    y = BF16(((float)acc * s_tok) * s_ch) + bias (a BF16 add)."""
    shape = x.shape
    q, s = quantize_tokens(x.reshape(-1, shape[-1]).float())
    y = ((int_matmul(q, W).float() * s) * s_ch[None, :]).to(torch.bfloat16)
    if bias is not None:
        y = y + bias
    return y.reshape(*shape[:-1], W.shape[0])


def _norm_threads(D):
    """Threads of one row in the kernels' canonical order: one 16-element chunk each, a multiple of 32, 32..512."""
    return min(max(-(-(D // 16) // 32) * 32, 32), 512)


def row_sum(v):
    """Sum of each row of v (M, D) FP32 in one fixed order (the order the norm kernels use, so that a norm computed
    here and one computed there agree bit for bit): the row is cut into 16-element chunks; chunk c belongs to thread
    c mod T (T = _norm_threads(D); D > 8192 wraps four chunks onto each thread), and each thread keeps one running sum
    over its chunks' elements in index order, starting from 0; the threads' sums are combined within each group of 32
    by halving (element i of the first half plus element i of the second half, five times); the 32-groups' results
    are added in group order, starting from 0."""
    M, D = v.shape
    T = _norm_threads(D)
    NC = 1 if D <= 8192 else 4
    chunks = torch.zeros(M, NC * T, 16, dtype=torch.float32, device=v.device)
    chunks[:, :D // 16] = v.reshape(M, D // 16, 16)
    per_thread = chunks.view(M, NC, T, 16).transpose(1, 2).reshape(M, T, NC * 16)
    part = torch.zeros(M, T, dtype=torch.float32, device=v.device)
    for i in range(NC * 16):
        part = part + per_thread[:, :, i]
    g = part.view(M, T // 32, 32)
    while g.shape[-1] > 1:
        half = g.shape[-1] // 2
        g = g[..., :half] + g[..., half:]
    total = torch.zeros(M, dtype=torch.float32, device=v.device)
    for w in range(T // 32):
        total = total + g[:, w, 0]
    return total[:, None]


def add_norm(x, delta, weight, bias, eps, kind, mod=None, mod_rows=1):
    """Residual add + norm in PyTorch ops: h = BF16(x + delta) (x when delta is None), n = BF16(norm(h)) with
    RMSNorm n = (h * r) * w, r = rsqrt(sum(h^2) / D + eps), or LayerNorm n = ((h - mu) * r) * w + b, mu = sum(h) / D,
    r = rsqrt(sum((h - mu)^2) / D + eps) (FP32; true divisions; the sums in `row_sum`'s fixed order), then the AdaLN
    modulation n * (1 + scale) + shift when mod = (scale, shift) (one (D,) row per mod_rows rows). Returns (h, n)."""
    h = x if delta is None else x + delta
    D = h.shape[-1]
    hf = h.reshape(-1, D).float()
    div = torch.full((hf.shape[0], 1), float(D), dtype=torch.float32, device=hf.device)
    if kind == 'rms':
        r = torch.rsqrt(row_sum(hf * hf) / div + eps)
        n = hf * r
    else:
        mu = row_sum(hf) / div
        c = hf - mu
        r = torch.rsqrt(row_sum(c * c) / div + eps)
        n = c * r
    if weight is not None:
        n = n * weight.float()
    if bias is not None:
        n = n + bias.float()
    if mod is not None:
        scale, shift = mod
        scale = scale.reshape(-1, D).float().repeat_interleave(mod_rows, dim=0)
        shift = shift.reshape(-1, D).float().repeat_interleave(mod_rows, dim=0)
        n = n * (1.0 + scale) + shift
    return h, n.to(torch.bfloat16).view(h.shape)


def rope(x, cos, sin, heads):
    """Half-split rotary embedding of x (B, T, heads * D) BF16 with cos / sin (T, D/2) FP32: for each head,
    (a, b) -> (a cos - b sin, a sin + b cos), rounded to BF16."""
    B, T, W = x.shape
    D = W // heads
    v = x.float().view(B, T, heads, 2, D // 2)
    a, b = v[..., 0, :], v[..., 1, :]
    c, s = cos[None, :, None, :], sin[None, :, None, :]
    out = torch.stack((a * c - b * s, a * s + b * c), dim=3)
    return out.reshape(B, T, W).to(torch.bfloat16)
