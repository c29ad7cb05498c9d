"""CPU oracle for the W2A8 trellis-coded Linear: a numpy restatement of the reference arithmetic.

TEST INFRASTRUCTURE ONLY. Nothing in the product package imports this module; only `tests/`,
`__graft_entry__.smoke()` and `bench.py`'s CPU-baseline leg (`--impl reference` and the `cpu_baseline` field)
may call it, and only as the checker / the timed CPU reference, never as the thing measured on the GPU.

Every function restates one function of the reference checkout (ForeverBlue816/yanlongvla), cited as
`deploy/tcq_kernels/<file>:<line>`. The arithmetic is fixed so that results are bit-identical to the reference's
PyTorch definition on CPU:
  * FP32 butterflies in the order h = 1, 2, 4, ... with (a + b, a - b) pairs, then an FP32 multiply by
    float32(1 / sqrt(w)) per power-of-two block (tcq_format.py:36-55);
  * the per-token quantizer divides with a true FP32 division and rounds half to even (tcq_format.py:119-122);
  * integer products are exact (float64 dot products of int8 values, tcq_format.py:110-116);
  * the epilogue is ((float)acc * s) * rs in FP32 (tcq_format.py:135);
  * FP32 -> BF16 is round-to-nearest-even with NaN -> 0x7fc0, as c10::BFloat16 (kernels.py:20-25).

Parity pin: `tests/golden/make_golden.py` runs the reference's own `tcq_format.py` on seeded inputs and stores its
outputs under `tests/golden/`; `tests/test_oracle_golden.py` checks this module against them bit for bit.

BF16 and FP16 values travel as numpy uint16 bit patterns (BF16) or numpy float16 (FP16).
"""
import math

import numpy as np

# ----------------------------------------------------------------------------------------------------------- numerics
def bf16_to_f32(b):
    """BF16 bit patterns (uint16) -> float32 (exact)."""
    b = np.asarray(b, dtype=np.uint16)
    return (b.astype(np.uint32) << np.uint32(16)).view(np.float32)


def f32_to_bf16(x):
    """float32 -> BF16 bit patterns, round to nearest even, NaN -> 0x7fc0 (kernels.py:20-25, c10::BFloat16)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    nan = (u & 0x7fffffff) > 0x7f800000
    r = ((u + 0x7fff + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = 0x7fc0
    return r


def to_f32(x, dtype):
    """Input activations -> float32 (`x.float()` in tcq_format.py:130): dtype 'bf16' (uint16 bits), 'f16' or 'f32'."""
    if dtype == 'bf16':
        return bf16_to_f32(x)
    return np.asarray(x).astype(np.float32)


# ----------------------------------------------------------------------------------------------------------- rotation
def block_widths(width):
    """Binary decomposition of a width into descending power-of-two blocks (tcq_format.py:26-30)."""
    out = []
    while width:
        b = 1 << (width.bit_length() - 1)
        out.append(b)
        width -= b
    return out


def block_scale(w):
    """FP32 constant 1 / sqrt(w) of one block (tcq_format.py:36-41; kernels.py:144)."""
    return np.float32(1.0 / math.sqrt(w))


def fwht(x):
    """Block Walsh on the last dim in FP32, stages h = 1, 2, 4, ..., scaled per block (tcq_format.py:44-55)."""
    x = np.asarray(x, dtype=np.float32)
    lead = x.shape[:-1]
    outs, off = [], 0
    for w in block_widths(x.shape[-1]):
        y, h = x[..., off:off + w], 1
        while h < w:
            y = y.reshape(*lead, w // (2 * h), 2, h)
            a, b = y[..., 0, :], y[..., 1, :]
            y = np.stack((a + b, a - b), axis=-2).reshape(*lead, w)
            h *= 2
        outs.append(y * block_scale(w))
        off += w
    return np.concatenate(outs, -1) if len(outs) > 1 else outs[0].copy()


def rotate(x, signs, dtype='f32', inverse=False):
    """Randomized Walsh rotation of rows: forward y = fwht(x * s); inverse x = fwht(y) * s (tcq_format.py:130,145)."""
    s = np.asarray(signs).astype(np.float32)
    xf = to_f32(x, dtype)
    return fwht(xf) * s if inverse else fwht(xf * s)


# ----------------------------------------------------------------------------------------------------------- trellis
def states_from_bits(bits, m, n):
    """Windowed read: state t of a tile = bits [4t, 4t+16) of its 512-bit stream, MSB first, tail-biting
    (tcq_format.py:58-63). bits: (m/16 * n/16, 32) int16/uint16 words -> (m, n/2) int64."""
    b = np.asarray(bits).astype(np.int64) & 0xffff
    t = np.arange(128)
    w, r = t // 4, t % 4
    st = (((b[:, w] << 16) | b[:, (w + 1) % 32]) >> (16 - 4 * r)) & 0xffff
    return st.reshape(m // 16, n // 16, 16, 8).transpose(0, 2, 1, 3).reshape(m, n // 2)


def lookup(states, table):
    """Hash decode: x = (s + 1) s; value pair = table[(x >> 6) & 511]; first coordinate negated when bit 15 of x is
    set (tcq_format.py:66-71; groot_tcq.py:143-151)."""
    x = (states + 1) * states
    v = np.asarray(table)[(x >> 6) & 511]
    v0 = np.where(((x >> 15) & 1).astype(bool), -v[..., 0], v[..., 0])
    return np.stack((v0, v[..., 1]), -1).reshape(states.shape[0], -1)


def snap(tlut_f16, row_scale_f16):
    """INT8 table at load: g = 127 / max|tlut| (FP32), t8 = clamp(round(tlut * g)), rs = row_scale / g (tcq_format.py:74-77).
    `127.0 / tensor` in PyTorch is `tensor.reciprocal() * 127.0`, so g = fl(fl(1 / max) * 127), not a true division."""
    t = np.asarray(tlut_f16, dtype=np.float16).astype(np.float32)
    g = np.float32(np.float32(np.float32(1.0) / np.abs(t).max()) * np.float32(127.0))
    t8 = np.clip(np.rint(t * g), -127, 127).astype(np.int8)
    rs = np.asarray(row_scale_f16, dtype=np.float16).astype(np.float32) / g
    return t8, rs.astype(np.float32), g


class Layer:
    """One quantized Linear: packed tensors + derived INT8 table / row scales (tcq_format.py:80-107)."""
    def __init__(self, bits, tlut, row_scale, su, sv, bias=None):
        self.bits = np.asarray(bits).view(np.uint16) if np.asarray(bits).dtype == np.int16 else np.asarray(bits, dtype=np.uint16)
        self.tlut = np.asarray(tlut, dtype=np.float16)
        self.row_scale = np.asarray(row_scale, dtype=np.float16)
        self.su = np.asarray(su, dtype=np.int8)
        self.sv = np.asarray(sv, dtype=np.int8)
        self.m, self.n = self.sv.size, self.su.size
        assert self.bits.shape == ((self.m // 16) * (self.n // 16), 32) and self.m % 16 == 0 and self.n % 16 == 0
        self.t8, self.rs, self.gain = snap(self.tlut, self.row_scale)
        self.bias = None if bias is None else np.asarray(bias, dtype=np.float32)

    def states(self):
        return states_from_bits(self.bits, self.m, self.n)

    def w8_reference(self):
        """Decoded INT8 weight in the rotated basis (tcq_format.py:97-98)."""
        return lookup(self.states(), self.t8.astype(np.int16)).astype(np.int8)

    def dense(self, table='fp16'):
        """Original-basis FP32 weight S_v H_m diag(r) Q H_n S_u (tcq_format.py:100-107)."""
        if table == 'fp16':
            q = lookup(self.states(), self.tlut.astype(np.float32)) * self.row_scale.astype(np.float32)[:, None]
        else:
            q = self.w8_reference().astype(np.float32) * self.rs[:, None]
        w = fwht(q) * self.su.astype(np.float32)[None, :]
        return (fwht(np.ascontiguousarray(w.T)) * self.sv.astype(np.float32)[None, :]).T


def decode_bf16_table(t8):
    """BF16 bit patterns of the INT8 table values (modules.py:51)."""
    return f32_to_bf16(np.asarray(t8).astype(np.float32))


def decode_bf16(layer):
    """Dense BF16 decode of the INT8 table values (kernels.py:320-337): sign applied as a BF16 sign-bit flip."""
    st = layer.states()
    x = (st + 1) * st
    tb = decode_bf16_table(layer.t8).reshape(512, 2)
    v = tb[(x >> 6) & 511]
    v0 = v[..., 0] ^ (((x >> 15) & 1).astype(np.uint16) << 15)
    return np.stack((v0, v[..., 1]), -1).reshape(layer.m, layer.n)


# ----------------------------------------------------------------------------------------------------------- activations
def quantize_tokens(h):
    """Per-token absmax INT8 quantizer: s = amax / 127 (true FP32 division; 1 when amax = 0),
    q = clamp(round_half_even(h / s), -127, 127) (tcq_format.py:119-122)."""
    h = np.asarray(h, dtype=np.float32)
    amax = np.abs(h).max(axis=1, keepdims=True)
    s = np.where(amax > 0, amax / np.float32(127.0), np.float32(1.0)).astype(np.float32)
    return np.clip(np.rint(h / s), -127, 127).astype(np.int8), s


def q4_words(q):
    """(M, K) int8 -> (K/4, M) int32 words: 4 consecutive inputs per little-endian word, token = column (kernels.py:170-183)."""
    q = np.ascontiguousarray(q, dtype=np.int8)
    M, K = q.shape
    return np.ascontiguousarray(q.view(np.int32).reshape(M, K // 4).T)


def int_matmul(q, w8):
    """Exact (M, K) int8 x (N, K) int8 -> (M, N) int32 (tcq_format.py:110-116, CPU branch)."""
    return (np.asarray(q).astype(np.float64) @ np.asarray(w8).astype(np.float64).T).astype(np.int32)


def scale_acc(acc, s, rs):
    """Epilogue ((float)acc * s_token) * rs_row in FP32 (tcq_format.py:135; kernels.py:545)."""
    return (np.asarray(acc).astype(np.float32) * np.asarray(s, dtype=np.float32).reshape(-1, 1)) * np.asarray(rs, dtype=np.float32)[None, :]


def pre(x, dtype, su):
    """k_pre: sign flip, block Walsh, per-token INT8 (kernels.py:208-219) -> q (M, K) int8, scale (M,) float32."""
    h = fwht(to_f32(x, dtype) * np.asarray(su).astype(np.float32))
    q, s = quantize_tokens(h)
    return q, s[:, 0]


def pre_h(x, dtype, su):
    """k_preh: rotated activations rounded to BF16 (kernels.py:309-317) -> (M, K) BF16 bits."""
    return f32_to_bf16(fwht(to_f32(x, dtype) * np.asarray(su).astype(np.float32)))


def post(z, sv, bias=None):
    """k_post on already-scaled FP32 z: block Walsh, sign, bias, BF16 (kernels.py:221-230; tcq_format.py:145-148)."""
    y = fwht(np.asarray(z, dtype=np.float32)) * np.asarray(sv).astype(np.float32)
    if bias is not None:
        y = y + np.asarray(bias, dtype=np.float32)
    return f32_to_bf16(y)


def post_acc(acc, acc_dtype, s, rs, sv, bias=None):
    """k_post_{i32,f32,bf16}: SCALE(acc) = ((float)a * s) * rs | a | bf2f(a) * rs, then post (kernels.py:545)."""
    if acc_dtype == 'i32':
        z = scale_acc(acc, s, rs)
    elif acc_dtype == 'f32':
        z = np.asarray(acc, dtype=np.float32)
    else:
        z = bf16_to_f32(acc) * np.asarray(rs, dtype=np.float32)[None, :]
    return post(z, sv, bias)


def reference_linear(x, dtype, layer, a8=True, table='int8', w8=None):
    """The W2A8 definition of one layer (tcq_format.py:125-148) -> (M, m) BF16 bits."""
    h = fwht(to_f32(x, dtype).reshape(-1, layer.n) * layer.su.astype(np.float32))
    if table == 'int8':
        w8 = layer.w8_reference() if w8 is None else w8
        if a8:
            q, s = quantize_tokens(h)
            z = scale_acc(int_matmul(q, w8), s, layer.rs)
        else:
            z = (h.astype(np.float64) @ w8.astype(np.float64).T).astype(np.float32) * layer.rs[None, :]
    else:
        wq = lookup(layer.states(), layer.tlut.astype(np.float32))
        if a8:
            q, s = quantize_tokens(h)
            z = scale_acc((q.astype(np.float64) @ wq.astype(np.float64).T).astype(np.float32), s, layer.row_scale.astype(np.float32))
        else:
            z = (h.astype(np.float64) @ wq.astype(np.float64).T).astype(np.float32) * layer.row_scale.astype(np.float32)[None, :]
    return post(z, layer.sv, layer.bias)


def gemm_z(q, w8, s, rs):
    """k_gemm_w8 / k_gemm_tcq output: z (M, N) FP32 = ((float)acc * s) * rs (kernels.py:355-363)."""
    return scale_acc(int_matmul(q, w8), s, rs)


def gemmf_z(h_bf16, w8, rs):
    """k_gemmf_*: BF16 rotated activations x INT8 weights, FP32 accumulation, z = acc * rs (kernels.py:430-489).
    The kernels sum in FP32 in their own order, so this float64 sum is a tolerance check, not a bit-exact one."""
    h = bf16_to_f32(h_bf16).astype(np.float64)
    return ((h @ np.asarray(w8).astype(np.float64).T) * np.asarray(rs, dtype=np.float64)[None, :]).astype(np.float32)


def int8_gemm_scaled(q, w8, s_tok, s_ch, out='bf16'):
    """W8A8 GEMM with the scale epilogue: BF16(((float)acc * s_tok) * s_ch) (config 3 of the path)."""
    z = scale_acc(int_matmul(q, w8), s_tok, s_ch)
    return f32_to_bf16(z) if out == 'bf16' else z


# ----------------------------------------------------------------------------------------------------------- MLP middles
def act_lut(lut, b):
    """BF16 activation by table: lut (65536,) BF16 bits indexed by the BF16 bit pattern (kernels.py:39-45, 563-569)."""
    return np.asarray(lut, dtype=np.uint16)[np.asarray(b, dtype=np.uint16)]


def bf16_mul(a_bits, b_bits):
    """BF16(a * b) of two BF16 values in FP32 (kernels.py:274)."""
    return f32_to_bf16(bf16_to_f32(a_bits) * bf16_to_f32(b_bits))


def postg(z, sv_cat, bias_cat, ns, lut=None, act0=False):
    """k_postg: several layers sharing an FP32 (already scaled) row, each rotated; optional activation on the
    first layer's BF16 output (kernels.py:249-261). Returns a list of BF16 arrays."""
    outs, c0 = [], 0
    for i, n in enumerate(ns):
        y = post(z[:, c0:c0 + n], sv_cat[c0:c0 + n], None if bias_cat is None else bias_cat[c0:c0 + n])
        if act0 and i == 0:
            y = act_lut(lut, y)
        outs.append(y)
        c0 += n
    return outs


def pre2(g_bits, u_bits, su):
    """k_pre2: x = BF16(g * u), then sign flip, block Walsh, INT8 (kernels.py:295-307)."""
    return pre(bf16_mul(g_bits, u_bits), 'bf16', su)


def mid2(z, sv_cat, lut, su_down):
    """k_mid2 on the scaled gate | up row z (M, 2N): g = act(BF16(post(gate))), u = BF16(post(up)),
    x = BF16(g * u) -> pre of the down projection (kernels.py:263-278). Returns q, scale."""
    N = z.shape[1] // 2
    g = act_lut(lut, post(z[:, :N], sv_cat[:N]))
    u = post(z[:, N:], sv_cat[N:])
    return pre2(g, u, su_down)


def mid1(z, sv, bias, lut, su_next):
    """k_mid1: act(BF16(post(z) + bias)) -> pre of the next layer (kernels.py:280-292). Returns q, scale."""
    y = act_lut(lut, post(z, sv, bias))
    return pre(y, 'bf16', su_next)
