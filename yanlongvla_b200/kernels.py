"""Launch helpers with the reference's operator interface, backed by the sm_100a C ABI.

Mirrors deploy/tcq_kernels/kernels.py of the reference (ForeverBlue816/yanlongvla): the same function names, argument
meaning and buffer layouts, so callers written against the reference work unchanged. Every call launches on
torch.cuda.current_stream(), allocates nothing except the cached per-stream workspace of gemm_tcq, and therefore
works inside torch.cuda.graph() captures. A non-zero status from the library raises TcqError.

  pre      x (M, K) BF16/F16/F32 -> q (M, K) int8 and/or q4 (K/4, ld) int32, scale (M,)     (kernels.py:602-606)
  post     acc (M, lda) I32 / F32 / BF16 columns col0.. -> y (M, N) BF16                    (kernels.py:612-615)
  post3    q / k / v outputs of one accumulator row in one launch                            (kernels.py:618-621)
  postg    up to three layers, one block per (token, layer), optional activation on layer 0  (kernels.py:624-628)
  pre2     BF16(g * u) -> rotate -> INT8                                                      (kernels.py:631-633)
  mid2     gated-MLP middle (GELU-tanh or SiLU)                                               (kernels.py:641-644)
  mid1     plain-MLP middle                                                                   (kernels.py:647-650)
  decode   trellis stream -> dense INT8 weights                                               (kernels.py:653-656)
  gemm_w8  INT8-resident small-M product                                                      (kernels.py:662-668)
  gemm_tcq trellis decode fused into the small-M product                                      (kernels.py:671-673)
  pre_h, decode_bf16                                                                          (kernels.py:677-686)
  rotate   the rotation op: fwht(x * s) and its inverse fwht(y) * s                          (tcq_format.py:44-55)
  int_mm   exact INT8 GEMM on tcgen05 tensor cores, the reference's torch._int_mm(q, W.t())  (modules.py:86)
  int8_gemm  the same with the per-token x per-channel scale epilogue (BF16 / FP32 out)      (tcq_format.py:135)
"""
import torch

from ._lib import DT_BF16, DT_F16, DT_F32, DT_I32, TcqError, check, lib

__all__ = ['quantize', 'pre', 'post', 'post3', 'postg', 'pre2', 'mid2', 'mid1', 'mid2_available', 'decode', 'decode_bf16', 'gemm_w8',
           'gemm_tcq', 'gemm_tcq_x', 'gemm_tcq_tc', 'gemmf_tcq', 'gemmf_w8', 'add_norm', 'chain', 'rope', 'workspace',
           'selftest_wait_expiry', 'pre_h', 'rotate', 'int_mm', 'int8_gemm', 'int8_gemm_bias', 'device_error', 'gelu_table', 'silu_table', 'act_table',
           'TcqError', 'LAUNCHES']

_DT = {torch.bfloat16: DT_BF16, torch.float32: DT_F32, torch.float16: DT_F16, torch.int32: DT_I32}
LAUNCHES = {}            # entry point -> number of calls (launch accounting for the benchmark)


def _p(t):
    return None if t is None else t.data_ptr()


def _stream():
    return torch.cuda.current_stream().cuda_stream


def _count(name):
    LAUNCHES[name] = LAUNCHES.get(name, 0) + 1


def _dt(t, allowed, what):
    if t.dtype not in allowed:
        raise TcqError(f'{what}: dtype {t.dtype} not supported (expected one of {allowed})')
    return _DT[t.dtype]


def _cuda(*ts):
    for t in ts:
        if t is not None and (not t.is_cuda or not t.is_contiguous()):
            raise TcqError('all tensors must be contiguous CUDA tensors')


# ------------------------------------------------------------------------------------------------ activation tables
_TABLES = {}


def act_table(kind='gelu', device=None):
    """BF16 activation of every BF16 bit pattern, computed by PyTorch on the device (65536 entries): the fused kernels
    look the activation up, so they reproduce PyTorch's own result exactly (kernels.py:563-569). kind: 'gelu' (tanh
    approximation, Gemma / SigLIP) or 'silu' (SwiGLU)."""
    device = torch.device('cuda') if device is None else torch.device(device)
    key = (kind, str(device))
    if key not in _TABLES:
        x = torch.arange(65536, dtype=torch.int32, device=device).to(torch.int16).view(torch.bfloat16)
        if kind == 'gelu':
            y = torch.nn.functional.gelu(x, approximate='tanh')
        elif kind == 'silu':
            y = torch.nn.functional.silu(x)
        else:
            raise ValueError(kind)
        _TABLES[key] = y.contiguous()
    return _TABLES[key]


def gelu_table(device=None):
    return act_table('gelu', device)


def silu_table(device=None):
    return act_table('silu', device)


# ------------------------------------------------------------------------------------------------ rotation + quantizer
def pre(x, su, q=None, q4=None, scale=None):
    """x (M, K) BF16 / F16 / F32 contiguous -> q (M, K) int8 and / or q4 (K/4, ld) int32, scale (M,) FP32."""
    _cuda(x, su, q, q4, scale)
    M, K = x.shape
    dt = _dt(x, (torch.bfloat16, torch.float16, torch.float32), 'pre')
    check(lib.tcq_pre(_p(x), dt, _p(su), _p(q), _p(q4), _p(scale), M, K, 0 if q4 is None else q4.shape[1], _stream()), 'tcq_pre')
    _count('pre')


def quantize(x, q=None, scale=None):
    """Per-token INT8 quantizer without rotation (tcq_format.quantize_tokens): x (M, K) -> q (M, K) int8, scale (M,)."""
    M, K = x.shape
    q = torch.empty(M, K, dtype=torch.int8, device=x.device) if q is None else q
    scale = torch.empty(M, dtype=torch.float32, device=x.device) if scale is None else scale
    _cuda(x, q, scale)
    check(lib.tcq_quantize(_p(x), _dt(x, (torch.bfloat16, torch.float16, torch.float32), 'quantize'), _p(q), _p(scale), M, K,
                           _stream()), 'tcq_quantize')
    _count('quantize')
    return q, scale


def pre2(g, u, su, q=None, q4=None, scale=None):
    _cuda(g, u, su, q, q4, scale)
    M, K = g.shape
    check(lib.tcq_pre2(_p(g), _p(u), _p(su), _p(q), _p(q4), _p(scale), M, K, 0 if q4 is None else q4.shape[1], _stream()),
          'tcq_pre2')
    _count('pre2')


def pre_h(x, su, h=None, hT=None):
    _cuda(x, su, h, hT)
    M, K = x.shape
    dt = _dt(x, (torch.bfloat16, torch.float16, torch.float32), 'pre_h')
    check(lib.tcq_pre_h(_p(x), dt, _p(su), _p(h), _p(hT), M, K, 0 if hT is None else hT.shape[1], _stream()), 'tcq_pre_h')
    _count('pre_h')


def _acc_dt(acc):
    return _dt(acc, (torch.int32, torch.float32, torch.bfloat16), 'accumulator')


def post(acc, s, rs, sv, bias, y, col0=0):
    """acc (M, lda) int32 (scaled here by s, rs), FP32 (already scaled) or BF16 (scaled by rs); columns col0 .. col0 + N
    -> y (M, N) BF16."""
    _cuda(acc, s, rs, sv, bias, y)
    M, N = y.shape
    check(lib.tcq_post(_p(acc), _acc_dt(acc), _p(s), _p(rs), _p(sv), _p(bias), _p(y), M, N, acc.shape[1], col0, _stream()),
          'tcq_post')
    _count('post')


def post3(acc, s, rs, sv, bias, ys):
    """q / k / v in one launch: rs, sv, bias concatenated over the three layers; ys = three (M, N_i) BF16 outputs."""
    _cuda(acc, s, rs, sv, bias, *ys)
    M = ys[0].shape[0]
    n = [y.shape[1] for y in ys]
    check(lib.tcq_post3(_p(acc), _acc_dt(acc), _p(s), _p(rs), _p(sv), _p(bias), _p(ys[0]), _p(ys[1]), _p(ys[2]), M, n[0], n[1],
                        n[2], acc.shape[1], _stream()), 'tcq_post3')
    _count('post3')


def postg(acc, s, rs, sv, bias, ys, gelu0=False, act='gelu'):
    """Two or three layers sharing the accumulator row, one block per (token, layer); optional activation (GELU-tanh,
    or SiLU with act='silu') on the first layer's output."""
    _cuda(acc, s, rs, sv, bias, *ys)
    M = ys[0].shape[0]
    yy = list(ys) + [None] * (3 - len(ys))
    n = [y.shape[1] for y in ys] + [0] * (3 - len(ys))
    lut = act_table(act, acc.device) if gelu0 else None
    check(lib.tcq_postg(_p(acc), _acc_dt(acc), _p(s), _p(rs), _p(sv), _p(bias), _p(lut), _p(yy[0]), _p(yy[1]), _p(yy[2]), M,
                        n[0], n[1], n[2], acc.shape[1], int(bool(gelu0)), _stream()), 'tcq_postg')
    _count('postg')


def mid2_available(N):
    """The fused gated-MLP middle holds N floats + N BF16 per token in shared memory: up to 16384 wide on sm_100a."""
    return N <= 16384


def mid2(acc, s, rs, sv, su, q=None, q4=None, scale=None, act='gelu'):
    """Gated-MLP middle: acc (M, 2N) gate | up; rs, sv concatenated (2N); su = input signs of the down projection (N)."""
    _cuda(acc, s, rs, sv, su, q, q4, scale)
    M = acc.shape[0]
    N = su.shape[0]
    lut = act_table(act, acc.device)
    check(lib.tcq_mid2(_p(acc), _acc_dt(acc), _p(s), _p(rs), _p(sv), _p(lut), _p(su), _p(q), _p(q4), _p(scale), M, N,
                       acc.shape[1], 0 if q4 is None else q4.shape[1], _stream()), 'tcq_mid2')
    _count('mid2')


def mid1(acc, s, rs, sv, bias, su, q=None, q4=None, scale=None, act='gelu'):
    """Plain-MLP middle: acc (M, N) of the first layer; su = input signs of the second layer."""
    _cuda(acc, s, rs, sv, bias, su, q, q4, scale)
    M, N = acc.shape
    lut = act_table(act, acc.device)
    check(lib.tcq_mid1(_p(acc), _acc_dt(acc), _p(s), _p(rs), _p(sv), _p(bias), _p(lut), _p(su), _p(q), _p(q4), _p(scale), M, N,
                       N, 0 if q4 is None else q4.shape[1], _stream()), 'tcq_mid1')
    _count('mid1')


def rotate(x, signs, inverse=False, out_dtype=torch.float32, out=None):
    """The rotation op: forward y = fwht(x * signs), inverse y = fwht(x) * signs, over the last dim (block Walsh over
    its binary decomposition, FP32 arithmetic). x (..., D) BF16 / F16 / F32; y FP32 or BF16."""
    shape = x.shape
    x2 = x.reshape(-1, shape[-1])
    if not x2.is_contiguous():
        x2 = x2.contiguous()
    M, D = x2.shape
    y = torch.empty(M, D, dtype=out_dtype, device=x.device) if out is None else out.view(M, D)
    _cuda(x2, signs, y)
    dt = _dt(x2, (torch.bfloat16, torch.float16, torch.float32), 'rotate')
    check(lib.tcq_rotate(_p(x2), dt, _p(signs), _p(y), _dt(y, (torch.float32, torch.bfloat16), 'rotate out'), M, D,
                         int(bool(inverse)), _stream()), 'tcq_rotate')
    _count('rotate')
    return y.view(*shape)


# ------------------------------------------------------------------------------------------------ W2 float path
def gemmf_tcq(bits, t8, hT, rs, z, K, bounds=(1 << 30, 1 << 30)):
    """W2 product with the trellis decode fused (reference kernels.gemmf_tcq): hT (K, ld) BF16 rotated activations
    (pre_h's hT), t8 per-layer INT8 tables, FP32 accumulation -> z (M, N) = (h . w) * rs."""
    M, N = z.shape
    _cuda(bits, t8, hT, rs, z)
    if hT.dtype != torch.bfloat16 or hT.shape[0] != K or hT.shape[1] < M:
        raise TcqError('gemmf_tcq: hT must be (K, >= M) BF16')
    check(lib.tcq_gemmf_tcq(_p(bits), _p(t8), _p(hT), _p(rs), _p(z), M, N, K, hT.shape[1], int(bounds[0]), int(bounds[1]),
                            _stream()), 'tcq_gemmf_tcq')
    _count('gemmf_tcq')
    return z


def gemmf_w8(W, hT, rs, z):
    """W2 product on INT8-resident weights W (N, K) (reference kernels.gemmf_w8)."""
    M, N = z.shape
    K = W.shape[1]
    _cuda(W, hT, rs, z)
    if hT.dtype != torch.bfloat16 or hT.shape[0] != K or hT.shape[1] < M or W.shape[0] != N:
        raise TcqError('gemmf_w8: hT must be (K, >= M) BF16 and W (N, K)')
    check(lib.tcq_gemmf_w8(_p(W), _p(hT), _p(rs), _p(z), M, N, K, hT.shape[1], _stream()), 'tcq_gemmf_w8')
    _count('gemmf_w8')
    return z


# ------------------------------------------------------------------------------------------------ policy glue
def add_norm(x, y=None, weight=None, bias=None, eps=1e-6, kind='rms', h_out=None, out=None, mod=None, mod_rows=1):
    """Residual add + RMSNorm / LayerNorm in one launch (tcq_add_norm). x, y (..., D) BF16; returns (h, n) with
    h = x + y (x itself when y is None; written to h_out when given, which may be x) and n = norm(h) in BF16.
    kind 'rms': n = (h * rsqrt(mean(h^2) + eps)) * weight; kind 'ln': n = ((h - mean) * rsqrt(var + eps)) * weight + bias
    (weight / bias FP32, None = 1 / 0). mod = (scale, shift) BF16 (G, D) views, one row per group of mod_rows rows:
    n = n * (1 + scale) + shift."""
    shape = x.shape
    D = shape[-1]
    x2 = x.reshape(-1, D)
    M = x2.shape[0]
    y2 = None if y is None else y.reshape(-1, D)
    for t in (x2, y2):
        if t is not None and (t.dtype != torch.bfloat16 or not t.is_contiguous()):
            raise TypeError('add_norm: x and y must be contiguous BF16')
    h = x2 if y2 is None else (torch.empty_like(x2) if h_out is None else h_out.view(M, D))
    n = torch.empty_like(x2) if out is None else out.view(M, D)
    ms = mh = None
    ld = 0
    if mod is not None:
        ms, mh = mod
        if ms.dtype != torch.bfloat16 or mh.dtype != torch.bfloat16 or ms.stride(-1) != 1 or ms.stride(0) != mh.stride(0):
            raise TypeError('add_norm: mod must be BF16 (G, D) views with unit inner stride')
        ld = ms.stride(0) if ms.dim() > 1 else D
    _cuda(x2, n, *(t for t in (y2, weight, bias) if t is not None))
    if ms is not None and not (ms.is_cuda and mh.is_cuda and ms.shape[-1] == D and mh.shape[-1] == D):
        raise TcqError('add_norm: mod must be CUDA (G, D) tensors')
    if h.shape != x2.shape or n.shape != x2.shape or (y2 is not None and y2.shape != x2.shape):
        raise TcqError('add_norm: x, y and the outputs must have the same shape')
    wdt = [t.dtype for t in (weight, bias) if t is not None]
    if any(d != wdt[0] for d in wdt) or (wdt and wdt[0] not in (torch.float32, torch.bfloat16)):
        raise TcqError(f'add_norm: weight / bias must both be float32 or both bfloat16, got {wdt}')
    for t in (weight, bias):
        if t is not None and t.numel() != D:
            raise TcqError(f'add_norm: weight / bias must have {D} elements')
    check(lib.tcq_add_norm(_p(x2), None if y2 is None else _p(y2), None if y2 is None else _p(h), _p(n),
                           None if weight is None else _p(weight), None if bias is None else _p(bias),
                           _DT[wdt[0]] if wdt else DT_F32,
                           None if ms is None else _p(ms), None if mh is None else _p(mh), int(mod_rows), int(ld),
                           float(eps), {'rms': 0, 'ln': 1}[kind], M, D, _stream()), 'tcq_add_norm')
    _count('add_norm')
    return h.view(shape), n.view(shape)


def chain(x, kind, weight=None, nbias=None, eps=1e-6, *, acc=None, s=None, rs=None, sv=None, bias=None, col0=0, y=None,
          mod=None, mod_rows=1, su=None, q=None, q4=None, scale=None, h_out=None, want_n=True):
    """Fused post -> residual add -> norm -> pre of one block boundary (tcq_chain). x (M, N) BF16 residual; the add
    takes the post of acc (FP32 z, or INT32 with token scales s and row scales rs; sv / bias of the producing layer,
    its columns from col0) or a BF16 tensor y; the norm is add_norm's (kind, weight, nbias, eps, mod); with su the next
    layer's rotation + INT8 quantization goes to q and/or q4 (K/4, ldq) words and scale (M,); with q / q4 but no su,
    the plain per-token quantization of BF16(n) (a W8A8 consumer, kernels.quantize's arithmetic). Returns (h, n): h the
    new residual (x itself without an add), n the BF16 norm output (None when want_n is False)."""
    M, N = x.shape
    if x.dtype != torch.bfloat16 or not x.is_contiguous():
        raise TcqError('chain: x must be contiguous (M, N) BF16')
    if acc is not None and y is not None:
        raise TcqError('chain: give acc or y, not both')
    adt = 0
    if acc is not None:
        adt = _dt(acc, (torch.float32, torch.int32), 'chain acc')
        if acc.dim() != 2 or acc.shape[0] != M or acc.shape[1] < col0 + N:
            raise TcqError('chain: acc must be (M, >= col0 + N)')
    if y is not None and (y.shape != x.shape or y.dtype != torch.bfloat16):
        raise TcqError('chain: y must be (M, N) BF16')
    wdt = [t.dtype for t in (weight, nbias) if t is not None]
    if any(d != wdt[0] for d in wdt) or (wdt and wdt[0] not in (torch.float32, torch.bfloat16)):
        raise TcqError(f'chain: norm weight / bias must both be float32 or both bfloat16, got {wdt}')
    for t in (weight, nbias, sv, su):
        if t is not None and t.numel() != N:
            raise TcqError(f'chain: per-column vectors must have {N} elements')
    ms = mh = None
    ld = 0
    if mod is not None:
        ms, mh = mod
        if ms.dtype != torch.bfloat16 or mh.dtype != torch.bfloat16 or ms.shape[-1] != N or ms.stride(-1) != 1 or ms.stride(0) != mh.stride(0):
            raise TcqError('chain: mod must be BF16 (G, N) views with unit inner stride')
        ld = ms.stride(0)
    quant = su is not None or q is not None or q4 is not None
    if quant and (scale is None or (q is None and q4 is None)):
        raise TcqError('chain: the quantized output needs scale and q and/or q4')
    h = x if (acc is None and y is None) else (torch.empty_like(x) if h_out is None else h_out)
    n = torch.empty_like(x) if (want_n or not quant) else None
    _cuda(x, acc, y, h, n, weight, nbias, sv, bias, su, q, q4, scale)
    check(lib.tcq_chain(_p(acc), adt, _p(s), _p(rs), _p(sv), _p(bias), 0 if acc is None else acc.shape[1], int(col0),
                        _p(y), _p(x), None if (acc is None and y is None) else _p(h), _p(n), _p(weight), _p(nbias),
                        _DT[wdt[0]] if wdt else DT_F32, _p(ms), _p(mh), int(mod_rows), int(ld), float(eps),
                        {'rms': 0, 'ln': 1}[kind], _p(su), _p(q), _p(q4), _p(scale), 0 if q4 is None else q4.shape[1], M, N,
                        _stream()), 'tcq_chain')
    _count('chain')
    return h, n


def rope(x, cos, sin, heads, out=None):
    """Rotary embedding (half-split form) on x (B, T, heads * D) BF16 with cos / sin (T, D/2) FP32 tables."""
    B, T, W = x.shape
    D = W // heads
    if x.dtype != torch.bfloat16 or x.stride(-1) != 1 or x.stride(0) != T * x.stride(1):
        raise TypeError('rope: x must be BF16 with contiguous rows')
    y = torch.empty(B, T, W, dtype=torch.bfloat16, device=x.device) if out is None else out
    _cuda(x, y, cos, sin)
    if W % heads or D % 2 or y.shape != x.shape or y.dtype != torch.bfloat16:
        raise TcqError('rope: x (B, T, heads * D) with even D, out of the same shape, BF16')
    if cos.dtype != torch.float32 or sin.dtype != torch.float32 or cos.shape != (T, D // 2) or sin.shape != (T, D // 2):
        raise TcqError(f'rope: cos / sin must be float32 ({T}, {D // 2})')
    check(lib.tcq_rope(_p(x), _p(y), _p(cos), _p(sin), B * T, T, heads, D, x.stride(1), y.stride(1), _stream()), 'tcq_rope')
    _count('rope')
    return y


# ------------------------------------------------------------------------------------------------ trellis weights
def decode(bits, t8, out):
    """bits (m/16 * n/16, 32) int16/uint16 words, t8 (512, 2) int8 -> out (m, n) int8."""
    _cuda(bits, t8, out)
    m, n = out.shape
    check(lib.tcq_decode(_p(bits), _p(t8), _p(out), m, n, _stream()), 'tcq_decode')
    _count('decode')


def decode_bf16(bits, tb, out):
    _cuda(bits, tb, out)
    m, n = out.shape
    check(lib.tcq_decode_bf16(_p(bits), _p(tb), _p(out), m, n, _stream()), 'tcq_decode_bf16')
    _count('decode_bf16')


def gemm_w8(W, q4, s, rs, z):
    """W (N, K) int8 resident, q4 (K/4, M) int32, z (M, N) FP32 = ((float)acc * s) * rs."""
    _cuda(W, q4, s, rs, z)
    N, K = W.shape
    M = q4.shape[1]
    check(lib.tcq_gemm_w8(_p(W), _p(q4), _p(s), _p(rs), _p(z), M, N, K, _stream()), 'tcq_gemm_w8')
    _count('gemm_w8')


_WS = {}


def workspace(M, N, device):
    """Zero-filled workspace of tcq_gemm_tcq / tcq_gemm_tcq_tc for the current stream (every call leaves it zero;
    grown on demand)."""
    need = max(int(lib.tcq_gemm_tcq_workspace(M, N)), int(lib.tcq_gemm_tcq_tc_workspace(M, N)))
    key = (str(device), _stream())
    ws = _WS.get(key)
    if ws is None or ws.numel() * 4 < need:
        ws = torch.zeros(max(need // 4, 1 << 16), dtype=torch.int32, device=device)
        _WS[key] = ws
    return ws


def gemm_tcq(bits, t8, q4, s, rs, z, K, bounds=(1 << 30, 1 << 30)):
    """Fused trellis decode + product: bits (N/16 * K/16, 32) of up to three row-concatenated layers, t8 their tables
    concatenated (1024 bytes each), bounds = tile-row boundaries between layers; z (M, N) FP32."""
    _cuda(bits, t8, q4, s, rs, z)
    M, N = z.shape
    ws = workspace(M, N, z.device)
    check(lib.tcq_gemm_tcq(_p(bits), _p(t8), _p(q4), _p(s), _p(rs), _p(z), M, N, K, int(bounds[0]), int(bounds[1]), _p(ws),
                           ws.numel() * 4, _stream()), 'tcq_gemm_tcq')
    _count('gemm_tcq')


GEMV_X_MAX_M, GEMV_X_MAX_K = 4, 8192


def gemm_tcq_x(bits, t8, x, su, rs, z, K, bounds=(1 << 30, 1 << 30)):
    """pre + gemm_tcq in one launch (tcq_gemm_tcq_x) for M <= 4 tokens and K <= 8192: x (M, K) BF16 / F16 / F32
    activations, su the layer's input signs; z (M, N) FP32 exactly as pre followed by gemm_tcq."""
    _cuda(bits, t8, x, su, rs, z)
    M, N = z.shape
    if x.shape != (M, K):
        raise TcqError(f'gemm_tcq_x: x must be ({M}, {K})')
    dt = _dt(x, (torch.bfloat16, torch.float16, torch.float32), 'gemm_tcq_x')
    ws = workspace(M, N, z.device)
    check(lib.tcq_gemm_tcq_x(_p(bits), _p(t8), _p(x), dt, _p(su), _p(rs), _p(z), M, N, K, int(bounds[0]), int(bounds[1]),
                             _p(ws), ws.numel() * 4, _stream()), 'tcq_gemm_tcq_x')
    _count('gemm_tcq_x')


# ------------------------------------------------------------------------------------------------ W8A8 GEMM
def int_mm(q, W, out=None):
    """acc (M, N) int32 = q (M, K) int8 @ W (N, K) int8 ^T, exact (tcgen05 kind::i8); replaces torch._int_mm(q, W.t())."""
    _cuda(q, W, out)
    M, K = q.shape
    N = W.shape[0]
    out = torch.empty(M, N, dtype=torch.int32, device=q.device) if out is None else out
    check(lib.tcq_int_mm(_p(q), _p(W), _p(out), M, N, K, _stream()), 'tcq_int_mm')
    _count('int_mm')
    return out


def int8_gemm(q, W, s_tok, s_ch, out=None, out_dtype=torch.bfloat16):
    """out (M, N) = ((float)(q @ W^T) * s_tok[:, None]) * s_ch[None, :] in BF16 or FP32, one launch."""
    _cuda(q, W, s_tok, s_ch, out)
    M, K = q.shape
    N = W.shape[0]
    out = torch.empty(M, N, dtype=out_dtype, device=q.device) if out is None else out
    check(lib.tcq_int8_gemm(_p(q), _p(W), _p(s_tok), _p(s_ch), _p(out), _dt(out, (torch.bfloat16, torch.float32), 'int8_gemm out'),
                            M, N, K, _stream()), 'tcq_int8_gemm')
    _count('int8_gemm')
    return out


def int8_gemm_bias(q, W, s_tok, s_ch, bias=None, act=None, out=None):
    """out (M, N) BF16 = act(BF16(int8_gemm(q, W, s_tok, s_ch)) + bias) in one launch (tcq_int8_gemm_bias): the BF16
    product, the bias as a BF16 tensor add, then the activation table `act` (kernels.act_table: 'gelu' / 'silu') or
    none, bit-identical to the three PyTorch ops."""
    _cuda(q, W, s_tok, s_ch, bias, out)
    M, K = q.shape
    N = W.shape[0]
    if bias is not None and (bias.dtype != torch.bfloat16 or bias.numel() != N or not bias.is_contiguous()):
        raise TcqError('int8_gemm_bias: bias must be a contiguous (N,) BF16 vector')
    lut = None if act is None else act_table(act, q.device)
    out = torch.empty(M, N, dtype=torch.bfloat16, device=q.device) if out is None else out
    if out.dtype != torch.bfloat16 or out.shape != (M, N):
        raise TcqError('int8_gemm_bias: out must be (M, N) BF16')
    check(lib.tcq_int8_gemm_bias(_p(q), _p(W), _p(s_tok), _p(s_ch), _p(bias), _p(lut), _p(out), M, N, K, _stream()),
          'tcq_int8_gemm_bias')
    _count('int8_gemm')
    return out


def selftest_wait_expiry(limit_us=10000):
    """Run the bounded-wait failure path once (tcq_selftest_wait_expiry): returns the device error flags afterwards
    (1 expected), then clears them."""
    check(lib.tcq_selftest_wait_expiry(int(limit_us), _stream()), 'tcq_selftest_wait_expiry')
    flags = device_error(reset=True)
    return flags


def device_error(reset=True):
    """Error flags raised by the kernels' bounded pipeline waits (0 = none). Synchronizes the device."""
    return int(lib.tcq_device_error(int(bool(reset))))


def gemm_tcq_tc(bits, t8, q, s, rs, z, K, bounds=(1 << 30, 1 << 30)):
    """Tensor-core fused decode-GEMM: q (M, K) int8 row-major (pre's q output), 1 <= M <= 256; z (M, N) FP32 =
    ((float)acc * s) * rs, the weights decoded from the trellis stream inside the kernel. Layer bounds (tile rows) must
    be multiples of 8."""
    _cuda(bits, t8, q, s, rs, z)
    M, N = z.shape
    ws = workspace(M, N, z.device)
    check(lib.tcq_gemm_tcq_tc(_p(bits), _p(t8), _p(q), _p(s), _p(rs), _p(z), M, N, K, int(bounds[0]), int(bounds[1]), _p(ws),
                              ws.numel() * 4, _stream()), 'tcq_gemm_tcq_tc')
    _count('gemm_tcq_tc')
