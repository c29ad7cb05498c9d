"""Seeded synthetic inputs shared by the golden-fixture generator and the tests.

Every input is drawn from numpy's default_rng with a fixed seed, so the fixture generator (which runs the
reference's own tcq_format.py) and the tests (which run the oracle and the CUDA path) see identical bytes.

Layers follow the packed format of deploy/tcq_kernels/tcq_format.py:3-12: bits = uniform uint16 words
(every 512-bit tail-biting stream is a valid code of the L=16 bitshift trellis, tcq_format.py:58-63),
tlut = N(0, 0.968^2) rounded to FP16 (the scale of the k-means table of groot_tcq.py:92-108), row_scale
FP16 in [0.005, 0.03], su / sv random signs.
"""
import numpy as np

# (name, m, n, tokens, input dtype, bias)
LAYERS = [
    ('tile', 16, 16, (1, 3), 'bf16', False),
    ('odd', 48, 80, (1, 5, 17), 'bf16', True),         # 80 = 64 + 16
    ('vit_in', 64, 1152, (3, 20), 'bf16', True),       # 1152 = 1024 + 128
    ('vit_fc2', 32, 4304, (2,), 'f32', False),         # 4304 = 4096 + 128 + 64 + 16
    ('dit', 1536, 1536, (1, 10), 'bf16', False),       # 1536 = 1024 + 512
    ('config1', 4096, 4096, (1,), 'f16', False),       # benchmark config 1
]

# (T, D) for the standalone rotation (config 2 widths; T kept small for the CPU reference)
ROTATIONS = [(1, 16), (3, 48), (2, 1024), (5, 1152), (64, 4096), (2, 4304), (1, 8192), (4, 16384)]

# (M, K, N) for the W8A8 GEMM (config 3 shapes at sizes the CPU reference finishes in seconds)
GEMMS = [(1, 2048, 2048), (16, 2048, 6144), (64, 2048, 2048), (16, 8192, 2048), (3, 80, 48)]


SNAP_TABLES = 64


def snap_inputs(i):
    """Table and row scales for the load-time INT8 snap (tcq_format.py:74-77): tables of varied scale."""
    r = rng('snap', i)
    tlut = (r.standard_normal((512, 2)) * r.uniform(0.2, 3.0)).astype(np.float16)
    rsc = r.uniform(0.001, 0.05, size=64).astype(np.float16)
    return tlut, rsc


def rng(*key):
    seed = 0
    for k in key:
        seed = (seed * 1000003 + (hash_str(k) if isinstance(k, str) else int(k))) % (1 << 63)
    return np.random.default_rng(seed)


def hash_str(s):
    h = 0
    for c in s.encode():
        h = (h * 131 + c) % (1 << 61)
    return h


def f32_to_bf16_bits(x):
    """float32 -> BF16 bit patterns (round to nearest even); the generator only needs finite values."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7fff + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def layer_tensors(name, m, n, bias=False):
    """Packed tensors of one synthetic layer: dict(bits uint16 (m/16*n/16, 32), tlut f16 (512, 2), row_scale f16 (m,),
    su int8 (n,), sv int8 (m,)) and optionally a float32 bias (m,)."""
    r = rng('layer', name, m, n)
    t = dict(
        bits=r.integers(0, 1 << 16, size=((m // 16) * (n // 16), 32), dtype=np.uint32).astype(np.uint16),
        tlut=(r.standard_normal((512, 2)) * 0.968).astype(np.float16),
        row_scale=r.uniform(0.005, 0.03, size=m).astype(np.float16),
        su=np.where(r.random(n) < 0.5, -1, 1).astype(np.int8),
        sv=np.where(r.random(m) < 0.5, -1, 1).astype(np.int8),
    )
    b = (r.standard_normal(m) * 0.1).astype(np.float32) if bias else None
    return t, b


def activations(name, M, K, dtype, scale=3.0):
    """x (M, K) ~ N(0, scale^2): 'bf16' -> uint16 bits, 'f16' -> float16, 'f32' -> float32. Row 0 of a
    multi-row input is all zeros when M >= 5 (the amax = 0 branch of the quantizer)."""
    r = rng('x', name, M, K, dtype)
    x = (r.standard_normal((M, K)) * scale).astype(np.float32)
    if M >= 5:
        x[0] = 0.0
    if dtype == 'bf16':
        return f32_to_bf16_bits(x)
    if dtype == 'f16':
        return x.astype(np.float16)
    return x


def rotation_input(T, D):
    """bf16 [T, D] ~ N(0, 1) and a +-1 sign vector (config 2)."""
    r = rng('rot', T, D)
    x = f32_to_bf16_bits(r.standard_normal((T, D)).astype(np.float32))
    s = np.where(r.random(D) < 0.5, -1, 1).astype(np.int8)
    return x, s


def gemm_inputs(M, K, N):
    """Config 3: A bf16 [M, K] ~ N(0,1) with 1 % of entries x20; W int8 [N, K] uniform in [-127, 127];
    per-channel scales float32 ~ U(1e-3, 1e-2)."""
    r = rng('gemm', M, K, N)
    a = r.standard_normal((M, K)).astype(np.float32)
    out = r.random((M, K)) < 0.01
    a[out] *= 20.0
    w = r.integers(-127, 128, size=(N, K), dtype=np.int32).astype(np.int8)
    sc = r.uniform(1e-3, 1e-2, size=N).astype(np.float32)
    return f32_to_bf16_bits(a), w, sc
