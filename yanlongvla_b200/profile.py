"""Kernel-class breakdown of one CUDA-graph replay (the reference's runner.kernel_classes, runner.py:227-266).

A torch.profiler (CUPTI) trace of a single replay; device time per kernel class, launch counts, wall time and the
gaps between kernels, plus each class's share of the critical path (a kernel's time from the previous kernel's end to
its own end: with programmatic dependent launch a kernel's own time range includes its wait for the predecessor).
Classes are matched by regex on the kernel name, first match wins.
"""
import re
from collections import Counter, defaultdict

import torch

CLASSES = [
    ('trellis decode-GEMV (SIMT)', r'k_gemm_tcq<'),
    ('trellis decode-GEMM (tcgen05)', r'k_gemm_tcq_tc'),
    ('trellis decode', r'k_decode'),
    ('INT8 GEMM (tcgen05)', r'k_gemm_i8'),
    ('INT8-resident GEMV', r'k_gemm_w8'),
    ('rotate + quantize', r'k_pre|k_quant'),
    ('post + add + norm + pre chain', r'k_chain'),
    ('scale + rotate', r'k_post'),
    ('MLP middles', r'k_mid'),
    ('attention', r'flash|fmha|attention|softmax|sdpa'),
    ('matrix product (BF16, cuBLAS)', r'gemm|cutlass|cublas|Gemv|gemv|matmul|nvjet'),
    ('norm', r'rms|layer_norm|LayerNorm|norm'),
    ('copies / casts', r'copy|cast|Copy|fill|zero|memset|Memset|memcpy|Memcpy'),
    ('NCCL', r'nccl'),
    ('other elementwise', r'.*'),
]


def kernel_classes(graph, warm=3):
    """Profile one replay of `graph` (a torch.cuda.CUDAGraph). Returns a dict of times in ms."""
    from torch.profiler import ProfilerActivity, profile
    for _ in range(warm):
        graph.replay()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with profile(activities=[ProfilerActivity.CUDA, ProfilerActivity.CPU]) as prof:
        start.record()
        graph.replay()
        end.record()
        end.synchronize()
    wall = start.elapsed_time(end)
    by, launches, top = defaultdict(float), Counter(), Counter()
    excl, excl_top = defaultdict(float), Counter()
    kernels = sorted((e for e in prof.events() if e.device_type.name == 'CUDA'), key=lambda e: e.time_range.start)
    prev_end = None
    for e in kernels:
        dur = e.time_range.elapsed_us() / 1000
        cls = next(c for c, pat in CLASSES if re.search(pat, e.name))
        by[cls] += dur
        launches[cls] += 1
        name = e.name.replace('(anonymous namespace)::', '')[:90]
        top[name] += dur
        # Kernels launched early by programmatic dependent launch wait for their predecessor inside their own time
        # range, so a kernel's share of the critical path is the time from the previous kernel's end to its own end.
        t0, t1 = e.time_range.start, e.time_range.end
        x = (t1 - max(t0, prev_end if prev_end is not None else t0)) / 1000
        if x > 0:
            excl[cls] += x
            excl_top[name] += x
        prev_end = t1 if prev_end is None else max(prev_end, t1)
    total = sum(by.values())
    return dict(wall_ms=wall, kernel_ms=total, gaps_ms=max(wall - sum(excl.values()), 0.0), launches=sum(launches.values()),
                by_class_ms={k: round(v, 3) for k, v in sorted(by.items(), key=lambda kv: -kv[1])},
                critical_path_ms_by_class={k: round(v, 3) for k, v in sorted(excl.items(), key=lambda kv: -kv[1])},
                launches_by_class=dict(launches), top=[(nm, round(d, 3)) for nm, d in top.most_common(12)],
                critical_path_top=[(nm, round(d, 3)) for nm, d in excl_top.most_common(16)])


# ----------------------------------------------------------------------------------------------- profiling cases
# Small, seeded invocations of one kernel each, for a profiler to capture (nothing is timed or checked here):
#   python -m yanlongvla_b200.profile gemv [--n 4096] [--k 4096] [--tokens 1] [--launches 4]
#   python -m yanlongvla_b200.profile gemm [--m 4096] [--k 2048] [--n 8192] [--out i32|bf16] [--launches 4]
#   python -m yanlongvla_b200.profile pre|rotate [--m 4096] [--k 4096] [--launches 4]
#   python -m yanlongvla_b200.profile chain [--m 17] [--k 1536] [--launches 6]
#   python -m yanlongvla_b200.profile gemv_tc [--n 1536] [--k 1536] [--tokens 17] [--launches 4]
#   python -m yanlongvla_b200.profile policy [--tokens 1]    (kernel_classes of one chunk-graph replay, as JSON)
# `gemv` runs kernels.gemm_tcq on one trellis layer (uniform random streams, a snapped table), `gemm` runs
# kernels.int_mm (INT32 out) or kernels.int8_gemm (BF16 out with the scale epilogue) on uniform INT8 operands. Every launch of a case is identical, so the ones after the first two
# are warm in the driver and the code caches.
def _case_gemv(n, k, tokens, launches):
    from . import kernels as K
    from .tcq_format import snap
    dev = torch.device('cuda')
    g = torch.Generator(device=dev).manual_seed(11)
    bits = torch.randint(-32768, 32768, ((n // 16) * (k // 16), 32), dtype=torch.int32, device=dev, generator=g).to(torch.int16)
    t8, rs, _ = snap((torch.randn(512, 2, device=dev, generator=g) * 0.968).half(),
                     (torch.rand(n, device=dev, generator=g) * 0.02 + 0.005).half())
    q4 = torch.randint(-2 ** 31, 2 ** 31 - 1, (k // 4, tokens), dtype=torch.int32, device=dev, generator=g)
    s = torch.rand(tokens, device=dev, generator=g)
    z = torch.empty(tokens, n, device=dev)
    t8, rs = t8.contiguous(), rs.contiguous()
    for _ in range(launches):
        K.gemm_tcq(bits, t8, q4, s, rs, z, k)


def _case_gemv_tc(n, k, tokens, launches):
    """kernels.gemm_tcq_tc (tensor-core fused decode-GEMM) on one trellis layer and `tokens` INT8 token rows."""
    from . import kernels as K
    from .tcq_format import snap
    dev = torch.device('cuda')
    g = torch.Generator(device=dev).manual_seed(15)
    bits = torch.randint(-32768, 32768, ((n // 16) * (k // 16), 32), dtype=torch.int32, device=dev, generator=g).to(torch.int16)
    t8, rs, _ = snap((torch.randn(512, 2, device=dev, generator=g) * 0.968).half(),
                     (torch.rand(n, device=dev, generator=g) * 0.02 + 0.005).half())
    q = torch.randint(-127, 128, (tokens, k), dtype=torch.int8, device=dev, generator=g)
    s = torch.rand(tokens, device=dev, generator=g)
    z = torch.empty(tokens, n, device=dev)
    t8, rs = t8.contiguous(), rs.contiguous()
    for _ in range(launches):
        K.gemm_tcq_tc(bits, t8, q, s, rs, z, k)


def _case_gemm(m, k, n, launches, out_kind='i32'):
    from . import kernels as K
    dev = torch.device('cuda')
    g = torch.Generator(device=dev).manual_seed(12)
    q = torch.randint(-127, 128, (m, k), dtype=torch.int8, device=dev, generator=g)
    w = torch.randint(-127, 128, (n, k), dtype=torch.int8, device=dev, generator=g)
    if out_kind == 'bf16':
        s_tok = torch.rand(m, device=dev, generator=g) * 1e-2
        s_ch = torch.rand(n, device=dev, generator=g) * 1e-3
        out = torch.empty(m, n, dtype=torch.bfloat16, device=dev)
        for _ in range(launches):
            K.int8_gemm(q, w, s_tok, s_ch, out=out)
        return
    out = torch.empty(m, n, dtype=torch.int32, device=dev)
    for _ in range(launches):
        K.int_mm(q, w, out=out)


def _case_rows(kind, m, k, launches):
    """kernels.pre (BF16 -> INT8 + scales) or kernels.rotate (BF16 -> FP32) on an (m, k) activation."""
    from . import kernels as K
    dev = torch.device('cuda')
    g = torch.Generator(device=dev).manual_seed(13)
    x = torch.randn(m, k, device=dev, generator=g).bfloat16()
    su = (torch.randint(0, 2, (k,), device=dev, generator=g) * 2 - 1).to(torch.int8)
    q = torch.empty(m, k, dtype=torch.int8, device=dev)
    s = torch.empty(m, device=dev)
    y = torch.empty(m, k, device=dev)
    for _ in range(launches):
        if kind == 'pre':
            K.pre(x, su, q=q, scale=s)
        else:
            K.rotate(x, su, out=y)


def _case_chain(m, n, launches):
    """kernels.chain at a DiT block boundary: FP32 z of the previous layer -> post -> residual add -> RMSNorm -> the
    next layer's pre (INT8 + scales)."""
    from . import kernels as K
    dev = torch.device('cuda')
    g = torch.Generator(device=dev).manual_seed(14)
    x = torch.randn(m, n, device=dev, generator=g).bfloat16()
    z = torch.randn(m, n, device=dev, generator=g)
    w = (torch.rand(n, device=dev, generator=g) + 0.5).bfloat16()
    sv = (torch.randint(0, 2, (n,), device=dev, generator=g) * 2 - 1).to(torch.int8)
    su = (torch.randint(0, 2, (n,), device=dev, generator=g) * 2 - 1).to(torch.int8)
    q = torch.empty(m, n, dtype=torch.int8, device=dev)
    s = torch.empty(m, device=dev)
    for _ in range(launches):
        K.chain(x, 'rms', w, None, 1e-6, acc=z, sv=sv, su=su, q=q, scale=s, want_n=False)


def _case_policy(batch):
    """kernel_classes of one CUDA-graph replay of the fly policy's action chunk for `batch` observations."""
    import json
    from . import policy as P
    c = P.PolicyConfig()
    model, _, _ = P.build_policy('cuda', 'fly', c)
    obs = P.synthetic_observations(batch, c)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.no_grad(), torch.cuda.stream(s):
        for _ in range(2):
            model(*obs)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.no_grad(), torch.cuda.graph(g):
        model(*obs)
    print(json.dumps(kernel_classes(g), indent=1))


def main(argv=None):
    import argparse
    ap = argparse.ArgumentParser(description='one kernel case for a profiler')
    ap.add_argument('case', choices=['gemv', 'gemv_tc', 'gemm', 'pre', 'rotate', 'chain', 'policy'])
    ap.add_argument('--m', type=int, default=4096)
    ap.add_argument('--n', type=int, default=None)
    ap.add_argument('--k', type=int, default=None)
    ap.add_argument('--tokens', type=int, default=1)
    ap.add_argument('--launches', type=int, default=4)
    ap.add_argument('--out', choices=['i32', 'bf16'], default='i32', help='gemm case: INT32 or BF16 (scaled) output')
    a = ap.parse_args(argv)
    if a.case == 'gemv':
        _case_gemv(a.n or 4096, a.k or 4096, a.tokens, a.launches)
    elif a.case == 'gemv_tc':
        _case_gemv_tc(a.n or 1536, a.k or 1536, a.tokens, a.launches)
    elif a.case == 'gemm':
        _case_gemm(a.m, a.k or 2048, a.n or 8192, a.launches, a.out)
    elif a.case == 'policy':
        _case_policy(a.tokens)
    elif a.case == 'chain':
        _case_chain(a.m, a.k or 1536, a.launches)
    else:
        _case_rows(a.case, a.m, a.k or 4096, a.launches)
    torch.cuda.synchronize()
    from . import kernels as K
    err = K.device_error()
    print('ok', a.case, 'device_error', err)
    return 0 if err == 0 else 1


if __name__ == '__main__':
    raise SystemExit(main())
