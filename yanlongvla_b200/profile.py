"""Where one CUDA-graph replay spends its time, by kernel class, and small seeded kernel cases for a profiler.

`replay_breakdown(graph)` traces a single replay with torch.profiler (CUPTI) and attributes every device kernel to a
class (`classify`). Besides each class's device time it reports each class's share of the critical path: walking the
kernels in start order, a kernel is charged only for the time by which it moves the end of the work done so far
(with programmatic dependent launch a kernel starts early and waits for its predecessor inside its own time range,
so its raw duration overstates what it costs). What the replay spends outside every kernel is the idle time.
"""
import re
from collections import defaultdict

import torch

# (class, name fragments) in priority order: a kernel belongs to the first class one of whose fragments its
# (demangled) name contains; names matching nothing are 'other'.
_FRAGMENTS = (
    ('trellis decode-GEMV (SIMT)', ('k_gemm_tcq<',)),
    ('trellis decode-GEMM (tcgen05)', ('k_gemm_tcq_tc',)),
    ('trellis decode', ('k_decode',)),
    ('INT8 GEMM (tcgen05)', ('k_gemm_i8',)),
    ('INT8-resident GEMV', ('k_gemm_w8',)),
    ('rotate + quantize', ('k_pre', 'k_quant')),
    ('post + add + norm + pre chain', ('k_chain',)),
    ('scale + rotate', ('k_post',)),
    ('MLP middles', ('k_mid',)),
    ('residual add + norm', ('k_addnorm', 'k_add_norm')),
    ('rotary embedding', ('k_rope',)),
    ('attention', ('flash', 'fmha', 'attention', 'softmax', 'sdpa', 'cudnn')),
    ('BF16 matrix product (cuBLAS)', ('gemm', 'Gemm', 'gemv', 'Gemv', 'cublas', 'nvjet', 'cutlass', 'matmul')),
    ('NCCL', ('nccl', 'Nccl')),
    ('memory copies and fills', ('memcpy', 'Memcpy', 'memset', 'Memset', 'copy_', 'fill_', 'zero_')),
)


def classify(kernel_name):
    for cls, frags in _FRAGMENTS:
        if any(f in kernel_name for f in frags):
            return cls
    return 'other'


def _short(name, width=90):
    return re.sub(r'\(anonymous namespace\)::', '', name)[:width]


def replay_breakdown(graph, warm=3):
    """Trace one replay of `graph` (a torch.cuda.CUDAGraph) after `warm` untraced ones. Returns times in ms: the
    replay's wall time (CUDA events), total kernel time, idle time, launches, and per class the device time, the
    critical-path share and the launch count, plus the heaviest kernels by each measure."""
    from torch.profiler import ProfilerActivity, profile
    for _ in range(warm):
        graph.replay()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with profile(activities=[ProfilerActivity.CUDA, ProfilerActivity.CPU]) as trace:
        ev0.record()
        graph.replay()
        ev1.record()
        ev1.synchronize()
    replay_ms = ev0.elapsed_time(ev1)
    spans = sorted(((e.time_range.start, e.time_range.end, e.name) for e in trace.events() if e.device_type.name == 'CUDA'),
                   key=lambda sp: sp[0])
    device = defaultdict(float)
    critical = defaultdict(float)
    count = defaultdict(int)
    by_kernel = defaultdict(float)
    by_kernel_critical = defaultdict(float)
    frontier = None                         # latest end among the kernels seen so far (microseconds)
    for t0, t1, name in spans:
        cls, key = classify(name), _short(name)
        dur = (t1 - t0) / 1000.0
        device[cls] += dur
        count[cls] += 1
        by_kernel[key] += dur
        gain = (t1 - max(t0, frontier)) / 1000.0 if frontier is not None else dur
        if gain > 0:
            critical[cls] += gain
            by_kernel_critical[key] += gain
        frontier = t1 if frontier is None else max(frontier, t1)

    def ranked(d, n=None):
        items = sorted(d.items(), key=lambda kv: kv[1], reverse=True)[:n]
        return {k: round(v, 3) for k, v in items}
    busy = sum(critical.values())
    return dict(replay_ms=replay_ms, kernel_ms=sum(device.values()), idle_ms=max(replay_ms - busy, 0.0), launches=len(spans),
                device_ms_by_class=ranked(device), critical_ms_by_class=ranked(critical), launches_by_class=dict(count),
                heaviest=list(ranked(by_kernel, 12).items()), heaviest_critical=list(ranked(by_kernel_critical, 16).items()))


# ----------------------------------------------------------------------------------------------- profiling cases
# Small, seeded invocations of one kernel each, for a profiler to capture (nothing is timed or checked here):
#   python -m yanlongvla_b200.profile gemv [--n 4096] [--k 4096] [--tokens 1] [--launches 4]
#   python -m yanlongvla_b200.profile gemm [--m 4096] [--k 2048] [--n 8192] [--out i32|bf16] [--launches 4]
#   python -m yanlongvla_b200.profile pre|rotate [--m 4096] [--k 4096] [--launches 4]
#   python -m yanlongvla_b200.profile chain [--m 17] [--k 1536] [--launches 6]
#   python -m yanlongvla_b200.profile gemv_tc [--n 1536] [--k 1536] [--tokens 17] [--launches 4]
#   python -m yanlongvla_b200.profile policy [--tokens 1]    (replay_breakdown of one chunk-graph replay, as JSON)
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
    """replay_breakdown of one CUDA-graph replay of the fly policy's action chunk for `batch` observations."""
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
    print(json.dumps(replay_breakdown(g), indent=1))


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
