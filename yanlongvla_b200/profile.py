"""Kernel-class breakdown of one CUDA-graph replay (the reference's runner.kernel_classes, runner.py:227-266).

A torch.profiler (CUPTI) trace of a single replay; device time per kernel class, launch counts, wall time and the
gaps between kernels. Classes are matched by regex on the kernel name, first match wins.
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
    for e in prof.events():
        if e.device_type.name != 'CUDA':
            continue
        dur = e.time_range.elapsed_us() / 1000
        cls = next(c for c, pat in CLASSES if re.search(pat, e.name))
        by[cls] += dur
        launches[cls] += 1
        top[e.name[:90]] += dur
    total = sum(by.values())
    return dict(wall_ms=wall, kernel_ms=total, gaps_ms=max(wall - total, 0.0), launches=sum(launches.values()),
                by_class_ms={k: round(v, 3) for k, v in sorted(by.items(), key=lambda kv: -kv[1])},
                launches_by_class=dict(launches), top=[(nm, round(d, 3)) for nm, d in top.most_common(12)])
