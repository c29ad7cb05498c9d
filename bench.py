"""Benchmark of the fused 2-bit trellis decode-GEMV (the benchmark metric) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--layers L]

Workload (benchmark config 1 at its own shape): L = 64 distinct 4096 x 4096 trellis-coded layers (2 bits / weight,
L = 16 bitshift trellis, 16 x 16 tiles, 512 x 2 table, seeded synthetic streams) -> 256 MiB of 2-bit stream per step,
twice the 126 MB L2, so every step streams the weights from HBM (no L2 flush needed). One step = the decode-GEMV of
every layer on its own token (M = 1), one launch per layer, captured in one CUDA graph with programmatic dependent
launch edges. value = algorithmic bytes of all layers / step time (GB/s); roofline against the measured HBM copy
bandwidth of MEASURED_PEAKS.json.

e2e: the same layers through the public operator API (pre -> gemm_tcq -> post, i.e. the whole quantized Linear) with
the step's FP16 inputs copied from pinned host memory and the BF16 outputs copied back inside the timed region.

--impl reference: the reference's CPU path of the same metric: the reference's operator sequence in PyTorch CPU ops
(`definition`: trellis decode + the whole quantized Linear with the float64 exact INT8 product) on a bounded sample
of the layers, all host threads.

Multi-GPU (torchrun): every rank streams its own L layers (weak scaling, no collective on the data path); time = max
over ranks of the device-timed region.

Sub-objects of the line (each device-timed with CUDA events, its own roofline against MEASURED_PEAKS.json):
  rotation  config 2: the rotation op over T in {1, 64, 512, 4096} x D in {1024 ... 16384}, forward and inverse
  gemm      config 3: the W8A8 GEMM with scale epilogue over M in {1 ... 4096} x four (K, N), beside cuBLASLt
            (torch._int_mm) on the same operands
  policy    configs 4 / 5: the GR00T-style quantized policy (random-init weights, seeded synthetic observations): the
            B = 1 action-chunk latency on one GPU, and actions/s of the whole box for every total batch
            B in {1, 8, 32, 128, 512} split over the N GPUs (one CUDA-graph replay of the chunk, then one NCCL
            all-gather of the action chunks to rank 0), max over ranks; its cpu_baseline is the same policy in
            PyTorch CPU ops at B = 1.
The grids run in the N = 1 run only; the CPU baselines on rank 0 at N = 1 only.
"""
import argparse
import json
import os
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
M_N = 4096                      # config 1: W is 4096 x 4096
TOKENS = 1


# dram__bytes_read.sum + dram__bytes_write.sum of one k_gemm_tcq<1, 1> launch on a 4096 x 4096 layer, M = 1, from
# one ncu --set full capture of that launch (cold cache; the algorithmic bytes are 4,232,196).
NCU_TRAFFIC_BYTES = 4244992


def layer_bytes(m, n, M):
    """Algorithmic HBM bytes of one decode-GEMV launch: 2-bit stream m*n/4 + INT8 table 1024 + row scales 4m +
    INT8 activations M*n + token scales 4M + FP32 outputs 4*M*m."""
    return m * n // 4 + 1024 + 4 * m + M * n + 4 * M + 4 * M * m


def peaks():
    p = ROOT / 'MEASURED_PEAKS.json'
    if p.exists():
        d = json.loads(p.read_text())
        return float(d['hbm_gbs']), 'measured'
    return 6650.0, 'fallback'


# ------------------------------------------------------------------------------------------------ clocks
class Clocks:
    """nvidia-smi samples of the SM clock and throttle reasons during the timed region."""
    FIELDS = 'clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,' \
             'clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap'
    NAMES = ['hw_slowdown', 'hw_thermal_slowdown', 'sw_thermal_slowdown', 'sw_power_cap']

    def __init__(self, gpu):
        self.gpu, self.proc, self.lines = gpu, None, []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(['nvidia-smi', '-i', str(self.gpu), f'--query-gpu={self.FIELDS}', '--format=csv,noheader,nounits',
                                          '-lms', '100'], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except (OSError, FileNotFoundError):
            self.proc = None
        time.sleep(0.25)
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc is not None:
            time.sleep(0.15)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], [], set()
        for line in self.lines:
            f = [x.strip() for x in line.split(',')]
            if len(f) < 7:
                continue
            try:
                sm.append(float(f[0]))
                mx.append(float(f[1]))
            except ValueError:
                continue
            for name, v in zip(self.NAMES, f[3:7]):
                if v.lower().startswith('active'):
                    reasons.add(name)
        if not sm:
            return {'sm_mhz': None, 'sm_max_mhz': None, 'reasons': [], 'samples': 0}
        return {'sm_mhz': float(np.median(sm)), 'sm_max_mhz': float(max(mx)), 'reasons': sorted(reasons), 'samples': len(sm)}


# ------------------------------------------------------------------------------------------------ our arm
def make_layers(torch, L, seed, dev):
    """L seeded synthetic 4096 x 4096 layers on the device: uniform 2-bit streams, FP16-rounded N(0, 0.968^2) tables
    snapped to INT8 (tcq_format.py:74-77), row scales, signs. Streams are generated on the device (256 MiB)."""
    from yanlongvla_b200.tcq_format import snap
    g = torch.Generator(device=dev).manual_seed(seed)
    layers = []
    for i in range(L):
        bits = torch.randint(-32768, 32768, ((M_N // 16) * (M_N // 16), 32), dtype=torch.int32, device=dev, generator=g).to(torch.int16)
        tlut = (torch.randn(512, 2, device=dev, generator=g) * 0.968).half()
        row_scale = (torch.rand(M_N, device=dev, generator=g) * 0.025 + 0.005).half()
        t8, rs, _ = snap(tlut, row_scale)
        su = (torch.randint(0, 2, (M_N,), device=dev, generator=g) * 2 - 1).to(torch.int8)
        sv = (torch.randint(0, 2, (M_N,), device=dev, generator=g) * 2 - 1).to(torch.int8)
        layers.append(dict(bits=bits, t8=t8.contiguous(), rs=rs.contiguous(), su=su, sv=sv))
    return layers


def run_ours(args, rank, world, dist):
    import torch
    from yanlongvla_b200 import kernels as K
    dev = torch.device('cuda', int(os.environ.get('LOCAL_RANK', 0)))
    torch.cuda.set_device(dev)
    L = args.layers
    layers = make_layers(torch, L, 1000 + rank, dev)
    M = TOKENS
    g = torch.Generator(device=dev).manual_seed(7 + rank)
    x = torch.randn(L, M, M_N, device=dev, generator=g).half()
    q4 = torch.empty(L, M_N // 4, M, dtype=torch.int32, device=dev)
    s = torch.empty(L, M, dtype=torch.float32, device=dev)
    z = torch.empty(L, M, M_N, dtype=torch.float32, device=dev)
    y = torch.empty(L, M, M_N, dtype=torch.bfloat16, device=dev)
    for i, Ly in enumerate(layers):
        K.pre(x[i], Ly['su'], q4=q4[i], scale=s[i])
    torch.cuda.synchronize()

    def gemv_step():
        for i, Ly in enumerate(layers):
            K.gemm_tcq(Ly['bits'], Ly['t8'], q4[i], s[i], Ly['rs'], z[i], M_N)

    def linear_step():
        for i, Ly in enumerate(layers):
            K.gemm_tcq_x(Ly['bits'], Ly['t8'], x[i], Ly['su'], Ly['rs'], z[i], M_N)      # pre fused into the GEMV
            K.post(z[i], None, None, Ly['sv'], None, y[i])

    stream = torch.cuda.Stream(device=dev)
    graphs = {}
    with torch.cuda.stream(stream):
        for name, fn in (('gemv', gemv_step), ('linear', linear_step)):
            fn()
            torch.cuda.synchronize()
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr, stream=stream):
                fn()
            graphs[name] = gr
    torch.cuda.synchronize()

    def barrier():
        if dist is not None:
            dist.barrier()

    def timed(fn, steps, warmup):
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            e0.record(stream)
            for _ in range(steps):
                fn()
            e1.record(stream)
        e1.synchronize()
        barrier()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1)
        if dist is not None:
            t = torch.tensor([ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    with Clocks(dev.index) as clk:
        ms = timed(lambda: graphs['gemv'].replay(), args.steps, args.warmup)
    clocks = clk.summary()
    per_layer = layer_bytes(M_N, M_N, M)
    step_ms = ms / args.steps
    gbs_rank = per_layer * L / (step_ms * 1e-3) / 1e9
    value = gbs_rank * world                         # weak scaling: every rank streams its own L layers

    # e2e: whole quantized Linear through the operator API, FP16 inputs from pinned host memory, BF16 outputs back
    xh = torch.randn(L, M, M_N, generator=torch.Generator().manual_seed(3 + rank)).half().pin_memory()
    yh = torch.empty(L, M, M_N, dtype=torch.bfloat16).pin_memory()

    def e2e_step():
        with torch.cuda.stream(stream):
            x.copy_(xh, non_blocking=True)
            graphs['linear'].replay()
            yh.copy_(y, non_blocking=True)

    e2e_ms = timed(e2e_step, args.steps, args.warmup) / args.steps
    e2e_gbs = per_layer * L / (e2e_ms * 1e-3) / 1e9 * world

    # correctness spot check of one layer against the oracle is the test suite's job; here only finite outputs
    assert torch.isfinite(z).all().item()
    peak, peak_kind = peaks()
    achieved = per_layer / (step_ms / L * 1e-3) / 1e9
    out = dict(
        metric='fused 2-bit decode-GEMV HBM GB/s', value=round(value, 1), unit='GB/s', n_gpus=world, steps=args.steps,
        warmup=args.warmup, ms_per_step=round(step_ms, 4), higher_is_better=True, scaling='weak', vs_baseline=None,
        dtype='int8 x int8 -> int32 (2-bit trellis weights)', data='synthetic (seeded trellis streams, N(0,1) activations)',
        config=dict(workload='config1: 4096x4096 2-bit trellis decode-GEMV, M=1, %d distinct layers per step per GPU' % L,
                    layers_per_gpu=L, m=M_N, n=M_N, tokens=M, bytes_per_layer=per_layer,
                    l2='inputs larger than L2 (%.0f MiB of 2-bit stream per step per GPU)' % (L * M_N * M_N / 4 / 2 ** 20),
                    launch='one CUDA graph per step, one launch per layer, programmatic dependent launch',
                    parallelism='dp%d (independent layers per GPU, no collective)' % world),
        roofline=dict(bound='hbm', achieved=round(achieved, 1), peak=peak, unit='GB/s', frac=round(achieved / peak, 4),
                      traffic=NCU_TRAFFIC_BYTES, peak_kind=peak_kind,
                      note='achieved = bytes_per_layer / (graph step time / layers); includes inter-launch gaps. '
                           'traffic: DRAM bytes read + written by one launch of this kernel at this shape '
                           '(one ncu --set full capture of this kernel at this shape)'),
        e2e=dict(value=round(e2e_gbs, 1), unit='GB/s', h2d_bytes_per_step=int(xh.numel() * 2), d2h_bytes_per_step=int(yh.numel() * 2),
                 ms_per_step=round(e2e_ms, 4), path='kernels.gemm_tcq_x (pre fused into the decode-GEMV) -> post per layer (whole quantized Linear)'),
        gpu_launches=args.steps * L,
        clocks=clocks,
        single_layer_us=round(step_ms / L * 1e3, 3),
    )
    return out


# ------------------------------------------------------------------------------------------------ kernel grids (configs 2, 3)
L2_BYTES = 126 * 2 ** 20


def _ring(bytes_per_launch, cap=64):
    """Launches per timed graph so that the ring of distinct buffers spans at least twice the L2 (at most `cap`)."""
    return max(1, min(cap, -(-2 * L2_BYTES // max(bytes_per_launch, 1))))


def _graph_time(torch, stream, fns, reps, flush):
    """Median over `reps` of the device time of one CUDA-graph replay of `fns` (called in order), each replay after an
    L2 flush (a write of `flush`, twice the L2). Returns ms per replay."""
    with torch.cuda.stream(stream):
        for f in fns:
            f()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        for f in fns:
            f()
    ts = []
    for r in range(reps + 2):
        with torch.cuda.stream(stream):
            flush.fill_(r)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            g.replay()
            e1.record(stream)
        e1.synchronize()
        if r >= 2:                                     # two untimed warm-up replays
            ts.append(e0.elapsed_time(e1))
    del g
    return float(np.median(ts))


def run_rotation_grid(args, dev):
    """Config 2: the rotation op y = fwht(x * s) (forward) and x = fwht(y) * s (inverse), BF16 in and out, for every
    T x D of the grid; each timed graph cycles through distinct buffers spanning twice the L2 and starts after an L2
    flush. Bytes per launch = 2 T D (read) + 2 T D (write) + D (signs)."""
    import torch
    from yanlongvla_b200 import kernels as K
    peak, kind = peaks()
    stream = torch.cuda.Stream(device=dev)
    flush = torch.empty(2 * L2_BYTES // 4, dtype=torch.int32, device=dev)
    g = torch.Generator(device=dev).manual_seed(2)
    rows, launches = [], 0
    for D in (1024, 2048, 4096, 8192, 16384):
        sg = (torch.randint(0, 2, (D,), device=dev, generator=g) * 2 - 1).to(torch.int8)
        for T in (1, 64, 512, 4096):
            nbytes = 4 * T * D + D
            R = _ring(nbytes)
            xs = [torch.randn(T, D, device=dev, generator=g).bfloat16() for _ in range(R)]
            ys = [torch.empty(T, D, dtype=torch.bfloat16, device=dev) for _ in range(R)]
            fwd = _graph_time(torch, stream, [lambda i=i: K.rotate(xs[i], sg, out_dtype=torch.bfloat16, out=ys[i]) for i in range(R)],
                              args.grid_reps, flush) / R
            inv = _graph_time(torch, stream, [lambda i=i: K.rotate(ys[i], sg, inverse=True, out_dtype=torch.bfloat16, out=xs[i])
                                              for i in range(R)], args.grid_reps, flush) / R
            launches += 2 * R * (args.grid_reps + 3)
            gbs = nbytes / (fwd * 1e-3) / 1e9
            rows.append(dict(T=T, D=D, fwd_us=round(fwd * 1e3, 2), inv_us=round(inv * 1e3, 2), fwd_gbs=round(gbs, 1),
                             frac=round(gbs / peak, 4), ring=R))
            del xs, ys
    torch.cuda.empty_cache()
    big = [r for r in rows if r['T'] == 4096 and r['D'] == 4096][0]
    return dict(op='kernels.rotate BF16 -> BF16 (forward and inverse)', peak_gbs=peak, peak_kind=kind, launches=launches,
                headline=dict(T=4096, D=4096, fwd_gbs=big['fwd_gbs'], frac=big['frac']),
                timing='CUDA-graph replay of a ring of distinct buffers spanning 2x L2, after an L2 flush; per-launch time',
                rows=rows)


def run_gemm_grid(args, dev):
    """Config 3: W8A8 GEMM with the per-token x per-channel scale epilogue, BF16 out (kernels.int8_gemm), for every
    M x (K, N) of the grid, beside the plain INT32 product (kernels.int_mm) and cuBLASLt's torch._int_mm on the same
    operands (token rows zero-padded to 32 below 32, as the reference's int_matmul does). Operands: INT8 activations
    quantized per token from N(0, 1) BF16 with 1 % outliers x 20, INT8 weights uniform in [-127, 127], channel scales
    U(1e-3, 1e-2). Each timed graph cycles through operand sets spanning twice the L2 (at most 16) after an L2 flush."""
    import torch
    from yanlongvla_b200 import kernels as K
    pk = json.loads((ROOT / 'MEASURED_PEAKS.json').read_text()) if (ROOT / 'MEASURED_PEAKS.json').exists() else {}
    int8_peak = 2.0 * float(pk.get('bf16_tflops', 1590.0))
    stream = torch.cuda.Stream(device=dev)
    flush = torch.empty(2 * L2_BYTES // 4, dtype=torch.int32, device=dev)
    g = torch.Generator(device=dev).manual_seed(3)
    rows, launches = [], 0
    for Kd, N in ((2048, 2048), (2048, 6144), (2048, 8192), (8192, 2048)):
        for M in (1, 16, 64, 256, 1024, 4096):
            nbytes = M * Kd + N * Kd + 2 * M * N
            R = _ring(nbytes, cap=16)
            sets = []
            for _ in range(R):
                a = torch.randn(M, Kd, device=dev, generator=g)
                a = torch.where(torch.rand(M, Kd, device=dev, generator=g) < 0.01, a * 20, a).bfloat16()
                q, s = K.quantize(a)
                w = torch.randint(-127, 128, (N, Kd), dtype=torch.int8, device=dev, generator=g)
                sc = torch.rand(N, device=dev, generator=g) * 9e-3 + 1e-3
                qp = torch.cat((q, q.new_zeros(32 - M, Kd))) if M < 32 else q
                sets.append(dict(q=q, s=s, w=w, sc=sc, qp=qp, out=torch.empty(M, N, dtype=torch.bfloat16, device=dev),
                                 acc=torch.empty(M, N, dtype=torch.int32, device=dev)))
            ours = _graph_time(torch, stream, [lambda d=d: K.int8_gemm(d['q'], d['w'], d['s'], d['sc'], out=d['out']) for d in sets],
                               args.grid_reps, flush) / R
            ours32 = _graph_time(torch, stream, [lambda d=d: K.int_mm(d['q'], d['w'], out=d['acc']) for d in sets],
                                 args.grid_reps, flush) / R
            cublas = _graph_time(torch, stream, [lambda d=d: torch._int_mm(d['qp'], d['w'].t()) for d in sets],
                                 args.grid_reps, flush) / R
            launches += 2 * R * (args.grid_reps + 3)
            tops = 2.0 * M * N * Kd / (ours * 1e-3) / 1e12
            rows.append(dict(M=M, K=Kd, N=N, bf16_out_us=round(ours * 1e3, 2), int32_out_us=round(ours32 * 1e3, 2),
                             cublaslt_int_mm_us=round(cublas * 1e3, 2), tops=round(tops, 1), frac=round(tops / int8_peak, 4),
                             vs_cublaslt=round(cublas / ours, 3), ring=R))
            del sets
    torch.cuda.empty_cache()
    big = [r for r in rows if r['M'] >= 1024]
    return dict(op='kernels.int8_gemm (tcgen05 kind::i8, BF16 out with scale epilogue); kernels.int_mm (INT32 out); '
                   'torch._int_mm (cuBLASLt, INT32 out)',
                int8_peak_tops=int8_peak, int8_peak_kind='2 x measured bf16_tflops (dense INT8 = 2 x dense BF16 on B200)',
                launches=launches, timing='CUDA-graph replay of a ring of operand sets spanning 2x L2 (<= 16), after an L2 flush',
                m_ge_1024_beats_cublaslt=sum(r['vs_cublaslt'] >= 1.0 for r in big), m_ge_1024_shapes=len(big), rows=rows)


# ------------------------------------------------------------------------------------------------ policy (configs 4, 5)
POLICY_BATCHES = (1, 8, 32, 128, 512)


def run_policy(args, rank, world, dist):
    """Config 4 (B = 1 action-chunk latency on one GPU) and config 5 (actions/s of the whole box for every total batch
    B of the config, split over the N ranks: strong scaling at fixed B), one CUDA-graph replay per chunk, then one
    NCCL all-gather of the action chunks to rank 0; device-timed, max over ranks. e2e: the same with the observations
    copied from pinned host memory and the actions copied back, inside the timed region."""
    import torch
    from yanlongvla_b200 import dp, modules, policy as P
    dev = torch.device('cuda', int(os.environ.get('LOCAL_RANK', 0)))
    c = P.PolicyConfig()
    model, _, info = P.build_policy(dev, args.policy_runtime, c, seed=0)
    stream = torch.cuda.Stream(device=dev)

    def forward():
        if args.policy_runtime == 'hybrid':
            modules.decode_chunk(model)
        return model(*obs_now[0])

    obs_now = [None]

    def capture(B, seed):
        obs_now[0] = P.synthetic_observations(B, c, dev, seed=seed)
        with torch.no_grad(), torch.cuda.stream(stream):
            for _ in range(2):
                out = forward()
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                out = forward()
        torch.cuda.synchronize()
        return g, obs_now[0], out

    def time_steps(fn, steps, warmup):
        with torch.cuda.stream(stream):
            for _ in range(warmup):
                fn()
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()
        ts = []
        for _ in range(steps):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            with torch.cuda.stream(stream):             # the replay, the copies and the gather all run on `stream`
                e0.record(stream)
                fn()
                e1.record(stream)
            e1.synchronize()
            ts.append(e0.elapsed_time(e1))
        ts = torch.tensor(ts, device=dev)
        if dist is not None:
            dist.all_reduce(ts, op=dist.ReduceOp.MAX)
        ts = ts.cpu().tolist()
        return float(np.median(ts)), float(np.percentile(ts, 95))

    out = dict(runtime=args.policy_runtime, quantized_layers=dict(w2a8=info['layers'], w8a8=c.vit_layers * 6),
               groups=info['groups'], fused_mlps=info['fused_mlps'])
    # config 4: one observation, one GPU (every rank measures its own; max over ranks)
    g1, _, _ = capture(1, 100 + rank)
    out['chunk_ms_b1'], out['chunk_p95_ms_b1'] = time_steps(lambda: g1.replay(), args.policy_steps, 3)
    del g1
    torch.cuda.empty_cache()
    # config 5: every total batch B, split over the ranks; ranks without observations gather an empty slice
    points = []
    for B in POLICY_BATCHES:
        b0, b1 = dp.shard(B, world, rank)
        if b1 > b0:
            g, obs, acts = capture(b1 - b0, 200 + 7 * B + rank)
        else:
            g, obs, acts = None, (), torch.zeros(0, c.chunk, c.action_dim, device=dev)
        est = torch.tensor([0.0], device=dev)
        if g is not None:                               # steps sized to ~2 s of timed work per point
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            with torch.cuda.stream(stream):
                e0.record(stream)
                g.replay()
                e1.record(stream)
            e1.synchronize()
            est[0] = e0.elapsed_time(e1)
        if dist is not None:
            dist.all_reduce(est, op=dist.ReduceOp.MAX)
        steps = int(max(3, min(args.policy_steps, 2000.0 / max(float(est[0]), 1e-3))))

        def dp_step():
            if g is not None:
                g.replay()
            with torch.cuda.stream(stream):
                if dist is not None:
                    dp.gather_actions(acts, B)

        med, p95 = time_steps(dp_step, steps, 3)
        host = [t.cpu().pin_memory() for t in obs]
        act_host = torch.empty(acts.shape, dtype=acts.dtype).pin_memory()

        def e2e_step():
            with torch.cuda.stream(stream):
                for d, h in zip(obs, host):
                    d.copy_(h, non_blocking=True)
            if g is not None:
                g.replay()
            with torch.cuda.stream(stream):
                if dist is not None:
                    dp.gather_actions(acts, B)
                act_host.copy_(acts, non_blocking=True)

        med_e, _ = time_steps(e2e_step, steps, 3)
        points.append(dict(batch=B, batch_per_gpu_max=dp.max_shard(B, world), chunk_ms=round(med, 4), chunk_p95_ms=round(p95, 4),
                           actions_per_s=round(B * c.chunk / (med * 1e-3), 1), steps=steps,
                           e2e=dict(chunk_ms=round(med_e, 4), actions_per_s=round(B * c.chunk / (med_e * 1e-3), 1),
                                    h2d_bytes_per_step=int(sum(h.numel() * h.element_size() for h in host)),
                                    d2h_bytes_per_step=int(act_host.numel() * act_host.element_size())),
                           finite=bool(torch.isfinite(acts).all().item())))
        del g, obs, acts, host, act_host
        torch.cuda.empty_cache()
    out['dp'] = dict(scaling='strong (total batch B fixed, split over the GPUs)', points=points,
                     gather='nccl all_gather_into_tensor of the (B/N, 16, 32) FP32 chunks' if dist is not None else 'none (1 GPU)')
    return {k: (round(v, 4) if isinstance(v, float) else v) for k, v in out.items()}


def policy_cpu_baseline(dev, min_seconds=8.0):
    """Config 4 on the host: the same synthetic policy (seed 0) in the 'reference' runtime on the CPU, B = 1: every
    quantized Linear is the W2A8 / W8A8 definition in PyTorch CPU ops (float64 exact INT8 products, as the reference's
    int_matmul on the CPU, tcq_format.py:110-116) with resident INT8 weights (decoded once on the GPU before timing, as
    the reference's RefLinear holds them), attention and norms in PyTorch CPU ops, all host threads. One warm-up
    chunk, then chunks until `min_seconds` of timed work (at least one)."""
    import torch
    from yanlongvla_b200 import policy as P
    from yanlongvla_b200.tcq_format import Layer
    torch.set_num_threads(os.cpu_count())
    c = P.PolicyConfig()
    ref_gpu, layers, _ = P.build_policy(dev, 'reference', c, seed=0)
    w8 = {name: m.w8.cpu() for name, m in ref_gpu.named_modules() if hasattr(m, 'w8') and name in layers}
    del ref_gpu
    cpu_layers = {name: Layer(name, dict(bits=L.bits.cpu(), tlut=L.tlut.cpu(), row_scale=L.row_scale.cpu(), su=L.su.cpu(),
                                         sv=L.sv.cpu()), bias=None if L.bias is None else L.bias.cpu(), device='cpu')
                  for name, L in layers.items()}
    del layers
    torch.cuda.empty_cache()
    model, _, _ = P.build_policy('cpu', 'reference', c, seed=0, layers=cpu_layers, ref_w8=w8)
    obs = P.synthetic_observations(1, c, device='cpu', seed=100)
    ts = []
    with torch.no_grad():
        model(*obs)
        while not ts or sum(ts) < min_seconds:
            t0 = time.perf_counter()
            a = model(*obs)
            ts.append(time.perf_counter() - t0)
    return dict(chunk_ms=round(float(np.median(ts)) * 1e3, 1), actions_per_s=round(c.chunk / float(np.median(ts)), 2),
                cores=torch.get_num_threads(), kind='port', chunks_timed=len(ts), finite=bool(torch.isfinite(a).all()),
                sample='one B = 1 action chunk per timed run (config 4, full depth), after one warm-up chunk; PyTorch CPU ops '
                       'of the definition, INT8 weights resident')


# ------------------------------------------------------------------------------------------------ CPU reference arm
def cpu_reference(sample_layers, min_seconds=0.0, max_layers=64):
    """The reference's CPU path of the metric on config-1 layers: the package's PyTorch-ops restatement of
    tcq_format.py (`definition.decode_w8` + `definition.linear`: windowed trellis read, hash decode, rotation,
    quantizer, float64 exact INT8 product, scale epilogue, rotation) on the CPU, all host threads; the same operator
    sequence as the reference's Layer.w8_reference() + reference_linear (measured at 0.95x the reference's own time on
    the same cores, same outputs, by oracle/calibrate_cpu.py). `sample_layers` layers, or more (up to `max_layers`)
    until the timed layers took `min_seconds`; the first layer is a warm-up. Returns (GB/s, seconds, timed layers)."""
    import torch
    from yanlongvla_b200 import definition as D
    from yanlongvla_b200.tcq_format import snap
    torch.set_num_threads(os.cpu_count())
    g = torch.Generator().manual_seed(0)
    per = layer_bytes(M_N, M_N, TOKENS)
    elapsed, n, i = 0.0, 0, 0

    class _L:
        pass
    while i < sample_layers or (elapsed < min_seconds and i < max_layers):
        L = _L()
        L.m = L.n = M_N
        L.bits = torch.randint(-32768, 32768, ((M_N // 16) ** 2, 32), dtype=torch.int32, generator=g).to(torch.int16)
        L.t8, L.rs, _ = snap((torch.randn(512, 2, generator=g) * 0.968).half(), (torch.rand(M_N, generator=g) * 0.025 + 0.005).half())
        L.su = (torch.randint(0, 2, (M_N,), generator=g) * 2 - 1).to(torch.int8)
        L.sv = (torch.randint(0, 2, (M_N,), generator=g) * 2 - 1).to(torch.int8)
        L.bias = None
        x = torch.randn(TOKENS, M_N, generator=g).half()
        t0 = time.perf_counter()                       # one layer: decode + the whole quantized Linear
        D.linear(x, L, D.decode_w8(L.bits, L.t8, M_N, M_N))
        d = time.perf_counter() - t0
        if i > 0:
            elapsed += d
            n += 1
        i += 1
    n = max(n, 1)
    dt = max(elapsed, 1e-9)
    return per * n / dt / 1e9, dt, n


def run_reference(args, rank, world):
    if rank != 0:
        return None
    threads = os.cpu_count()
    vals = []
    for _ in range(args.warmup):
        cpu_reference(2)
    secs = 0.0
    for _ in range(args.steps):
        v, dt, n = cpu_reference(args.ref_layers + 1)
        vals.append(v)
        secs += dt
    value = float(np.median(vals))
    return dict(
        impl='reference', metric='fused 2-bit decode-GEMV HBM GB/s', value=round(value, 6), unit='GB/s', n_gpus=world, steps=args.steps,
        warmup=args.warmup, ms_per_step=round(secs / args.steps * 1e3, 2), higher_is_better=True, scaling='weak', vs_baseline=None,
        dtype='int8 x int8 -> int32 (2-bit trellis weights)', data='synthetic (seeded trellis streams)',
        config=dict(workload='config1: 4096x4096 2-bit trellis decode-GEMV, M=1, 64 distinct layers per step per GPU '
                             '(CPU: a sample of %d layers per step)' % args.ref_layers, m=M_N, n=M_N, tokens=TOKENS),
        cpu_baseline=dict(value=round(value, 6), unit='GB/s', cores=threads, kind='port',
                          sample='%d config-1 layers per step: trellis decode + the whole quantized Linear, PyTorch CPU ops '
                                 '(the reference\'s operator sequence)' % args.ref_layers),
        e2e=dict(value=round(value, 6), unit='GB/s', h2d_bytes_per_step=0, d2h_bytes_per_step=0),
    )


def _claim_stdout():
    """The driver reads exactly one JSON line from stdout. Libraries print to file descriptor 1 on their own (NCCL's
    version banner at initialization, for one): point descriptor 1 at stderr and keep a private copy of the original
    stdout for the result line."""
    sys.stdout.flush()
    result = os.fdopen(os.dup(1), 'w')
    os.dup2(2, 1)
    return result


def main():
    out_file = _claim_stdout()
    ap = argparse.ArgumentParser()
    ap.add_argument('--gpus', type=int, default=1)
    ap.add_argument('--steps', type=int, default=50)
    ap.add_argument('--warmup', type=int, default=5)
    ap.add_argument('--impl', choices=['ours', 'reference'], default='ours')
    ap.add_argument('--layers', type=int, default=64)
    ap.add_argument('--ref-layers', type=int, default=2)
    ap.add_argument('--no-cpu-baseline', action='store_true')
    ap.add_argument('--no-policy', action='store_true')
    ap.add_argument('--no-grids', action='store_true', help='skip the config-2 rotation and config-3 GEMM grids')
    ap.add_argument('--grid-reps', type=int, default=5)
    ap.add_argument('--policy-runtime', default='fly', choices=['fly', 'resident', 'hybrid'])
    ap.add_argument('--policy-steps', type=int, default=20)
    args = ap.parse_args()
    world = int(os.environ.get('WORLD_SIZE', 1))
    rank = int(os.environ.get('RANK', 0))
    if args.impl == 'reference':
        out = run_reference(args, rank, world)
        if out is not None:
            print(json.dumps(out), file=out_file, flush=True)
        return
    import torch
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        local = int(os.environ.get('LOCAL_RANK', 0))
        torch.cuda.set_device(local)
        dist.init_process_group('nccl', timeout=datetime.timedelta(seconds=120), device_id=torch.device('cuda', local))
    out = run_ours(args, rank, world, dist)
    dev = torch.device('cuda', int(os.environ.get('LOCAL_RANK', 0)))
    if not args.no_grids and world == 1:               # single-GPU kernel grids: measured in the N = 1 run only
        out['rotation'] = run_rotation_grid(args, dev)
        out['gemm'] = run_gemm_grid(args, dev)
    if not args.no_policy:
        out['policy'] = run_policy(args, rank, world, dist)
    if rank == 0:
        if not args.no_cpu_baseline and world == 1:
            v, dt, nl = cpu_reference(args.ref_layers + 1, min_seconds=10.0)
            out['cpu_baseline'] = dict(value=round(v, 6), unit='GB/s', cores=os.cpu_count(), kind='port',
                                       sample='%d config-1 layers (trellis decode + the whole quantized Linear, PyTorch CPU ops), '
                                              '%.1f s' % (nl, dt))
            if not args.no_policy:
                out['policy']['cpu_baseline'] = policy_cpu_baseline(dev)
        print(json.dumps(out), file=out_file, flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == '__main__':
    main()
