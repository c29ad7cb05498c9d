"""Benchmark of the fused 2-bit trellis decode-GEMV (BASELINE metric) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--layers L]

Workload (BASELINE config 1 at its own shape): L = 64 distinct 4096 x 4096 trellis-coded layers (2 bits / weight,
L = 16 bitshift trellis, 16 x 16 tiles, 512 x 2 table, seeded synthetic streams) -> 256 MiB of 2-bit stream per step,
twice the 126 MB L2, so every step streams the weights from HBM (no L2 flush needed). One step = the decode-GEMV of
every layer on its own token (M = 1), one launch per layer, captured in one CUDA graph with programmatic dependent
launch edges. value = algorithmic bytes of all layers / step time (GB/s); roofline against the measured HBM copy
bandwidth of MEASURED_PEAKS.json.

e2e: the same layers through the public operator API (pre -> gemm_tcq -> post, i.e. the whole quantized Linear) with
the step's FP16 inputs copied from pinned host memory and the BF16 outputs copied back inside the timed region.

--impl reference: the reference's CPU path of the same metric (the numpy restatement under oracle/: trellis decode +
exact INT8 product + scale epilogue) on a bounded sample of the layers, all host threads.

Multi-GPU (torchrun): every rank streams its own L layers (weak scaling, no collective on the data path); time = max
over ranks of the device-timed region.

The `policy` field measures the GR00T-style quantized policy (BASELINE configs 4 and 5, random-init weights, seeded
synthetic observations): the action-chunk latency at batch 1 on one GPU, and actions/s of data-parallel replicas with
--policy-batch observations per GPU (one CUDA-graph replay of the whole chunk per step, then one NCCL all-gather of
the action chunks to rank 0), device-timed, max over ranks.
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
# the ncu capture summarized in profiles/gemm_tcq_m1_4096x4096.md (cold cache; the algorithmic bytes are 4,232,196).
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
                           '(ncu --set full capture, profiles/gemm_tcq_m1_4096x4096.md)'),
        e2e=dict(value=round(e2e_gbs, 1), unit='GB/s', h2d_bytes_per_step=int(xh.numel() * 2), d2h_bytes_per_step=int(yh.numel() * 2),
                 ms_per_step=round(e2e_ms, 4), path='kernels.gemm_tcq_x (pre fused into the decode-GEMV) -> post per layer (whole quantized Linear)'),
        gpu_launches=args.steps * L,
        clocks=clocks,
        single_layer_us=round(step_ms / L * 1e3, 3),
    )
    return out


# ------------------------------------------------------------------------------------------------ policy (configs 4, 5)
def run_policy(args, rank, world, dist):
    import torch
    from yanlongvla_b200 import dp, modules, policy as P
    dev = torch.device('cuda', int(os.environ.get('LOCAL_RANK', 0)))
    c = P.PolicyConfig()
    model, _, info = P.build_policy(dev, args.policy_runtime, c, seed=0)
    stream = torch.cuda.Stream(device=dev)

    def capture(B, seed):
        obs = P.synthetic_observations(B, c, dev, seed=seed)
        with torch.no_grad(), torch.cuda.stream(stream):
            for _ in range(2):
                if args.policy_runtime == 'hybrid':
                    modules.decode_chunk(model)
                out = model(*obs)
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                if args.policy_runtime == 'hybrid':
                    modules.decode_chunk(model)
                out = model(*obs)
        torch.cuda.synchronize()
        return g, obs, out

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
    # config 5: B = policy_batch * world observations, one shard per rank, one gather of the chunks to rank 0
    B = args.policy_batch * world
    b0, b1 = dp.shard(B, world, rank)
    g, obs, acts = capture(b1 - b0, 200 + rank)

    def dp_step():
        g.replay()
        with torch.cuda.stream(stream):
            if dist is not None:
                dp.gather_actions(acts, B)

    med, p95 = time_steps(dp_step, args.policy_steps, 3)
    out.update(batch=B, batch_per_gpu=b1 - b0, chunk_ms=med, chunk_p95_ms=p95, actions_per_s=B * c.chunk / (med * 1e-3),
               gather='nccl all_gather_into_tensor of the (B/N, 16, 32) FP32 chunks' if dist is not None else 'none (1 GPU)',
               finite=bool(torch.isfinite(acts).all().item()))
    # e2e: observations from pinned host memory, actions back to the host, all inside the timed region
    host = [t.cpu().pin_memory() for t in obs]
    act_host = torch.empty(acts.shape, dtype=acts.dtype).pin_memory()

    def e2e_step():
        with torch.cuda.stream(stream):
            for d, h in zip(obs, host):
                d.copy_(h, non_blocking=True)
        g.replay()
        with torch.cuda.stream(stream):
            if dist is not None:
                dp.gather_actions(acts, B)
            act_host.copy_(acts, non_blocking=True)

    med_e, _ = time_steps(e2e_step, args.policy_steps, 3)
    out['e2e'] = dict(chunk_ms=med_e, actions_per_s=B * c.chunk / (med_e * 1e-3),
                      h2d_bytes_per_step=int(sum(h.numel() * h.element_size() for h in host)),
                      d2h_bytes_per_step=int(act_host.numel() * act_host.element_size()))
    del g
    return {k: (round(v, 4) if isinstance(v, float) else v) for k, v in out.items()}


# ------------------------------------------------------------------------------------------------ CPU reference arm
def cpu_reference(sample_layers, threads, min_seconds=0.0, max_layers=64):
    """The reference's CPU path of the metric (numpy restatement of tcq_format.py: windowed trellis read, hash decode,
    exact INT8 product, scale epilogue) on `sample_layers` config-1 layers, or more (up to `max_layers`) until the
    timed layers have taken `min_seconds`. Returns (GB/s, seconds, timed layers)."""
    sys.path.insert(0, str(ROOT / 'oracle'))
    import tcq_oracle as O
    rng = np.random.default_rng(0)
    per = layer_bytes(M_N, M_N, TOKENS)
    elapsed, n, i = 0.0, 0, 0
    while i < sample_layers or (elapsed < min_seconds and i < max_layers):
        bits = rng.integers(0, 1 << 16, size=((M_N // 16) ** 2, 32), dtype=np.uint32).astype(np.uint16)
        tlut = (rng.standard_normal((512, 2)) * 0.968).astype(np.float16)
        rsc = rng.uniform(0.005, 0.03, M_N).astype(np.float16)
        sg = np.ones(M_N, dtype=np.int8)
        layer = O.Layer(bits, tlut, rsc, sg, sg)
        q = rng.integers(-127, 128, size=(TOKENS, M_N)).astype(np.int8)
        s = np.ones(TOKENS, dtype=np.float32)
        t0 = time.perf_counter()                       # only the layer's decode + product + epilogue is timed
        O.gemm_z(q, layer.w8_reference(), s, layer.rs)
        d = time.perf_counter() - t0
        if i > 0:                                      # the first layer is the warm-up
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
    os.environ.setdefault('OMP_NUM_THREADS', str(threads))
    vals = []
    for _ in range(args.warmup):
        cpu_reference(2, threads)
    secs = 0.0
    for _ in range(args.steps):
        v, dt, n = cpu_reference(args.ref_layers + 1, threads)
        vals.append(v)
        secs += dt
    value = float(np.median(vals))
    return dict(
        impl='reference', metric='fused 2-bit decode-GEMV HBM GB/s', value=round(value, 6), unit='GB/s', n_gpus=world, steps=args.steps,
        warmup=args.warmup, ms_per_step=round(secs / args.steps * 1e3, 2), higher_is_better=True, scaling='weak', vs_baseline=None,
        dtype='int8 x int8 -> int32 (2-bit trellis weights)', data='synthetic (seeded trellis streams)',
        config=dict(workload='config1: 4096x4096 2-bit trellis decode-GEMV, M=1 (CPU sample of %d layers per step)' % args.ref_layers,
                    m=M_N, n=M_N, tokens=TOKENS),
        cpu_baseline=dict(value=round(value, 6), unit='GB/s', cores=threads, kind='port',
                          sample='%d config-1 layers per step (decode + exact product + epilogue), numpy/BLAS' % args.ref_layers),
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
    ap.add_argument('--policy-runtime', default='fly', choices=['fly', 'resident', 'hybrid'])
    ap.add_argument('--policy-batch', type=int, default=16, help='observations per GPU for the data-parallel policy')
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
    if not args.no_policy:
        out['policy'] = run_policy(args, rank, world, dist)
    if rank == 0:
        if not args.no_cpu_baseline:
            v, dt, nl = cpu_reference(args.ref_layers + 1, os.cpu_count(), min_seconds=10.0)
            out['cpu_baseline'] = dict(value=round(v, 6), unit='GB/s', cores=os.cpu_count(), kind='port',
                                       sample='%d config-1 layers (decode + exact product + epilogue), %.1f s' % (nl, dt))
        print(json.dumps(out), file=out_file, flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == '__main__':
    main()
