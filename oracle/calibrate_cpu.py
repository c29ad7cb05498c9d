"""Calibration of the CPU baselines against the reference's own CPU code (run where a reference checkout exists; the
reference itself never travels with the repository).

    python oracle/calibrate_cpu.py path/to/reference/deploy/tcq_kernels [--repeats 5]

TEST INFRASTRUCTURE: it times, on this host's cores and the same seeded config-1 layer (4096 x 4096, 2-bit trellis,
M = 1 FP16 token), the work of one decode-GEMV step of the benchmark's CPU baseline:
  reference   the reference's tcq_format.py: Layer(device='cpu').w8_reference() + reference_linear(x, layer, w8=...)
              (deploy/tcq_kernels/tcq_format.py:80-148)
  definition  the package's PyTorch-ops restatement (yanlongvla_b200.definition: decode_w8 + linear), the benchmark's
              CPU baseline
  oracle      the numpy restatement (oracle/tcq_oracle.py: w8_reference + the exact product and epilogue)
and checks that all three give the same BF16 output. Prints one JSON line (median seconds of each, threads).
"""
import argparse
import importlib
import json
import os
import sys
import time
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
sys.path.insert(0, str(HERE.parent))
sys.path.insert(0, str(HERE.parent / 'tests' / 'golden'))


def median_time(fn, repeats):
    fn()                                                  # warm-up
    ts = []
    for _ in range(repeats):
        t0 = time.perf_counter()
        out = fn()
        ts.append(time.perf_counter() - t0)
    return float(np.median(ts)), out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument('ref_root', nargs='?', default=os.environ.get('TCQ_REF_ROOT'))
    ap.add_argument('--repeats', type=int, default=5)
    a = ap.parse_args()
    if not a.ref_root:
        raise SystemExit('calibrate_cpu.py: give the reference directory deploy/tcq_kernels (argument or TCQ_REF_ROOT)')
    sys.dont_write_bytecode = True
    sys.path.insert(0, a.ref_root)
    F = importlib.import_module('tcq_format')
    import cases
    import tcq_oracle as O
    from yanlongvla_b200 import definition as D
    torch.set_num_threads(os.cpu_count())
    m = n = 4096
    t, _ = cases.layer_tensors('config1', m, n)
    tens = dict(bits=torch.from_numpy(t['bits'].view(np.int16).copy()), tlut=torch.from_numpy(t['tlut']),
                row_scale=torch.from_numpy(t['row_scale']), su=torch.from_numpy(t['su']), sv=torch.from_numpy(t['sv']))
    x = cases.activations('config1', 1, n, 'f16')
    xt = torch.from_numpy(x)
    RL = F.Layer('config1', tens, device='cpu')
    OL = O.Layer(t['bits'], t['tlut'], t['row_scale'], t['su'], t['sv'])

    def ref_step():
        return F.reference_linear(xt, RL, w8=RL.w8_reference())

    def def_step():
        return D.linear(xt, RL, D.decode_w8(RL.bits, RL.t8, m, n))

    def oracle_step():
        return O.reference_linear(x, 'f16', OL, w8=OL.w8_reference())

    t_ref, y_ref = median_time(ref_step, a.repeats)
    t_def, y_def = median_time(def_step, a.repeats)
    t_orc, y_orc = median_time(oracle_step, a.repeats)
    yr = y_ref.view(torch.int16).numpy().view(np.uint16)
    same = bool(np.array_equal(yr, y_def.view(torch.int16).numpy().view(np.uint16)) and np.array_equal(yr, y_orc))
    print(json.dumps(dict(workload='config1 4096x4096, M=1: decode + reference_linear', threads=torch.get_num_threads(),
                          cpu=os.cpu_count(), reference_s=round(t_ref, 4), definition_s=round(t_def, 4), oracle_s=round(t_orc, 4),
                          definition_over_reference=round(t_def / t_ref, 3), oracle_over_reference=round(t_orc / t_ref, 3),
                          identical_outputs=same, repeats=a.repeats)))


if __name__ == '__main__':
    main()
