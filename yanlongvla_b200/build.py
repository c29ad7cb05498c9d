"""Build the C-ABI library libtcq_b200.so in-tree with nvcc for sm_100a (no GPU needed).

    python -m yanlongvla_b200.build [--force] [--verbose]

Every .cu under csrc/ is compiled to an object with
    nvcc -gencode arch=compute_100a,code=sm_100a -lineinfo -O3 -std=c++17 -fmad=false -Xcompiler -fPIC
(-fmad=false: no FMA contraction, the FP32 arithmetic must match the reference definition bit for bit) and linked into
yanlongvla_b200/libtcq_b200.so. Objects are rebuilt only when a source or header is newer.
"""
import argparse
import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / 'csrc'
OBJ = PKG / '_build'
LIB = PKG / 'libtcq_b200.so'
NVCC = os.environ.get('NVCC', 'nvcc')
ARCH = ['-gencode', 'arch=compute_100a,code=sm_100a']
FLAGS = ['-lineinfo', '-O3', '-std=c++17', '-fmad=false', '-Xcompiler', '-fPIC', '--expt-relaxed-constexpr',
         f'-I{ROOT / "include"}', f'-I{CSRC}']


def _headers():
    return list(CSRC.glob('*.cuh')) + list((ROOT / 'include').glob('*.h'))


def _compile(src, verbose=False, extra=()):
    obj = OBJ / (src.stem + '.o')
    newest = max(p.stat().st_mtime for p in [src] + _headers())
    if obj.exists() and obj.stat().st_mtime >= newest:
        return obj, None
    cmd = [NVCC, *ARCH, *FLAGS, *extra, '-c', str(src), '-o', str(obj)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if verbose or r.returncode:
        sys.stderr.write(' '.join(cmd) + '\n' + r.stdout + r.stderr)
    if r.returncode:
        raise RuntimeError(f'nvcc failed on {src.name}')
    return obj, r.stderr


def build(force=False, verbose=False, extra=()):
    OBJ.mkdir(exist_ok=True)
    if force:
        for o in OBJ.glob('*.o'):
            o.unlink()
    srcs = sorted(CSRC.glob('*.cu'))
    with ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        objs = [o for o, _ in ex.map(lambda s: _compile(s, verbose, extra), srcs)]
    if LIB.exists() and LIB.stat().st_mtime >= max(o.stat().st_mtime for o in objs) and not force:
        return LIB
    cmd = [NVCC, *ARCH, '-shared', '-o', str(LIB), *map(str, objs)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode:
        sys.stderr.write(' '.join(cmd) + '\n' + r.stdout + r.stderr)
        raise RuntimeError('link failed')
    return LIB


if __name__ == '__main__':
    ap = argparse.ArgumentParser()
    ap.add_argument('--force', action='store_true')
    ap.add_argument('--verbose', action='store_true')
    ap.add_argument('--ptxas', action='store_true', help='print register / shared-memory use (-Xptxas -v)')
    a = ap.parse_args()
    print(build(force=a.force or a.ptxas, verbose=a.verbose or a.ptxas, extra=('-Xptxas', '-v') if a.ptxas else ()))
