"""Generate the golden fixtures by running the reference's own PyTorch definition on CPU.

    python tests/golden/make_golden.py path/to/reference/deploy/tcq_kernels
    TCQ_REF_ROOT=path/to/reference/deploy/tcq_kernels python tests/golden/make_golden.py

Imports `tcq_format.py` from the reference checkout (read-only; its directory is the first argument, or the
TCQ_REF_ROOT environment variable; one of them is required), feeds it the seeded inputs of `cases.py`, and writes
`golden.npz` (small outputs in full) and `golden_sha256.json` (SHA-256 of the exact bytes of every output,
large ones included). The fixtures, not the reference, travel with the repository: the tests never import it.
"""
import hashlib
import json
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
import cases  # noqa: E402

FULL_LIMIT = 48 * 1024          # outputs up to this many bytes are stored in full


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def t_bits(u16):
    return torch.from_numpy(np.ascontiguousarray(u16).view(np.int16)).view(torch.bfloat16)


def bf16_np(t):
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def main():
    ref_root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get('TCQ_REF_ROOT')
    if not ref_root:
        raise SystemExit('make_golden.py: give the reference directory deploy/tcq_kernels as the first argument or in TCQ_REF_ROOT')
    sys.dont_write_bytecode = True
    sys.path.insert(0, ref_root)
    import tcq_format as F                            # the reference definition (read-only import)
    torch.set_num_threads(os.cpu_count())
    full, digests = {}, {}

    def put(key, arr):
        arr = np.ascontiguousarray(arr)
        digests[key] = dict(sha256=sha(arr), dtype=str(arr.dtype), shape=list(arr.shape))
        if arr.nbytes <= FULL_LIMIT:
            full[key] = arr

    for name, m, n, tokens, dt, has_bias in cases.LAYERS:
        t, b = cases.layer_tensors(name, m, n, has_bias)
        tens = dict(bits=torch.from_numpy(t['bits'].view(np.int16).copy()), tlut=torch.from_numpy(t['tlut']),
                    row_scale=torch.from_numpy(t['row_scale']), su=torch.from_numpy(t['su']), sv=torch.from_numpy(t['sv']))
        L = F.Layer(name, tens, bias=None if b is None else torch.from_numpy(b), device='cpu')
        w8 = L.w8_reference()
        put(f'{name}/t8', L.t8.numpy()); put(f'{name}/rs', L.rs.numpy()); put(f'{name}/gain', np.float32(L.gain).reshape(1))
        put(f'{name}/states', L.states().numpy().astype(np.int32))
        put(f'{name}/w8', w8.numpy())
        if m * n <= 64 * 1152:
            put(f'{name}/dense_fp16', L.dense('fp16').numpy()); put(f'{name}/dense_int8', L.dense('int8').numpy())
        for M in tokens:
            x = cases.activations(name, M, n, dt)
            xt = t_bits(x) if dt == 'bf16' else torch.from_numpy(x)
            h = F.fwht(xt.float() * L.su.float())
            q, s = F.quantize_tokens(h)
            acc = F.int_matmul(q, w8)
            z = (acc.float() * s) * L.rs[None, :]
            y = F.reference_linear(xt, L, w8=w8)
            put(f'{name}/M{M}/h', h.numpy()); put(f'{name}/M{M}/q', q.numpy()); put(f'{name}/M{M}/scale', s[:, 0].numpy())
            put(f'{name}/M{M}/acc', acc.numpy()); put(f'{name}/M{M}/z', z.numpy()); put(f'{name}/M{M}/y', bf16_np(y))
            if m * n <= 1536 * 1536:
                put(f'{name}/M{M}/y_a16', bf16_np(F.reference_linear(xt, L, a8=False, w8=w8)))
                put(f'{name}/M{M}/y_fp16table', bf16_np(F.reference_linear(xt, L, table='fp16')))
                put(f'{name}/M{M}/y_fp16table_a16', bf16_np(F.reference_linear(xt, L, a8=False, table='fp16')))
        print(name, 'done', flush=True)

    for i in range(cases.SNAP_TABLES):
        tlut, rsc = cases.snap_inputs(i)
        t8, rs, g = F.snap(torch.from_numpy(tlut), torch.from_numpy(rsc))
        put(f'snap/{i}/t8', t8.numpy()); put(f'snap/{i}/rs', rs.numpy()); put(f'snap/{i}/gain', np.float32(g).reshape(1))
    print('snap done', flush=True)

    for T, D in cases.ROTATIONS:
        x, s = cases.rotation_input(T, D)
        fwd = F.fwht(t_bits(x).float() * torch.from_numpy(s).float())
        inv = F.fwht(fwd) * torch.from_numpy(s).float()
        put(f'rot/{T}x{D}/fwd', fwd.numpy()); put(f'rot/{T}x{D}/inv', inv.numpy())
    print('rotations done', flush=True)

    for M, K, N in cases.GEMMS:
        a, w, sc = cases.gemm_inputs(M, K, N)
        q, s = F.quantize_tokens(t_bits(a).float())
        acc = F.int_matmul(q, torch.from_numpy(w))
        out = ((acc.float() * s) * torch.from_numpy(sc)[None, :]).to(torch.bfloat16)
        put(f'gemm/{M}x{K}x{N}/q', q.numpy()); put(f'gemm/{M}x{K}x{N}/scale', s[:, 0].numpy())
        put(f'gemm/{M}x{K}x{N}/acc', acc.numpy()); put(f'gemm/{M}x{K}x{N}/out', bf16_np(out))
    print('gemms done', flush=True)

    np.savez_compressed(HERE / 'golden.npz', **full)
    meta = dict(generator='tests/golden/make_golden.py', reference='deploy/tcq_kernels/tcq_format.py (ForeverBlue816/yanlongvla)',
                torch=torch.__version__, digests=digests)
    (HERE / 'golden_sha256.json').write_text(json.dumps(meta, indent=1, sort_keys=True))
    print('wrote', len(full), 'full arrays,', len(digests), 'digests')


if __name__ == '__main__':
    main()
