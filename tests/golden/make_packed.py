"""Generate the packed-format interop fixtures with the reference's own tcq_format.py (run once, in a checkout that has
the reference; the fixtures, not the reference, travel with the repository).

    python tests/golden/make_packed.py path/to/reference/deploy/tcq_kernels
    TCQ_REF_ROOT=path/to/reference/deploy/tcq_kernels python tests/golden/make_packed.py

1. Reference -> repository: seeded layers become the reference's `Layer` objects, and their packed tensors are written
   as the reference's `build` writes them (`<name>::<field>` tensors, contiguous, one safetensors file;
   deploy/tcq_kernels/tcq_format.py:191-227) to `packed_ref.safetensors`, with the SHA-256 of each layer's
   `w8_reference()` (deploy/tcq_kernels/tcq_format.py:97-98) in `packed_ref.json`.
2. Repository -> reference: the same layers written by this repository's `tcq_format.save` into a temporary
   VLA_ROOT are read back by the reference's own `load` (deploy/tcq_kernels/tcq_format.py:230-237); the JSON records
   whether every tensor and every `w8_reference()` it produced equals the reference-written file's.

tests/test_packed_interop.py checks the repository's loader, writer and decoders against these fixtures.
"""
import hashlib
import importlib
import json
import os
import sys
import tempfile
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
sys.path.insert(0, str(HERE.parent.parent))
import cases  # noqa: E402

ROW = 'interop_row'
LAYERS = [('blk.0.attn.q_proj', 256, 256, False), ('blk.0.mlp.fc1', 64, 1152, True), ('blk.0.odd', 48, 80, False)]
FIELDS = ('bits', 'tlut', 'row_scale', 'su', 'sv')


def sha(t):
    return hashlib.sha256(t.contiguous().numpy().tobytes()).hexdigest()


def packed_tensors(name, m, n, has_bias):
    t, _ = cases.layer_tensors('packed.' + name, m, n, has_bias)
    return dict(bits=torch.from_numpy(t['bits'].view(np.int16).copy()), tlut=torch.from_numpy(t['tlut']),
                row_scale=torch.from_numpy(t['row_scale']), su=torch.from_numpy(t['su']), sv=torch.from_numpy(t['sv']))


def main():
    ref_root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get('TCQ_REF_ROOT')
    if not ref_root:
        raise SystemExit('make_packed.py: give the reference directory deploy/tcq_kernels as the first argument or in TCQ_REF_ROOT')
    from safetensors.torch import save_file
    sys.dont_write_bytecode = True
    with tempfile.TemporaryDirectory() as tmp:
        os.environ['VLA_ROOT'] = tmp                      # the reference resolves its packed path from VLA_ROOT at import
        sys.path.insert(0, ref_root)
        F = importlib.import_module('tcq_format')
        # 1. the reference's objects and writer layout
        out, record = {}, {}
        for name, m, n, has_bias in LAYERS:
            L = F.Layer(name, packed_tensors(name, m, n, has_bias), device='cpu')
            for k in FIELDS:
                out[f'{name}::{k}'] = getattr(L, k).contiguous()
            record[name] = dict(shape=[m, n], w8_reference_sha256=sha(L.w8_reference()), t8_sha256=sha(L.t8), rs_sha256=sha(L.rs))
        save_file(out, str(HERE / 'packed_ref.safetensors'))
        # 2. this repository's writer, the reference's reader
        from yanlongvla_b200 import tcq_format as TF
        p = Path(tmp) / 'models' / 'pi05_tcq' / ROW / 'packed.safetensors'
        p.parent.mkdir(parents=True)
        TF.save(p, {name: packed_tensors(name, m, n, b) for name, m, n, b in LAYERS})
        back = F.load(ROW, device='cpu', names=[name for name, *_ in LAYERS])
        same = {}
        for name, *_ in LAYERS:
            B = back[name]
            same[name] = bool(all(torch.equal(getattr(B, k), out[f'{name}::{k}']) for k in FIELDS)
                              and sha(B.w8_reference()) == record[name]['w8_reference_sha256'])
    meta = dict(generator='tests/golden/make_packed.py', reference='deploy/tcq_kernels/tcq_format.py (ForeverBlue816/yanlongvla)',
                torch=torch.__version__, row=ROW, layers=record, repo_written_read_by_reference=same)
    (HERE / 'packed_ref.json').write_text(json.dumps(meta, indent=1, sort_keys=True))
    print(json.dumps(same))


if __name__ == '__main__':
    main()
