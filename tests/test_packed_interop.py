"""Packed on-disk format (`<name>::bits/tlut/row_scale/su/sv` safetensors) against the reference's own reader and
writer, through the fixtures of tests/golden/make_packed.py:

  * a file in the layout the reference's `build` writes (packed_ref.safetensors) loads with this repository's
    `tcq_format.load`, and its layers decode to the reference's `w8_reference()` bytes (PyTorch-ops decoder on the
    CPU here; the sm_100a decode kernel in the GPU test);
  * this repository's `tcq_format.save` writes the same tensors under the same keys, dtypes and shapes;
  * the generator recorded that the reference's `load` reads a file written by `tcq_format.save` back to identical
    tensors and identical `w8_reference()`.
"""
import hashlib
import json
from pathlib import Path

import numpy as np
import pytest
import torch

HERE = Path(__file__).resolve().parent / 'golden'
META = json.loads((HERE / 'packed_ref.json').read_text())
FIELDS = ('bits', 'tlut', 'row_scale', 'su', 'sv')


def _sha(t):
    return hashlib.sha256(t.contiguous().cpu().numpy().tobytes()).hexdigest()


def _raw(path):
    from safetensors.torch import load_file
    return load_file(str(path))


def test_reference_file_loads_and_decodes():
    from yanlongvla_b200 import definition as D
    from yanlongvla_b200 import tcq_format as TF
    layers = TF.load(HERE / 'packed_ref.safetensors', device='cpu')
    assert sorted(layers) == sorted(META['layers'])
    for name, rec in META['layers'].items():
        L = layers[name]
        assert [L.m, L.n] == rec['shape']
        assert _sha(L.t8) == rec['t8_sha256'] and _sha(L.rs) == rec['rs_sha256']          # load-time snap
        assert _sha(D.decode_w8(L.bits, L.t8, L.m, L.n)) == rec['w8_reference_sha256']


def test_writer_matches_reference_layout(tmp_path):
    from yanlongvla_b200 import tcq_format as TF
    ref = _raw(HERE / 'packed_ref.safetensors')
    names = sorted({k.split('::')[0] for k in ref})
    p = tmp_path / 'packed.safetensors'
    TF.save(p, {nm: {k: ref[f'{nm}::{k}'] for k in FIELDS} for nm in names})
    mine = _raw(p)
    assert sorted(mine) == sorted(ref)
    for k, v in ref.items():
        assert mine[k].dtype == v.dtype and mine[k].shape == v.shape and torch.equal(mine[k], v), k
    assert ref[f'{names[0]}::bits'].dtype == torch.int16                 # uint16 words stored as their int16 view


def test_writer_takes_uint16_words_as_int32(tmp_path):
    """Words held as int32 values 0..65535 (how numpy uint16 arrays often arrive) are stored as the int16 view."""
    from yanlongvla_b200 import tcq_format as TF
    ref = _raw(HERE / 'packed_ref.safetensors')
    nm = sorted({k.split('::')[0] for k in ref})[0]
    t = {k: ref[f'{nm}::{k}'] for k in FIELDS}
    words = torch.from_numpy(t['bits'].numpy().view(np.uint16).astype(np.int32))
    p = tmp_path / 'p.safetensors'
    TF.save(p, {nm: dict(t, bits=words)})
    assert torch.equal(_raw(p)[f'{nm}::bits'], t['bits'])


def test_reference_reads_repository_files():
    assert META['repo_written_read_by_reference'] and all(META['repo_written_read_by_reference'].values())


@pytest.mark.gpu
def test_reference_file_decodes_on_gpu():
    if not torch.cuda.is_available():
        pytest.skip('no CUDA device')
    from yanlongvla_b200 import tcq_format as TF
    layers = TF.load(HERE / 'packed_ref.safetensors', device='cuda')
    for name, rec in META['layers'].items():
        assert _sha(layers[name].w8()) == rec['w8_reference_sha256'], name
