"""Access to the committed golden fixtures (outputs of the reference's tcq_format.py on the inputs of cases.py)."""
import hashlib
import json
from functools import lru_cache
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


@lru_cache(maxsize=1)
def _full():
    with np.load(HERE / 'golden.npz') as f:
        return {k: f[k] for k in f.files}


@lru_cache(maxsize=1)
def _digests():
    return json.loads((HERE / 'golden_sha256.json').read_text())['digests']


def keys():
    return sorted(_digests())


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def check(key, arr):
    """True when arr has the exact bytes, dtype and shape the reference produced for `key`."""
    d = _digests()[key]
    arr = np.ascontiguousarray(arr)
    assert str(arr.dtype) == d['dtype'], (key, arr.dtype, d['dtype'])
    assert list(arr.shape) == d['shape'], (key, arr.shape, d['shape'])
    if sha(arr) == d['sha256']:
        return True
    full = _full().get(key)
    if full is not None:
        bad = np.flatnonzero(full.reshape(-1) != arr.reshape(-1))
        raise AssertionError(f'{key}: {bad.size} mismatching elements, first at {bad[:5]}')
    raise AssertionError(f'{key}: sha256 mismatch')


def get(key):
    return _full()[key]
