"""Helpers shared by the GPU parity tests: numpy <-> torch conversions and seeded layers on the device."""
import numpy as np
import torch

import cases
import tcq_oracle as O


def dev():
    return torch.device('cuda')


def t(a, dtype=None):
    """numpy -> CUDA tensor; uint16 arrays become BF16 tensors (bit patterns), int16/uint16 bits stay int16 when asked."""
    a = np.ascontiguousarray(a)
    if dtype == 'bf16' or (dtype is None and a.dtype == np.uint16):
        return torch.from_numpy(a.view(np.int16).copy()).view(torch.bfloat16).to(dev())
    if dtype == 'i16':
        return torch.from_numpy(a.view(np.int16).copy()).to(dev())
    return torch.from_numpy(a.copy()).to(dev())


def n(x):
    """CUDA tensor -> numpy (BF16 -> uint16 bit patterns)."""
    x = x.detach().cpu().contiguous()
    if x.dtype == torch.bfloat16:
        return x.view(torch.int16).numpy().view(np.uint16)
    return x.numpy()


class DevLayer:
    """Seeded synthetic layer (tests/golden/cases.py) as the oracle Layer and its device tensors."""
    def __init__(self, name, m, nn, bias=False):
        tens, b = cases.layer_tensors(name, m, nn, bias)
        self.ref = O.Layer(tens['bits'], tens['tlut'], tens['row_scale'], tens['su'], tens['sv'], bias=b)
        self.m, self.n = m, nn
        self.bits = t(tens['bits'], 'i16')
        self.t8 = t(self.ref.t8)
        self.rs = t(self.ref.rs)
        self.su = t(tens['su'])
        self.sv = t(tens['sv'])
        self.bias = None if b is None else t(b)


def x_dev(x, dt):
    return t(x, 'bf16') if dt == 'bf16' else t(x)
