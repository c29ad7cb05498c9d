"""Packed trellis-coded layers on the device: the reference's on-disk format and the load-time INT8 snap.

packed.safetensors, per quantized Linear `name` (the reference's layout, deploy/tcq_kernels/tcq_format.py:3-12):
  <name>::bits       int16 view of the uint16 words (m/16 * n/16, 32): 512 bits per 16 x 16 tile
  <name>::tlut       FP16 (512, 2) lookup table
  <name>::row_scale  FP16 (m,)
  <name>::su, ::sv   int8 (n,), (m,) signs of the two-sided randomized block-Walsh rotation
At load the INT8 runtime derives t8 = round(tlut * g), g = 127 / max|tlut|, and rs = FP32(row_scale) / g
(tcq_format.py:74-77): decoded weight = sign * t8[hash(state)] * rs[row] in the rotated basis.

Decoding, rotation and products run through the sm_100a kernels (`kernels`); this module holds no arithmetic of its
own beyond the load-time snap, which is PyTorch on the device exactly as in the reference.
"""
import os
from pathlib import Path

import torch

from . import kernels as K

FIELDS = ('bits', 'tlut', 'row_scale', 'su', 'sv')


def block_widths(width):
    """Binary decomposition of a width into descending power-of-two blocks (tcq_format.py:26-30)."""
    out = []
    while width:
        b = 1 << (width.bit_length() - 1)
        out.append(b)
        width -= b
    return out


def snap(tlut, row_scale):
    """INT8 table and FP32 row scales derived at load (tcq_format.py:74-77). The expression is kept exactly as the
    reference writes it: `127.0 / t` is PyTorch's reciprocal-then-multiply, which the bit-exact parity depends on."""
    g = (127.0 / tlut.float().abs().max()).to(torch.float32)
    t8 = torch.round(tlut.float() * g).clamp(-127, 127).to(torch.int8)
    return t8, row_scale.float() / g, g


class Layer:
    """One quantized Linear on a device: packed tensors + derived INT8 table / row scales (tcq_format.py:80-107)."""
    def __init__(self, name, tensors, bias=None, device='cuda'):
        self.name = name
        self.bits = tensors['bits'].to(device).contiguous()
        self.tlut = tensors['tlut'].to(device)
        self.row_scale = tensors['row_scale'].to(device)
        self.su, self.sv = tensors['su'].to(device).contiguous(), tensors['sv'].to(device).contiguous()
        self.m, self.n = self.sv.numel(), self.su.numel()
        if not (self.bits.shape == ((self.m // 16) * (self.n // 16), 32) and self.m % 16 == 0 and self.n % 16 == 0):
            raise ValueError(f'{name}: bits {tuple(self.bits.shape)} do not match a ({self.m}, {self.n}) layer of 16 x 16 tiles')
        self.t8, self.rs, self.gain = snap(self.tlut, self.row_scale)
        self.t8 = self.t8.contiguous()
        self.rs = self.rs.contiguous()
        self.bias = None if bias is None else bias.float().to(device).contiguous()

    def w8(self, out=None):
        """Decoded INT8 weight (m, n) in the rotated basis (the sm_100a decode kernel)."""
        out = torch.empty(self.m, self.n, dtype=torch.int8, device=self.bits.device) if out is None else out
        K.decode(self.bits, self.t8, out)
        return out

    def dense(self):
        """Original-basis weight S_v H_m diag(rs) Q8 H_n S_u (FP32) with the INT8 table (tcq_format.py:100-107)."""
        q = self.w8().float() * self.rs[:, None]
        w = K.rotate(q, self.su, inverse=True)                      # (Q H_n) S_u, H symmetric
        return K.rotate(w.t().contiguous(), self.sv, inverse=True).t()


def save(path, layers):
    """Write `layers` ({name: dict of the five packed tensors}) as packed.safetensors, atomically (temp + rename)."""
    from safetensors.torch import save_file
    path = Path(path)
    out = {}
    for name, t in layers.items():
        for k in FIELDS:
            v = t[k]
            if k == 'bits' and v.dtype != torch.int16:
                v = v.view(torch.int16) if v.element_size() == 2 else v.to(torch.int16)
            out[f'{name}::{k}'] = v.detach().cpu().contiguous()
    tmp = path.with_suffix('.partial')
    save_file(out, str(tmp))
    os.replace(tmp, path)


def load(path, device='cuda', names=None, biases=None):
    """packed.safetensors -> {name: Layer} (tcq_format.py:230-237)."""
    from safetensors import safe_open
    out = {}
    with safe_open(str(path), framework='pt', device='cpu') as f:
        keys = sorted({k.split('::')[0] for k in f.keys()})
        for name in (names or keys):
            out[name] = Layer(name, {k: f.get_tensor(f'{name}::{k}') for k in FIELDS}, bias=(biases or {}).get(name), device=device)
    return out
