"""Test helpers for zero padding and formatted buffer strides: the zero-interval mask
(zero_pad_ir.rs: any padded axis coordinate in [left, right)) and packing of a logical
batch-major tensor into / out of a formatted buffer (config.rs:1463-1522 stride
resolution, nd_ir.rs:1190-1260 pack / unpack)."""
import numpy as np


def pad_mask(dims, pads):
    mask = np.zeros(dims, dtype=bool)
    for axis, (lo, hi) in pads.items():
        idx = [slice(None)] * len(dims)
        idx[int(axis)] = slice(lo, hi)
        mask[tuple(idx)] = True
    return mask


def resolve(dims, strides, batch_stride):
    st = [1] * len(dims)
    for a in range(len(dims) - 2, -1, -1):
        st[a] = (strides or {}).get(a, st[a + 1] * dims[a + 1])
    return st, (batch_stride or st[0] * dims[0])


def _offsets(dims, st):
    idx = np.indices(dims).reshape(len(dims), -1)
    return sum(idx[a] * st[a] for a in range(len(dims)))


def pack(x, dims, strides=None, batch_stride=None, fill=7.0):
    st, bs = resolve(dims, strides, batch_stride)
    phys = np.full(bs * x.shape[0], fill, dtype=x.dtype)
    off = _offsets(dims, st)
    for b in range(x.shape[0]):
        phys[b * bs + off] = x[b].reshape(-1)
    return phys


def unpack(phys, dims, strides, batch_stride, batch):
    st, bs = resolve(dims, strides, batch_stride)
    off = _offsets(dims, st)
    return np.stack([phys[b * bs + off].reshape(dims) for b in range(batch)])
