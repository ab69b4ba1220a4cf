"""Drop-in for the reference's engine entry points (model/bitexact.py), run on the B200.

Same names, arguments and results as the reference:

    matvec_ternary(scales_f16 (M,G), codes (M,K) uint8 {0,1,2}, x8 (K,) int8, B, R) -> int32 (M,)
        model/bitexact.py:101-119
    matvec_ternary_rows(scales, codes, x8_rows (nr+1,K), B, R) -> int32 (nr+1, M)
        model/bitexact.py:121-125
    matvec_q8(scales_f16 (M,K/32), q8w (M,K) int8, x8 (K,) int8, B, R) -> int32 (M,)
        model/bitexact.py:127-144

The codes are packed once into the converter's row packets (2-bit by default, or trit5 with
kind=5) and cached on the device by the identity of the arrays; the matvec runs in
libtrixium_b200.so.  Where the reference asserts (int48 accumulator or int32 result overflow,
model/bitexact.py:116,118), this raises AssertionError with the same message.
"""

import numpy as np
import torch

from . import _lib
from . import ops
from .image import Q8Tensor, TernaryTensor

_cache = {}


def _device_tensor(scales, codes, B, R, kind):
    key = (id(scales), id(codes), scales.shape, codes.shape, int(B), int(R), kind)
    hit = _cache.get(key)
    if hit is not None and hit[0] is scales and hit[1] is codes:
        return hit[2]
    t = TernaryTensor(scales, codes, kind=kind, bias=B, rshift=R)
    dt = ops.DeviceTensor(t)
    _cache[key] = (scales, codes, dt)
    return dt


def _raise_device(ctx):
    bits = ctx.errors()
    if bits & _lib.DEV_OVERFLOW:
        raise AssertionError("int48 accumulator overflow or int32 result overflow")
    if bits:
        raise _lib.TrxDeviceError(bits)


def matvec_ternary(scales_f16, codes, x8, B, R, kind=0):
    ctx = ops.default_context()
    codes = np.asarray(codes)
    dt = _device_tensor(scales_f16, codes, B, R, kind)
    x8_t = torch.from_numpy(np.ascontiguousarray(np.asarray(x8, dtype=np.int8))).to(ctx.device)
    out = ops.matvec_i8(ctx, dt, x8_t)
    _raise_device(ctx)
    return out.cpu().numpy()


def matvec_ternary_rows(scales_f16, codes, x8_rows, B, R, kind=0):
    ctx = ops.default_context()
    codes = np.asarray(codes)
    dt = _device_tensor(scales_f16, codes, B, R, kind)
    x = np.ascontiguousarray(np.asarray(x8_rows, dtype=np.int8))
    outs = []
    for c0 in range(0, x.shape[0], 32):  # up to 32 rows per launch (9..32 on the tensor cores)
        xt = torch.from_numpy(x[c0:c0 + 32]).to(ctx.device)
        outs.append(ops.matvec_i8_rows(ctx, dt, xt))
    _raise_device(ctx)
    return torch.cat(outs).cpu().numpy()


def matvec_q8(scales_f16, q8w, x8, B, R):
    ctx = ops.default_context()
    q8w = np.asarray(q8w)
    key = (id(scales_f16), id(q8w), np.shape(scales_f16), q8w.shape, int(B), int(R), "q8")
    hit = _cache.get(key)
    if hit is not None and hit[0] is scales_f16 and hit[1] is q8w:
        dt = hit[2]
    else:
        dt = ops.DeviceTensor(Q8Tensor(scales_f16, q8w, bias=B, rshift=R))
        _cache[key] = (scales_f16, q8w, dt)
    x8_t = torch.from_numpy(np.ascontiguousarray(np.asarray(x8, dtype=np.int8))).to(ctx.device)
    out = ops.matvec_q8(ctx, dt, x8_t)
    _raise_device(ctx)
    return out.cpu().numpy()
