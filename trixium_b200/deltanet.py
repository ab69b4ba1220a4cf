"""The integer gated-DeltaNet head step on the B200, with the reference's call surface.

`head_step(M, eM, kk, qh, vh, decay, beta, maxM=None)` is model/deltanet.py:99-147's function: one
value head's int16-range state M (hv x hk, updated in place) at exponent eM, the head's fp32 key,
query and value, decay and beta; it returns (o float32 (hv,), eM2, maxM2) and raises AssertionError
where the reference asserts.  The step runs as trx_deltanet_int_step on the device (host arrays are
copied in and out); `ops.deltanet_int_step` is the device-resident form over many heads.
"""

import numpy as np
import torch

from . import _lib, ops


def head_step(M, eM, kk, qh, vh, decay, beta, maxM=None, ctx=None):
    """model/deltanet.py:99 head_step on the device.  M: integer array (hv, hk), updated in place."""
    ctx = ctx or ops.default_context()
    dev = ctx.device
    M = np.asarray(M)
    hv, hk = M.shape
    if np.abs(M).max(initial=0) > 32767:
        raise AssertionError("state outside int16")
    st = torch.from_numpy(M.astype(np.int16).reshape(1, hv, hk)).to(dev)
    ex = torch.tensor([int(eM)], dtype=torch.int32, device=dev)
    mx = torch.tensor([-1 if maxM is None else int(maxM)], dtype=torch.int32, device=dev)
    f = lambda a: torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32).reshape(1, -1)).to(dev)
    o = ops.deltanet_int_step(ctx, st, ex, mx, f(kk), f(qh), f(vh), f([decay]).reshape(1), f([beta]).reshape(1))
    bits = ctx.errors()
    if bits & _lib.TRX_DEV_OVERFLOW:
        raise AssertionError("a value outside the reference's asserted ranges")
    if bits:
        raise _lib.TrxDeviceError(bits)
    M[:] = st.cpu().numpy()[0].astype(M.dtype)
    return o.cpu().numpy()[0], int(ex.item()), int(mx.item())


__all__ = ["head_step"]
