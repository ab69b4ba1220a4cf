"""Failure detection on the device without a fault: a matvec launch told to wait for a peer
exchange that no rank ever signals (trx_matvec_f_tp with a wait counter left at zero) gives up after
its bounded wait (200 ms of %globaltimer per CTA), records TRX_DEV_TIMEOUT in the context's error
word, finishes its work, and leaves the context usable: the next plain launch on the same context
is bit-exact and raises no error bit.  Nothing here faults, traps or hangs the GPU: the wait is a
plain bounded poll of a device counter."""
import ctypes
import time

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_unsignalled_exchange_times_out_and_context_survives():
    from oracle import build as cor
    from trixium_b200 import _lib, image, ops
    ctx = ops.Context(0)
    try:
        t, x = image.synthetic_matvec_case(512, 2048, seed=5, kind=5)
        w = ops.DeviceTensor(t)
        xd = torch.from_numpy(x).cuda()
        want, bad = cor.matvec_f(t.packed, t.rows, t.cols, 5, t.bias, t.rshift, x)
        assert bad == 0
        counter = torch.zeros(1, dtype=torch.int32, device="cuda")   # nothing ever adds to it
        step = torch.zeros(1, dtype=torch.int32, device="cuda")
        tp = _lib.TpXfer()
        tp.world, tp.rank = 2, 0                                     # waits for 2 arrivals
        tp.wait = ctypes.c_void_p(counter.data_ptr())
        tp.step = ctypes.c_void_p(step.data_ptr())
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        y = ops.matvec_f(ctx, w, xd, tp=tp)
        torch.cuda.synchronize()
        waited = time.perf_counter() - t0
        assert ctx.errors() == _lib.TRX_DEV_TIMEOUT
        assert 0.15 < waited < 5.0, waited
        # The launch still computed its rows from its own input.
        assert np.array_equal(y.cpu().numpy().view(np.uint32), want.view(np.uint32))
        # The context works afterwards: a plain launch, bit-exact, no error bits.
        y2 = ops.matvec_f(ctx, w, xd)
        assert np.array_equal(y2.cpu().numpy().view(np.uint32), want.view(np.uint32))
        assert ctx.errors() == 0
    finally:
        ctx.close()
