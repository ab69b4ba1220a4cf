"""K-segmented float projections (trx_matvec_f_kseg, through the C ABI) against the mirror's
(tests/golden/kseg_*.npz: model/bons.py split_wide segments of a 17408-wide ternary tensor, trit5 and
2-bit, and of a 9216-wide Q8 tensor, with model/mirror.py:664-678's float projection): fp32 bits."""
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN, load

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", ["t5_24x17408", "2b_40x17408", "q8_20x9216"])
def test_kseg_projection_bit_exact(name):
    from trixium_b200 import ops
    d = load(os.path.join(GOLDEN, f"kseg_{name}.npz"))
    ctx = ops.Context(0)
    try:
        rows, kind, B, R = int(d["rows"]), int(d["kind"]), int(d["B"]), int(d["R"])
        segs = [ops.DeviceTensor.from_packed(d[f"packed{k}"], rows, int(d[f"cols{k}"]), kind, B, R)
                for k in range(int(d["nseg"]))]
        x = torch.from_numpy(d["x"]).cuda()
        y = ops.matvec_f_kseg(ctx, segs, x)
        assert np.array_equal(y.cpu().numpy().view(np.uint32), d["y"].view(np.uint32))
        # With a residual: resid + y in fp32, as the mirror's x = x + y (model/mirror.py:1013).
        resid = torch.randn(rows, device="cuda")
        y2 = ops.matvec_f_kseg(ctx, segs, x, resid=resid)
        want = (resid.cpu().numpy() + d["y"]).astype(np.float32)
        assert np.array_equal(y2.cpu().numpy().view(np.uint32), want.view(np.uint32))
        assert ctx.errors() == 0
    finally:
        ctx.close()
