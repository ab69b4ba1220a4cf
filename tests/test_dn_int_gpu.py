"""The integer DeltaNet head step (trx_deltanet_int_step; model/deltanet.py:99-147 head_step) against
golden vectors made by the reference's own head_step (tests/golden/dn_int_steps.npz, the shapes and
token schedule of test/model/test_asm.py:554-590: the state starts empty at exponent -20, the first
tokens ratchet, the small last one does not): the int16 state, exponent, max |M| and fp32 output are
bit-exact, token after token with the state kept on the device; heads of one launch are independent;
the reference-surface drop-in (trixium_b200.deltanet.head_step) gives the same."""
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN, load

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def fx():
    return load(os.path.join(GOLDEN, "dn_int_steps.npz"))


@pytest.fixture(scope="module")
def ctx():
    from trixium_b200 import ops
    c = ops.Context(0)
    yield c
    c.close()


def _tok(d, tag, t, n):
    return d[f"{tag}_t{t}_{n}"]


@pytest.mark.parametrize("shape", [(64, 64, 1), (128, 128, 2), (128, 128, 3), (32, 64, 4)])
def test_int_head_step_bit_exact(fx, ctx, shape):
    from trixium_b200 import ops
    hv, hk, seed = shape
    tag = f"h{hv}x{hk}s{seed}"
    dev = ctx.device
    st = torch.zeros(1, hv, hk, dtype=torch.int16, device=dev)
    ex = torch.tensor([-20], dtype=torch.int32, device=dev)
    mx = torch.tensor([0], dtype=torch.int32, device=dev)
    for t in range(4):
        g = lambda n: torch.from_numpy(np.ascontiguousarray(_tok(fx, tag, t, n), dtype=np.float32).reshape(1, -1)).to(dev)
        assert int(ex.item()) == int(_tok(fx, tag, t, "eM")) and int(mx.item()) == int(_tok(fx, tag, t, "maxM"))
        o = ops.deltanet_int_step(ctx, st, ex, mx, g("k"), g("q"), g("v"), g("decay").reshape(1), g("beta").reshape(1))
        assert np.array_equal(st.cpu().numpy()[0], _tok(fx, tag, t, "M")), t
        assert int(ex.item()) == int(_tok(fx, tag, t, "eM2"))
        assert int(mx.item()) == int(_tok(fx, tag, t, "maxM2"))
        assert np.array_equal(o.cpu().numpy()[0].view(np.uint32), _tok(fx, tag, t, "o").view(np.uint32)), t
    assert ctx.errors() == 0


def test_int_heads_in_one_launch(fx, ctx):
    """Both 128 x 128 sequences as two heads of one launch, maxM computed by the kernel (negative)."""
    from trixium_b200 import ops
    dev = ctx.device
    tags = ["h128x128s2", "h128x128s3"]
    st = torch.zeros(2, 128, 128, dtype=torch.int16, device=dev)
    ex = torch.tensor([-20, -20], dtype=torch.int32, device=dev)
    for t in range(4):
        mx = torch.full((2,), -1, dtype=torch.int32, device=dev)
        g = lambda n: torch.from_numpy(np.stack([np.asarray(_tok(fx, tg, t, n), dtype=np.float32).reshape(-1)
                                                 for tg in tags])).to(dev)
        o = ops.deltanet_int_step(ctx, st, ex, mx, g("k"), g("q"), g("v"), g("decay").reshape(2), g("beta").reshape(2))
        for i, tg in enumerate(tags):
            assert np.array_equal(st.cpu().numpy()[i], _tok(fx, tg, t, "M")), (tg, t)
            assert int(ex[i].item()) == int(_tok(fx, tg, t, "eM2"))
            assert int(mx[i].item()) == int(_tok(fx, tg, t, "maxM2"))
            assert np.array_equal(o.cpu().numpy()[i].view(np.uint32), _tok(fx, tg, t, "o").view(np.uint32))
    assert ctx.errors() == 0


def test_reference_surface_head_step(fx):
    from trixium_b200 import deltanet
    tag = "h64x64s1"
    M = np.zeros((64, 64), dtype=np.int64)
    eM, maxM = -20, 0
    for t in range(4):
        g = lambda n: _tok(fx, tag, t, n)
        o, eM, maxM = deltanet.head_step(M, eM, g("k"), g("q"), g("v"), g("decay"), g("beta"), maxM=maxM)
        assert np.array_equal(M, g("M").astype(np.int64))
        assert eM == int(g("eM2")) and maxM == int(g("maxM2"))
        assert np.array_equal(o.view(np.uint32), g("o").view(np.uint32))
