"""The engine's blockwise Hadamard rotation (model/mirror.py:680-690) on the device: the
converter's block tensors through one batched float-projection launch, against the reference's
golden vectors and the oracle."""
import glob
import os

import numpy as np
import pytest
import torch

from oracle import ref
from trixium_b200 import image, ops, layout as L

from conftest import GOLDEN, load

pytestmark = pytest.mark.gpu

HAD_FILES = sorted(glob.glob(os.path.join(GOLDEN, "hadamard_*.npz")))


@pytest.fixture(scope="module")
def ctx():
    c = ops.default_context()
    c.raise_on_error()
    return c


@pytest.mark.parametrize("kind", [L.KIND_TERNARY, L.KIND_TERNARY5])
@pytest.mark.parametrize("path", HAD_FILES, ids=[os.path.basename(f)[9:-4] for f in HAD_FILES])
def test_hadamard_rotation_golden(ctx, path, kind):
    d = load(path)
    t = image.hadamard_tensor(d["signs"], int(d["block"]), kind=kind)
    y = ops.hadamard_rotate(ctx, ops.DeviceTensor(t), torch.from_numpy(d["x"]).cuda()).cpu().numpy()
    ctx.raise_on_error()
    assert np.array_equal(y.view(np.uint32), d["y"].view(np.uint32))


@pytest.mark.parametrize("width,block", [(17408, 512), (4096, 1024), (5120, 256)])
def test_hadamard_rotation_vs_oracle(ctx, width, block):
    rng = np.random.default_rng(width + block)
    signs = np.where(rng.random(width) < 0.5, -1.0, 1.0)
    x = (rng.standard_normal(width) * 3).astype(np.float32)
    x[: block] *= 1e-3                      # blocks quantise with their own exponent
    t = image.hadamard_tensor(signs, block)
    y = ops.hadamard_rotate(ctx, ops.DeviceTensor(t), torch.from_numpy(x).cuda()).cpu().numpy()
    ctx.raise_on_error()
    want = ref.hadamard_rotate(x, t.scales, t.codes, t.bias, t.rshift)
    assert np.array_equal(y.view(np.uint32), want.view(np.uint32))
