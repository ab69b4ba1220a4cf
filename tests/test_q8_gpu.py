"""The Q8 row-dot matvec (trx_matvec_q8) on the device against the reference's golden vectors and
the oracle (model/bitexact.py:127-144, matvec_q8).  Bit-exact: the results are integers."""
import glob
import os

import numpy as np
import pytest
import torch

from oracle import ref
from trixium_b200 import _lib, bitexact, image, ops, layout as L

from conftest import GOLDEN, load

pytestmark = pytest.mark.gpu

Q8_FILES = sorted(glob.glob(os.path.join(GOLDEN, "q8_*.npz")))


@pytest.fixture(scope="module")
def ctx():
    c = ops.default_context()
    c.raise_on_error()
    return c


def run_q8(ctx, packed, rows, cols, B, R, x8):
    dt = ops.DeviceTensor.from_packed(packed, rows, cols, L.KIND_Q8, B, R)
    xt = torch.from_numpy(np.ascontiguousarray(x8, dtype=np.int8)).cuda()
    y = ops.matvec_q8(ctx, dt, xt)
    torch.cuda.synchronize()
    return y.cpu().numpy(), ctx.errors()


@pytest.mark.parametrize("path", Q8_FILES, ids=[os.path.basename(f)[3:-4] for f in Q8_FILES])
def test_q8_golden(ctx, path):
    d = load(path)
    y, bits = run_q8(ctx, d["packed"], int(d["rows"]), int(d["cols"]), int(d["B"]), int(d["R"]), d["x8"])
    assert bits == 0
    assert np.array_equal(y, d["y_int"])


def test_q8_bitexact_dropin(ctx):
    d = load(os.path.join(GOLDEN, "q8_refacc_32x256.npz"))
    y = bitexact.matvec_q8(d["scales"], d["q8w"], d["x8"], int(d["B"]), int(d["R"]))
    assert y.dtype == np.int32 and np.array_equal(y, d["y_int"])


def test_q8_overflow_sets_the_error_word(ctx):
    """Where the reference asserts (R = 0 leaves the int32 result out of range) the device sets
    TRX_DEV_OVERFLOW and the drop-in raises AssertionError."""
    d = load(os.path.join(GOLDEN, "q8_bound_16x512.npz"))
    _, bits = run_q8(ctx, d["packed"], 16, 512, int(d["B"]), 0, d["x8"])
    assert bits & _lib.DEV_OVERFLOW
    with pytest.raises(AssertionError):
        bitexact.matvec_q8(d["scales"], d["q8w"], d["x8"], int(d["B"]), 0)
    ctx.raise_on_error()


def random_q8(rng, rows, cols, sigma=0.02):
    s = (rng.standard_normal((rows, cols // 32)) * sigma).astype(np.float16)
    w = rng.integers(-127, 128, (rows, cols), dtype=np.int8)
    return s, w


@pytest.mark.parametrize("rows,cols", [(1, 32), (7, 96), (300, 544), (1031, 4096), (129, 32768), (4096, 1056)])
def test_q8_random_vs_oracle(ctx, rows, cols):
    rng = np.random.default_rng(rows * 7 + cols)
    s, w = random_q8(rng, rows, cols)
    t = image.Q8Tensor(s, w)
    x8 = rng.integers(-127, 128, cols, dtype=np.int8)
    y, bits = run_q8(ctx, t.packed, rows, cols, t.bias, t.rshift, x8)
    assert bits == 0
    assert np.array_equal(y, ref.matvec_q8(s, w, x8, t.bias, t.rshift))


def test_q8_unaligned_activation(ctx):
    """x8 at an odd byte offset takes the kernel's byte-wise staging path; same result."""
    rng = np.random.default_rng(5)
    rows, cols = 70, 2080
    s, w = random_q8(rng, rows, cols)
    t = image.Q8Tensor(s, w)
    x8 = rng.integers(-127, 128, cols, dtype=np.int8)
    dt = ops.DeviceTensor(t)
    buf = torch.zeros(cols + 16, dtype=torch.int8, device="cuda")
    buf[3:3 + cols] = torch.from_numpy(x8).cuda()
    y = ops.matvec_q8(ctx, dt, buf[3:3 + cols]).cpu().numpy()
    ctx.raise_on_error()
    assert np.array_equal(y, ref.matvec_q8(s, w, x8, t.bias, t.rshift))


def test_q8_full_size_rows_are_independent(ctx):
    """A tensor larger than L2 (16384 x 8192 int8, 136 MB of packets): rows drawn at random from
    the whole tensor equal the oracle run on those rows alone."""
    rows, cols = 16384, 8192
    g = torch.Generator(device="cuda").manual_seed(11)
    w = torch.randint(-127, 128, (rows, cols), dtype=torch.int8, device="cuda", generator=g)
    rng = np.random.default_rng(11)
    s = (rng.uniform(0.005, 0.02, (rows, cols // 32))).astype(np.float16)
    B = image.scale_bias(s)
    R = image.result_shift(s, B, image.GS_MAX_Q8)
    G = cols // 32
    sb = L.ceil_div(G, L.SCALES_PER_BEAT) * L.BEAT_BYTES
    packed = torch.zeros(rows, L.q8_row_bytes(cols), dtype=torch.uint8, device="cuda")
    packed[:, :2 * G] = torch.from_numpy(s).cuda().view(torch.uint8)
    packed[:, sb:] = w.view(torch.uint8)
    x8 = rng.integers(-127, 128, cols, dtype=np.int8)
    dt = ops.DeviceTensor.from_packed(packed.reshape(-1), rows, cols, L.KIND_Q8, B, R)
    y = ops.matvec_q8(ctx, dt, torch.from_numpy(x8).cuda()).cpu().numpy()
    ctx.raise_on_error()
    pick = np.sort(rng.choice(rows, 64, replace=False))
    pick[-1] = rows - 1
    wp = w[torch.from_numpy(pick).cuda()].cpu().numpy()
    assert np.array_equal(y[pick], ref.matvec_q8(s[pick], wp, x8, B, R))


@pytest.mark.parametrize("rows,cols,xscale", [(96, 1024, 1.0), (257, 4160, 30.0), (33, 32, 1e-3), (16, 512, 0.0)])
def test_q8_float_projection(ctx, rows, cols, xscale):
    """trx_matvec_q8_f: quantise x (power of two), the Q8 row dot, scale by 2^(e8+R-B); equal in
    every fp32 bit to the oracle's restatement of model/mirror.py:664-678."""
    rng = np.random.default_rng(rows + cols)
    s, w = random_q8(rng, rows, cols)
    t = image.Q8Tensor(s, w)
    x = (rng.standard_normal(cols) * xscale).astype(np.float32)
    y = ops.matvec_q8_f(ctx, ops.DeviceTensor(t), torch.from_numpy(x).cuda()).cpu().numpy()
    ctx.raise_on_error()
    want = ref.matvec_q8_f(s, w, x, t.bias, t.rshift)
    assert np.array_equal(y.view(np.uint32), want.view(np.uint32))
