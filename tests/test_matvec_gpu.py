"""Parity of the B200 matvec kernels (through the C ABI) with the reference's golden vectors and
the oracle.  Integer results and the engine-arithmetic float projection are bit-exact; the fp
mode is within 1e-3 relative (denominator floored at 1% of the reference RMS).
"""
import os

import numpy as np
import pytest
import torch

from oracle import ref
from oracle import build as cor
from trixium_b200 import image, layout as L

from conftest import GOLDEN, golden_matvec_files, load, fp_rel_err

pytestmark = pytest.mark.gpu

FILES = golden_matvec_files()
IDS = [os.path.basename(f)[7:-4] for f in FILES]
KINDS = [L.KIND_TERNARY, L.KIND_TERNARY5]


@pytest.fixture(scope="module")
def ops():
    from trixium_b200 import ops as o
    return o


@pytest.fixture(scope="module")
def ctx(ops):
    c = ops.Context(0)
    yield c
    c.close()


def dev(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a))
    return t.to("cuda") if dtype is None else t.to("cuda", dtype)


def device_tensor(ops, d, kind):
    return ops.DeviceTensor.from_packed(d[f"packed_k{kind}"], int(d["rows"]), int(d["cols"]), kind,
                                        int(d["B"]), int(d["R"]))


@pytest.mark.parametrize("path", FILES, ids=IDS)
@pytest.mark.parametrize("kind", KINDS)
def test_int_matvec_golden(ops, ctx, path, kind):
    d = load(path)
    w = device_tensor(ops, d, kind)
    y = ops.matvec_i8(ctx, w, dev(d["x8"]))
    assert ctx.errors() == 0
    assert np.array_equal(y.cpu().numpy(), d["y_int"])


@pytest.mark.parametrize("path", [f for f in FILES if "x" in np.load(f)],
                         ids=[i for f, i in zip(FILES, IDS) if "x" in np.load(f)])
@pytest.mark.parametrize("kind", KINDS)
def test_float_projection_golden(ops, ctx, path, kind):
    d = load(path)
    w = device_tensor(ops, d, kind)
    y = ops.matvec_f(ctx, w, dev(d["x"]))
    assert ctx.errors() == 0
    assert np.array_equal(y.cpu().numpy().view(np.uint32), d["y_f"].view(np.uint32))
    yfp = ops.matvec_fp(ctx, w, dev(d["x"])).cpu().numpy()
    if np.any(d["y_f64"]):
        assert fp_rel_err(yfp, d["y_f64"]) < 1e-3
    else:
        assert np.all(yfp == 0)


def test_quantize_golden(ops, ctx):
    q = load(os.path.join(GOLDEN, "quantize.npz"))
    for x, x8, e8 in zip(q["x"], q["x8"], q["e8"]):
        a, b = ops.quantize_pow2(ctx, dev(x))
        assert np.array_equal(a.cpu().numpy(), x8) and int(b.item()) == int(e8)


@pytest.mark.parametrize("kind", KINDS)
@pytest.mark.parametrize("rows,cols", [(6144, 2048), (1024, 4096), (300, 5120), (257, 6144), (96, 12288),
                                       (40, 17408), (5, 128), (1, 256), (77, 384)])
def test_against_oracle_shapes(ops, ctx, kind, rows, cols):
    t, x = image.synthetic_matvec_case(rows, cols, seed=rows * 7 + cols, kind=kind)
    w = ops.DeviceTensor(t)
    y = ops.matvec_f(ctx, w, dev(x)).cpu().numpy()
    assert ctx.errors() == 0
    yo, bad = cor.matvec_f(t.packed, rows, cols, kind, t.bias, t.rshift, x)
    assert bad == 0
    assert np.array_equal(y.view(np.uint32), yo.view(np.uint32))
    x8, _ = ref.quantize_pow2(x)
    yi = ops.matvec_i8(ctx, w, dev(x8)).cpu().numpy()
    yio, _ = cor.matvec_int(t.packed, rows, cols, kind, x8, t.bias, t.rshift)
    assert np.array_equal(yi, yio)


@pytest.mark.parametrize("kind", KINDS)
def test_rmsnorm_prologue_and_residual(ops, ctx, kind):
    rows, cols = 512, 2048
    t, x = image.synthetic_matvec_case(rows, cols, seed=3, kind=kind)
    rng = np.random.default_rng(9)
    nw = rng.uniform(0.8, 1.2, cols).astype(np.float32)
    resid = rng.standard_normal(rows).astype(np.float32)
    eps = 1e-6
    w = ops.DeviceTensor(t)
    y = ops.matvec_f(ctx, w, dev(x), norm_w=dev(nw), eps=eps, resid=dev(resid)).cpu().numpy()
    assert ctx.errors() == 0
    xn = ref.rmsnorm(x, nw, eps)
    s, c = ref.decode_packed(t.packed, rows, cols, kind)
    expect = (resid + ref.matvec_f(s, c, xn, t.bias, t.rshift)).astype(np.float32)
    assert np.array_equal(y.view(np.uint32), expect.view(np.uint32))


@pytest.mark.parametrize("kind", KINDS)
def test_swiglu_epilogue(ops, ctx, kind):
    rows, cols = 768, 1024
    rng = np.random.default_rng(21)
    cg, sg = image.synthetic_codes_scales(rng, rows, cols)
    cu, su = image.synthetic_codes_scales(rng, rows, cols)
    x = rng.standard_normal(cols).astype(np.float32)
    nw = rng.uniform(0.8, 1.2, cols).astype(np.float32)
    tg, tu = image.TernaryTensor(sg, cg, kind), image.TernaryTensor(su, cu, kind)
    act = ops.matvec_swiglu(ctx, ops.DeviceTensor(tg), ops.DeviceTensor(tu), dev(x), norm_w=dev(nw),
                            eps=1e-6).cpu().numpy()
    assert ctx.errors() == 0
    xn = ref.rmsnorm(x, nw, 1e-6)
    g = ref.matvec_f(sg, cg, xn, tg.bias, tg.rshift)
    u = ref.matvec_f(su, cu, xn, tu.bias, tu.rshift)
    expect = (ref.silu(g) * u).astype(np.float32)
    assert fp_rel_err(act, expect) < 1e-5


@pytest.mark.parametrize("kind", KINDS)
def test_batch_equals_single(ops, ctx, kind):
    rows, cols, nj = 384, 2048, 5
    rng = np.random.default_rng(5)
    ts, xs = [], []
    for j in range(nj):
        c, s = image.synthetic_codes_scales(rng, rows, cols)
        ts.append(image.TernaryTensor(s, c, kind, bias=None, rshift=None))
        xs.append(rng.standard_normal(cols).astype(np.float32))
    # One shared B/R so a single entry describes every copy.
    B, R = ts[0].bias, max(t.rshift for t in ts)
    ts = [image.TernaryTensor(t.scales, t.codes, kind, bias=B, rshift=R) for t in ts]
    packed = np.concatenate([t.packed for t in ts])
    w = ops.DeviceTensor.from_packed(packed, rows, cols, kind, B, R)
    X = dev(np.stack(xs))
    Y = torch.empty(nj, rows, dtype=torch.float32, device="cuda")
    ops.matvec_f_batch(ctx, w, ts[0].packed.size, X, cols, Y, rows, nj)
    assert ctx.errors() == 0
    for j in range(nj):
        yo, _ = cor.matvec_f(ts[j].packed, rows, cols, kind, B, R, xs[j])
        assert np.array_equal(Y[j].cpu().numpy().view(np.uint32), yo.view(np.uint32))


@pytest.mark.parametrize("kind", KINDS)
def test_multirow_equals_rows(ops, ctx, kind):
    d = load(os.path.join(GOLDEN, "matvec_bench_48x2048.npz"))
    rng = np.random.default_rng(1)
    x8 = rng.integers(-127, 128, (5, 2048), dtype=np.int8)
    w = device_tensor(ops, d, kind)
    y = ops.matvec_i8_rows(ctx, w, dev(x8)).cpu().numpy()
    for i in range(5):
        assert np.array_equal(y[i], ref.matvec_int(d["scales"], d["codes"], x8[i], int(d["B"]), int(d["R"])))


def test_overflow_is_reported_not_fatal(ops, ctx):
    d = load(os.path.join(GOLDEN, "matvec_refbound_16x12288.npz"))
    w = ops.DeviceTensor.from_packed(d["packed_k5"], 16, 12288, 5, int(d["B"]), 0)  # R = 0 overflows
    ops.matvec_i8(ctx, w, dev(d["x8"]))
    bits = ctx.errors()
    assert bits & 0x1
    assert ctx.errors() == 0   # cleared, context still usable
    y = ops.matvec_i8(ctx, device_tensor(ops, d, 5), dev(d["x8"]))
    assert np.array_equal(y.cpu().numpy(), d["y_int"]) and ctx.errors() == 0


def test_invalid_trit5_byte_flagged(ops, ctx):
    d = load(os.path.join(GOLDEN, "matvec_bench_7x128.npz"))
    packed = d["packed_k5"].copy()
    w = device_tensor(ops, d, 5)
    ops.validate_packed(ctx, w)
    assert ctx.errors() == 0
    packed[L.scale_bytes(128) + 3] = 250
    ops.validate_packed(ctx, ops.DeviceTensor.from_packed(packed, 7, 128, 5, int(d["B"]), int(d["R"])))
    assert ctx.errors() & 0x2


def test_host_argument_checks(ops, ctx):
    from trixium_b200 import _lib
    d = load(os.path.join(GOLDEN, "matvec_bench_7x128.npz"))
    with pytest.raises(_lib.TrxError):
        bad = ops.DeviceTensor.from_packed(d["packed_k5"], 7, 100, 5, int(d["B"]), int(d["R"]))
        ops.matvec_i8(ctx, bad, dev(d["x8"]))
    with pytest.raises(_lib.TrxError):
        bad = ops.DeviceTensor.from_packed(d["packed_k5"], 7, 128, 3, int(d["B"]), int(d["R"]))
        ops.matvec_i8(ctx, bad, dev(d["x8"]))


def test_dropin_reference_surface():
    from trixium_b200 import bitexact as bx
    d = load(os.path.join(GOLDEN, "matvec_refacc_64x512.npz"))
    y = bx.matvec_ternary(d["scales"], d["codes"], d["x8"], int(d["B"]), int(d["R"]))
    assert y.dtype == np.int32 and np.array_equal(y, d["y_int"])
    y5 = bx.matvec_ternary(d["scales"], d["codes"], d["x8"], int(d["B"]), int(d["R"]), kind=5)
    assert np.array_equal(y5, d["y_int"])
    rows = bx.matvec_ternary_rows(d["scales"], d["codes"], np.stack([d["x8"], -d["x8"]]), int(d["B"]), int(d["R"]))
    assert rows.shape == (2, 64) and np.array_equal(rows[0], d["y_int"])
    with pytest.raises(AssertionError):
        b = load(os.path.join(GOLDEN, "matvec_refbound_16x12288.npz"))
        bx.matvec_ternary(b["scales"], b["codes"], b["x8"], int(b["B"]), 0)
