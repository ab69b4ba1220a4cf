"""The batched rows on the tensor cores (tcgen05 kind::i8; trx_matvec_i8_rows with 9..32 rows and
trx_matvec_f_rows), through the C ABI, against the oracle per row (model/bitexact.py:121-125: each
row is matvec_ternary) and the reference-made golden vectors (row 0 of every batch is the fixture's
own activation): int32 results bit-exact; float results fp32-bit-exact with each row quantised with
its own exponent (model/mirror.py:45-51, :664-678).  Shapes cover ragged group counts (a last chunk
of fewer than four groups, odd group counts), row counts that are not a multiple of the 128-row
tile, K splits over several CTAs, and both code kinds."""
import os

import numpy as np
import pytest
import torch

from oracle import ref
from trixium_b200 import layout as L
from conftest import GOLDEN, load

pytestmark = pytest.mark.gpu

KINDS = [L.KIND_TERNARY5, L.KIND_TERNARY]
FIXTURES = ["bench_48x2048", "bench_33x640", "bench_7x128", "bench_64x4096", "bench_20x2944", "bench_16x6144",
            "bench_3x17408", "refacc_64x512", "signed_24x1024"]


@pytest.fixture(scope="module")
def ops():
    from trixium_b200 import ops as o
    return o


@pytest.fixture(scope="module")
def ctx(ops):
    c = ops.Context(0)
    yield c
    c.close()


def _tensor(ops, d, kind):
    return ops.DeviceTensor.from_packed(d[f"packed_k{kind}"], int(d["rows"]), int(d["cols"]), kind, int(d["B"]),
                                        int(d["R"]))


@pytest.mark.parametrize("nb", [9, 16, 17, 32])
@pytest.mark.parametrize("kind", KINDS)
@pytest.mark.parametrize("name", FIXTURES)
def test_int_rows_on_tensor_cores_bit_exact(ops, ctx, name, kind, nb):
    d = load(os.path.join(GOLDEN, f"matvec_{name}.npz"))
    K = int(d["cols"])
    rng = np.random.default_rng(nb + K)
    x8 = rng.integers(-127, 128, (nb, K), dtype=np.int8)
    x8[0] = d["x8"]
    y = ops.matvec_i8_rows(ctx, _tensor(ops, d, kind), torch.from_numpy(x8).cuda()).cpu().numpy()
    assert np.array_equal(y[0], d["y_int"])
    for i in range(1, nb):
        assert np.array_equal(y[i], ref.matvec_int(d["scales"], d["codes"], x8[i], int(d["B"]), int(d["R"]))), i
    assert ctx.errors() == 0


@pytest.mark.parametrize("nb", [1, 5, 16, 32])
@pytest.mark.parametrize("kind", KINDS)
@pytest.mark.parametrize("name", ["bench_48x2048", "bench_64x4096", "bench_20x2944", "bench_3x17408"])
def test_float_rows_bit_exact(ops, ctx, name, kind, nb):
    d = load(os.path.join(GOLDEN, f"matvec_{name}.npz"))
    K = int(d["cols"])
    rng = np.random.default_rng(3 * nb + K)
    x = (rng.standard_normal((nb, K)) * rng.uniform(0.1, 10, (nb, 1))).astype(np.float32)
    x[0] = d["x"]
    y = ops.matvec_f_rows(ctx, _tensor(ops, d, kind), torch.from_numpy(x).cuda()).cpu().numpy()
    assert np.array_equal(y[0].view(np.uint32), d["y_f"].view(np.uint32))
    for i in range(nb):
        want = ref.matvec_f(d["scales"], d["codes"], x[i], int(d["B"]), int(d["R"]))
        assert np.array_equal(y[i].view(np.uint32), want.view(np.uint32)), i
    assert ctx.errors() == 0


@pytest.mark.parametrize("kind", KINDS)
def test_rows_large_tile_count_and_k_split(ops, ctx, kind):
    """6144 x 2048 (48 row tiles: split over K) and 20000 x 1024 (157 tiles: no split), 32 rows."""
    from trixium_b200 import image
    for rows, cols in ((6144, 2048), (20000, 1024)):
        t, x = image.synthetic_matvec_case(rows, cols, seed=rows, kind=kind)
        w = ops.DeviceTensor(t)
        rng = np.random.default_rng(rows)
        x8 = rng.integers(-127, 128, (32, cols), dtype=np.int8)
        y = ops.matvec_i8_rows(ctx, w, torch.from_numpy(x8).cuda()).cpu().numpy()
        for i in (0, 7, 31):
            assert np.array_equal(y[i], ref.matvec_int(t.scales, t.codes, x8[i], t.bias, t.rshift)), (rows, i)
        # Twice in a row: the K-split scratch and counts are left at zero by each launch.
        y2 = ops.matvec_i8_rows(ctx, w, torch.from_numpy(x8).cuda()).cpu().numpy()
        assert np.array_equal(y, y2)
    assert ctx.errors() == 0


@pytest.mark.parametrize("kind", KINDS)
def test_rows_multi_segments_with_norm(ops, ctx, kind):
    """trx_matvec_f_rows_multi (three tensors back to back, 128-row-aligned and not, the RMSNorm in
    front, a residual on one) equals the row-wise norm followed by one batched launch per tensor,
    bit for bit."""
    from trixium_b200 import decoder as D, layout as L
    gen = torch.Generator(device="cuda").manual_seed(9)
    K = 1024
    p = D.Packed(gen, [("a", 384), ("b", 200), ("c", 130)], K, kind, "cuda")
    nb = 12
    x = torch.randn(nb, K, generator=gen, device="cuda")
    nw = (1 + 0.1 * torch.randn(K, generator=gen, device="cuda")).contiguous()
    ys = [torch.empty(nb, e.rows, device="cuda") for e in p.entries]
    rs = [None, torch.randn(nb, 200, generator=gen, device="cuda"), None]
    ops.matvec_f_rows_multi(ctx, p.entries, p.data, x, ys, norm_w=nw, eps=1e-6, resids=rs)
    h = ops.rmsnorm_rows(ctx, x, nw, 1e-6)
    for i in range(3):
        want = ops.matvec_f_rows(ctx, p.tensor(i), h, resid=rs[i])
        assert torch.equal(ys[i].view(torch.int32), want.view(torch.int32)), i
    assert ctx.errors() == 0


@pytest.mark.parametrize("nb", [3, 16, 32])
@pytest.mark.parametrize("kind", KINDS)
def test_rows_k_segments_bit_exact(ops, ctx, kind, nb):
    """trx_matvec_f_rows_kseg (two K-segments of 8704 columns, one exponent per row over both,
    a residual) equals trx_matvec_f_kseg on each row, bit for bit."""
    from trixium_b200 import decoder as D
    gen = torch.Generator(device="cuda").manual_seed(21)
    segs = D.ksegmented(gen, 300, 17408, kind, "cuda")
    assert len(segs) == 2
    x = torch.randn(nb, 17408, generator=gen, device="cuda")
    r = torch.randn(nb, 300, generator=gen, device="cuda")
    y = ops.matvec_f_rows_kseg(ctx, segs, x, resid=r)
    for b in range(nb):
        want = ops.matvec_f_kseg(ctx, segs, x[b].contiguous(), resid=r[b].contiguous())
        assert torch.equal(y[b].view(torch.int32), want.view(torch.int32)), b
    assert ctx.errors() == 0
