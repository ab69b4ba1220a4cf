"""LM head + greedy token (trx_lmhead_argmax, through the C ABI) against the C oracle's float
projection (bit-exact logits) and the reference's argmax rule: first maximum, ties to the
smallest row (model/mirror.py:1033; doc/units.md:149).
"""
import numpy as np
import pytest
import torch

from oracle import ref
from oracle import build as cor
from trixium_b200 import image, layout as L

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops():
    from trixium_b200 import ops as o
    return o


@pytest.fixture(scope="module")
def ctx(ops):
    c = ops.Context(0)
    yield c
    c.close()


def head(ops, rows, cols, kind, seed):
    gen = torch.Generator(device="cuda")
    gen.manual_seed(seed)
    codes, scales = image.synthetic_codes_scales_torch(gen, rows, cols, "cuda")
    W = image.pack_rows_torch(scales, codes, kind)
    B = image.scale_bias(np.array([float(scales.float().abs().max())], dtype=np.float16))
    R = image.result_shift(scales.cpu().numpy(), B)
    return ops.DeviceTensor.from_packed(W, rows, cols, kind, B, R), W, B, R


def oracle_logits(W, rows, cols, kind, B, R, x):
    y, bad = cor.matvec_f(W.cpu().numpy(), rows, cols, kind, B, R, x)
    assert bad == 0
    return y


@pytest.mark.parametrize("kind", [L.KIND_TERNARY5, L.KIND_TERNARY])
def test_lmhead_full_vocab(ops, ctx, kind):
    """Vocabulary 151,936 x hidden 2048 (configs 1 and 3), with the final RMSNorm fused."""
    rows, cols = 151936, 2048
    w, W, B, R = head(ops, rows, cols, kind, seed=21 + kind)
    rng = np.random.default_rng(5)
    x = rng.standard_normal(cols).astype(np.float32)
    nw = (1 + 0.1 * rng.standard_normal(cols)).astype(np.float32)
    logits = torch.empty(rows, device="cuda")
    tok = ops.lmhead_argmax(ctx, w, torch.from_numpy(x).cuda(), logits=logits, norm_w=torch.from_numpy(nw).cuda(),
                            eps=1e-6)
    assert ctx.errors() == 0
    want = oracle_logits(W, rows, cols, kind, B, R, ref.rmsnorm(x, nw, 1e-6))
    assert np.array_equal(logits.cpu().numpy().view(np.uint32), want.view(np.uint32))
    assert int(tok.item()) == ref.argmax_first(want)


def test_lmhead_ties_and_reuse(ops, ctx):
    """A copy of the maximal row placed earlier wins; the keys clean themselves between calls."""
    rows, cols, kind = 3000, 512, L.KIND_TERNARY5
    w, W, B, R = head(ops, rows, cols, kind, seed=31)
    rb = L.row_bytes(cols, kind)
    x = np.random.default_rng(6).standard_normal(cols).astype(np.float32)
    want = oracle_logits(W, rows, cols, kind, B, R, x)
    top = ref.argmax_first(want)
    dup = 7 if top != 7 else 8
    W[dup * rb:(dup + 1) * rb] = W[top * rb:(top + 1) * rb].clone()
    xt = torch.from_numpy(x).cuda()
    for _ in range(3):
        tok = ops.lmhead_argmax(ctx, w, xt)
        assert int(tok.item()) == min(dup, top)
    y = np.random.default_rng(7).standard_normal(cols).astype(np.float32)
    tok = ops.lmhead_argmax(ctx, w, torch.from_numpy(y).cuda())
    assert int(tok.item()) == ref.argmax_first(oracle_logits(W, rows, cols, kind, B, R, y))
    assert ctx.errors() == 0


def test_lmhead_in_cuda_graph(ops, ctx):
    rows, cols, kind = 20000, 1024, L.KIND_TERNARY
    w, W, B, R = head(ops, rows, cols, kind, seed=41)
    x = torch.empty(cols, device="cuda")
    tok = torch.empty(1, dtype=torch.int32, device="cuda")
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        x.zero_()
        ops.lmhead_argmax(ctx, w, x, token=tok)
        torch.cuda.synchronize()
        with torch.cuda.graph(g, stream=s):
            ops.lmhead_argmax(ctx, w, x, token=tok)
    torch.cuda.synchronize()
    rng = np.random.default_rng(8)
    for _ in range(5):
        xv = rng.standard_normal(cols).astype(np.float32)
        x.copy_(torch.from_numpy(xv))
        g.replay()
        torch.cuda.synchronize()
        assert int(tok.item()) == ref.argmax_first(oracle_logits(W, rows, cols, kind, B, R, xv))
    assert ctx.errors() == 0
