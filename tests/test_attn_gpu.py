"""Parity of the decode-attention kernel (trx_attn_decode, through the C ABI) with the oracle's
restatement of model/mirror.py:945-996 with an fp16 KV cache.

Float outputs: within 1e-3 relative (denominator floored at 1% of the reference RMS).  The cache
rows the kernel writes (RMSNorm'd, RoPE'd k; v) match the oracle's fp16 rounding to 1 fp16 ulp.
"""
import numpy as np
import pytest
import torch

from oracle import ref
from conftest import fp_rel_err

pytestmark = pytest.mark.gpu

TOL = 1e-3

# (H, Hkv, hd, rope_dims, gated, max_pos): configs 1/2 (16/8 and 32/8 x 128, full RoPE) and the
# hybrids (16/4 and 24/4 x 256, partial RoPE over 64 dims, gated), plus MHA and a tiny case.
SHAPES = [
    (16, 8, 128, 128, False, 640),
    (32, 8, 128, 128, False, 1280),
    (16, 4, 256, 64, True, 2304),
    (24, 4, 256, 64, True, 4352),
    (4, 4, 64, 32, False, 96),
    (2, 1, 8, 8, False, 16),
]


@pytest.fixture(scope="module")
def ops():
    from trixium_b200 import ops as o
    return o


@pytest.fixture(scope="module")
def ctx(ops):
    c = ops.Context(0)
    yield c
    c.close()


class Case:
    def __init__(self, ops, H, Hkv, hd, rope, gated, max_pos, seed):
        self.rng = np.random.default_rng(seed)
        self.H, self.Hkv, self.hd, self.gated = H, Hkv, hd, gated
        self.shape = ops.attn_shape(H, Hkv, hd, max_pos, rope_dims=rope, gated=gated, eps=1e-6)
        self.qn = (1 + 0.1 * self.rng.standard_normal(hd)).astype(np.float32)
        self.kn = (1 + 0.1 * self.rng.standard_normal(hd)).astype(np.float32)
        self.freq = ref.rope_freq(rope, 1e6) if rope else np.zeros(0, np.float32)
        self.kc = np.zeros((max_pos, Hkv, hd), np.float16)
        self.vc = np.zeros((max_pos, Hkv, hd), np.float16)
        self.dkc = torch.zeros(max_pos, Hkv, hd, dtype=torch.float16, device="cuda")
        self.dvc = torch.zeros_like(self.dkc)
        self.dqn = torch.from_numpy(self.qn).cuda()
        self.dkn = torch.from_numpy(self.kn).cuda()
        self.dfreq = torch.from_numpy(self.freq).cuda() if rope else None
        self.dpos = torch.zeros(1, dtype=torch.int32, device="cuda")

    def prefill(self, n):
        """Fill positions [0, n) with random cache rows, identically on both sides."""
        k = (self.rng.standard_normal((n, self.Hkv, self.hd)) * 0.5).astype(np.float16)
        v = self.rng.standard_normal((n, self.Hkv, self.hd)).astype(np.float16)
        self.kc[:n], self.vc[:n] = k, v
        self.dkc[:n] = torch.from_numpy(k).cuda()
        self.dvc[:n] = torch.from_numpy(v).cuda()

    def step(self, ops, ctx, pos):
        """One step on both sides.  The new cache row is checked against the oracle's (1 fp16 ulp
        on k: cos/sin of the same fp32 angle may differ in the last bit between libraries; v
        exact); the oracle then attends over the kernel's own row, so the output comparison sees
        the attention arithmetic only."""
        H, Hkv, hd = self.H, self.Hkv, self.hd
        qf = self.rng.standard_normal((H, (2 if self.gated else 1) * hd)).astype(np.float32)
        k = self.rng.standard_normal((Hkv, hd)).astype(np.float32)
        v = self.rng.standard_normal((Hkv, hd)).astype(np.float32)
        q, gate = (qf[:, :hd], qf[:, hd:]) if self.gated else (qf, None)
        self.dpos.fill_(pos)
        got = self.run(ops, ctx, qf, k, v)
        assert ctx.errors() == 0
        krow, vrow = ref.attn_new_rows(k, v, pos, self.kn, 1e-6, self.freq)
        gk, gv = self.dkc[pos].cpu().numpy(), self.dvc[pos].cpu().numpy()
        check_row(gk, gv, krow, vrow)
        want = ref.attn_decode(q, k, v, self.kc, self.vc, pos, self.qn, self.kn, 1e-6, self.freq, gate=gate,
                               rows=(gk, gv))
        return got.reshape(H, hd), want

    def run(self, ops, ctx, qf, k, v):
        return ops.attn_decode(ctx, self.shape, torch.from_numpy(qf.reshape(-1)).cuda(),
                               torch.from_numpy(k.reshape(-1)).cuda(), torch.from_numpy(v.reshape(-1)).cuda(),
                               self.dqn, self.dkn, self.dfreq, self.dkc, self.dvc, self.dpos).cpu().numpy()


def check_row(gk, gv, krow, vrow):
    assert np.array_equal(gv, vrow)
    want = krow.astype(np.float32)
    ulp = np.spacing(np.abs(krow)).astype(np.float32)
    assert np.all(np.abs(gk.astype(np.float32) - want) <= ulp)


@pytest.mark.parametrize("shape", SHAPES, ids=[f"{s[0]}x{s[1]}x{s[2]}r{s[3]}{'g' if s[4] else ''}" for s in SHAPES])
def test_attn_steps_from_empty(ops, ctx, shape):
    """Positions 0..n: the first steps, the chunk boundary at 64, cache appends."""
    H, Hkv, hd, rope, gated, max_pos = shape
    case = Case(ops, H, Hkv, hd, rope, gated, max_pos, seed=1)
    last = min(max_pos, 70)
    for pos in range(last):
        got, want = case.step(ops, ctx, pos)
        assert fp_rel_err(got, want) < TOL, pos


@pytest.mark.parametrize("shape", SHAPES[:4], ids=[f"{s[0]}x{s[1]}x{s[2]}" for s in SHAPES[:4]])
def test_attn_long_context(ops, ctx, shape):
    """A prefilled cache: many chunks, the last position of the cache."""
    H, Hkv, hd, rope, gated, max_pos = shape
    case = Case(ops, H, Hkv, hd, rope, gated, max_pos, seed=2)
    for pos in (max_pos // 2 + 3, max_pos - 1):
        case.prefill(pos)
        got, want = case.step(ops, ctx, pos)
        assert fp_rel_err(got, want) < TOL, pos


def test_attn_position_out_of_range(ops, ctx):
    from trixium_b200 import _lib
    case = Case(ops, 4, 2, 64, 64, False, 32, seed=3)
    case.dpos.fill_(32)
    q = torch.zeros(4 * 64, device="cuda")
    kv = torch.zeros(2 * 64, device="cuda")
    ops.attn_decode(ctx, case.shape, q, kv, kv, case.dqn, case.dkn, case.dfreq, case.dkc, case.dvc, case.dpos)
    assert ctx.errors() == _lib.DEV_RANGE
    assert float(case.dkc.abs().sum()) == 0.0


def test_attn_in_cuda_graph(ops, ctx):
    """The position is read on the device: one captured step replays at successive positions."""
    H, Hkv, hd = 8, 2, 128
    case = Case(ops, H, Hkv, hd, 128, False, 256, seed=4)
    q = torch.empty(H * hd, device="cuda")
    k = torch.empty(Hkv * hd, device="cuda")
    v = torch.empty(Hkv * hd, device="cuda")
    out = torch.empty(H * hd, device="cuda")
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        ops.attn_decode(ctx, case.shape, q, k, v, case.dqn, case.dkn, case.dfreq, case.dkc, case.dvc, case.dpos, out)
        torch.cuda.synchronize()
        with torch.cuda.graph(g, stream=s):
            ops.attn_decode(ctx, case.shape, q, k, v, case.dqn, case.dkn, case.dfreq, case.dkc, case.dvc,
                            case.dpos, out)
    torch.cuda.synchronize()
    for pos in range(0, 100):
        qn = case.rng.standard_normal((H, hd)).astype(np.float32)
        kn = case.rng.standard_normal((Hkv, hd)).astype(np.float32)
        vn = case.rng.standard_normal((Hkv, hd)).astype(np.float32)
        q.copy_(torch.from_numpy(qn.reshape(-1)))
        k.copy_(torch.from_numpy(kn.reshape(-1)))
        v.copy_(torch.from_numpy(vn.reshape(-1)))
        case.dpos.fill_(pos)
        g.replay()
        torch.cuda.synchronize()
        krow, vrow = ref.attn_new_rows(kn, vn, pos, case.kn, 1e-6, case.freq)
        gk, gv = case.dkc[pos].cpu().numpy(), case.dvc[pos].cpu().numpy()
        check_row(gk, gv, krow, vrow)
        want = ref.attn_decode(qn, kn, vn, case.kc, case.vc, pos, case.qn, case.kn, 1e-6, case.freq, rows=(gk, gv))
        assert fp_rel_err(out.cpu().numpy().reshape(H, hd), want) < TOL, pos
    assert ctx.errors() == 0
