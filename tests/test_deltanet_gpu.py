"""Parity of the gated-DeltaNet step kernel (trx_deltanet_step, through the C ABI) with the oracle's
restatement of model/mirror.py:892-943 (mathematical profile).

Float outputs and the updated recurrent state: within 1e-3 relative (denominator floored at 1%
of the reference RMS).  The conv ring holds the raw qkv inputs: exact.
"""
import numpy as np
import pytest
import torch

from oracle import ref
from conftest import fp_rel_err

pytestmark = pytest.mark.gpu

TOL = 1e-3

# (nk, hk, nv, hv, K): config 3 (16 heads, dim 128), config 4 (48 value heads on 16 key heads),
# and smaller geometries.
SHAPES = [
    (16, 128, 16, 128, 4),
    (16, 128, 48, 128, 4),
    (4, 64, 8, 64, 4),
    (2, 32, 4, 32, 3),
    (1, 256, 2, 96, 2),
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


class Layer:
    def __init__(self, ops, nk, hk, nv, hv, K, seed):
        rng = self.rng = np.random.default_rng(seed)
        self.nk, self.hk, self.nv, self.hv, self.K = nk, hk, nv, hv, K
        self.C = 2 * nk * hk + nv * hv
        self.shape = ops.deltanet_shape(nk, hk, nv, hv, K, 1e-6)
        self.dt_bias = rng.uniform(-1, 1, nv).astype(np.float32)
        self.ssm_a = (-np.exp(rng.uniform(0, 2, nv))).astype(np.float32)
        self.conv_w = (rng.standard_normal((self.C, K)) / np.sqrt(K)).astype(np.float32)
        self.norm_w = (1 + 0.1 * rng.standard_normal(hv)).astype(np.float32)
        self.win = np.zeros((K - 1, self.C), np.float32)
        self.S = (rng.standard_normal((nv, hv, hk)) / np.sqrt(hk)).astype(np.float32)
        d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
        self.d = {k: d(getattr(self, k)) for k in ("dt_bias", "ssm_a", "conv_w", "norm_w")}
        self.ring = torch.zeros(K, self.C, device="cuda")
        self.dS = d(self.S.copy())
        self.dpos = torch.zeros(1, dtype=torch.int32, device="cuda")

    def inputs(self):
        r = self.rng
        return (r.standard_normal(self.C).astype(np.float32), r.standard_normal(self.nv * self.hv).astype(np.float32),
                r.standard_normal(self.nv).astype(np.float32), r.standard_normal(self.nv).astype(np.float32))

    def oracle(self, qkv, z, beta, alpha):
        return ref.deltanet_step(qkv, z, beta, alpha, self.dt_bias, self.ssm_a, self.conv_w, self.win, self.S,
                                 self.norm_w, 1e-6, self.nk, self.hk, self.nv, self.hv)

    def kernel(self, ops, ctx, qkv, z, beta, alpha, out=None):
        d = lambda a: torch.from_numpy(a).cuda()
        return ops.deltanet_step(ctx, self.shape, d(qkv), d(z), d(beta), d(alpha), self.d["dt_bias"], self.d["ssm_a"],
                                 self.d["conv_w"], self.d["norm_w"], self.ring, self.dS, self.dpos, out)

    def ring_window(self, pos):
        """The kernel's ring, as the oracle's window after step pos (oldest first)."""
        ring = self.ring.cpu().numpy()
        return np.stack([ring[(pos + 1 + i + 1) % self.K] for i in range(self.K - 1)])


@pytest.mark.parametrize("shape", SHAPES, ids=[f"nk{s[0]}hk{s[1]}nv{s[2]}hv{s[3]}K{s[4]}" for s in SHAPES])
def test_deltanet_steps(ops, ctx, shape):
    layer = Layer(ops, *shape, seed=11)
    for pos in range(7):
        qkv, z, beta, alpha = layer.inputs()
        layer.dpos.fill_(pos)
        got = layer.kernel(ops, ctx, qkv, z, beta, alpha).cpu().numpy()
        assert ctx.errors() == 0
        want = layer.oracle(qkv, z, beta, alpha)
        assert fp_rel_err(got, want) < TOL, pos
        assert fp_rel_err(layer.dS.cpu().numpy(), layer.S) < TOL, pos
        assert np.array_equal(layer.ring_window(pos), layer.win), pos


def test_deltanet_negative_position(ops, ctx):
    from trixium_b200 import _lib
    layer = Layer(ops, 2, 32, 4, 32, 4, seed=12)
    layer.dpos.fill_(-1)
    before = layer.dS.clone()
    layer.kernel(ops, ctx, *layer.inputs())
    assert ctx.errors() == _lib.DEV_RANGE
    assert torch.equal(before, layer.dS)


def test_deltanet_in_cuda_graph(ops, ctx):
    """The position is read on the device: one captured step replays at successive positions."""
    layer = Layer(ops, 4, 128, 8, 128, 4, seed=13)
    qkv = torch.zeros(layer.C, device="cuda")
    z = torch.zeros(layer.nv * layer.hv, device="cuda")
    beta = torch.zeros(layer.nv, device="cuda")
    alpha = torch.zeros(layer.nv, device="cuda")
    out = torch.empty(layer.nv * layer.hv, device="cuda")
    args = lambda: (ctx, layer.shape, qkv, z, beta, alpha, layer.d["dt_bias"], layer.d["ssm_a"], layer.d["conv_w"],
                    layer.d["norm_w"], layer.ring, layer.dS, layer.dpos, out)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    S0, ring0 = layer.dS.clone(), layer.ring.clone()
    with torch.cuda.stream(s):
        ops.deltanet_step(*args())   # warm-up outside the capture, then restore the state
        torch.cuda.synchronize()
        with torch.cuda.graph(g, stream=s):
            ops.deltanet_step(*args())
    torch.cuda.synchronize()
    layer.dS.copy_(S0)
    layer.ring.copy_(ring0)
    for pos in range(12):
        a = layer.inputs()
        for t, v in zip((qkv, z, beta, alpha), a):
            t.copy_(torch.from_numpy(v))
        layer.dpos.fill_(pos)
        g.replay()
        torch.cuda.synchronize()
        want = layer.oracle(*a)
        assert fp_rel_err(out.cpu().numpy(), want) < TOL, pos
    assert ctx.errors() == 0
