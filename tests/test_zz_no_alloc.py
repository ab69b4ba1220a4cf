"""The context-free decode attention (trx_attn_decode_static) against the context entry point
(trx_attn_decode), for callers that must not allocate device memory while they run: two calls in a
row on identical inputs and separate caches.  The static entry runs the scratch-merge kernel on the
library's static arrays, the context entry the tensor-core kernel for this shape, so the outputs
agree within the attention tolerance (1e-3 of the output scale), the cache rows written before
exactly and the new rows within one fp16 step.  Collected last on purpose: it must pass alone and
after every other test of the session.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_static_attention_matches_context_entry():
    from oracle import ref
    from trixium_b200 import ops
    ctx = ops.Context(0)
    try:
        rng = np.random.default_rng(21)
        H, Hkv, hd, max_pos = 16, 8, 128, 640
        shape = ops.attn_shape(H, Hkv, hd, max_pos, rope_dims=hd, eps=1e-6)
        d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
        qn = d((1 + 0.1 * rng.standard_normal(hd)).astype(np.float32))
        kn = d((1 + 0.1 * rng.standard_normal(hd)).astype(np.float32))
        freq = d(ref.rope_freq(hd, 1e6))
        prefill = rng.standard_normal((300, Hkv, hd)).astype(np.float16)
        caches = []
        for _ in range(2):
            kc = torch.zeros(max_pos, Hkv, hd, dtype=torch.float16, device="cuda")
            vc = torch.zeros_like(kc)
            kc[:300] = d(prefill)
            vc[:300] = d(prefill[::-1].copy())
            caches.append((kc, vc))
        err = torch.zeros(1, dtype=torch.int32, device="cuda")
        pos = torch.zeros(1, dtype=torch.int32, device="cuda")
        for step in range(2):
            pos.fill_(300 + step)
            q = d(rng.standard_normal(H * hd).astype(np.float32))
            k = d(rng.standard_normal(Hkv * hd).astype(np.float32))
            v = d(rng.standard_normal(Hkv * hd).astype(np.float32))
            want = ops.attn_decode(ctx, shape, q, k, v, qn, kn, freq, caches[0][0], caches[0][1], pos)
            got = ops.attn_decode_static(shape, q, k, v, qn, kn, freq, caches[1][0], caches[1][1], pos, err)
            torch.cuda.synchronize()
            scale = max(1.0, float(want.abs().max()))
            assert float((got - want).abs().max()) <= 1e-3 * scale
            p = 300 + step
            for a, b in zip(caches[0], caches[1]):
                assert torch.equal(a[:p], b[:p]) and torch.equal(a[p + 1:], b[p + 1:])
                assert torch.allclose(a[p].float(), b[p].float(), rtol=1e-3, atol=1e-3)
        assert int(err.item()) == 0
        assert ctx.errors() == 0
    finally:
        ctx.close()
