"""The context-free decode attention (trx_attn_decode_static), for callers that must not allocate
device memory while they run, checked against the context entry point (trx_attn_decode) and the
oracle: two calls in a row on identical inputs and separate caches, then a second shape (gated
query heads, head dim 64, another kv-head count) that reuses the same static arrays.  The static
entry runs the scratch-merge kernel on the library's static arrays, the context entry the
tensor-core kernel for the first shape, so the outputs agree within the attention tolerance (1e-3
of the output scale), the cache rows written before exactly and the new rows within one fp16 step.
The free device memory is the same before and after the static calls (the library allocates
nothing).  Collected last on purpose: it must pass alone and after every other test of the session.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _case(ctx, rng, H, Hkv, hd, max_pos, prefill_n, gated, compare_ctx):
    from oracle import ref
    from trixium_b200 import ops
    shape = ops.attn_shape(H, Hkv, hd, max_pos, rope_dims=hd, gated=gated, eps=1e-6)
    d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    qn_h = (1 + 0.1 * rng.standard_normal(hd)).astype(np.float32)
    kn_h = (1 + 0.1 * rng.standard_normal(hd)).astype(np.float32)
    freq_h = ref.rope_freq(hd, 1e6)
    qn, kn, freq = d(qn_h), d(kn_h), d(freq_h)
    prefill = rng.standard_normal((prefill_n, Hkv, hd)).astype(np.float16)
    caches = []
    for _ in range(2):
        kc = torch.zeros(max_pos, Hkv, hd, dtype=torch.float16, device="cuda")
        vc = torch.zeros_like(kc)
        kc[:prefill_n] = d(prefill)
        vc[:prefill_n] = d(prefill[::-1].copy())
        caches.append((kc, vc))
    kc_o = np.zeros((max_pos, Hkv, hd), dtype=np.float16)
    vc_o = np.zeros_like(kc_o)
    kc_o[:prefill_n], vc_o[:prefill_n] = prefill, prefill[::-1]
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    pos = torch.zeros(1, dtype=torch.int32, device="cuda")
    qrows = H * hd * (2 if gated else 1)
    for step in range(2):
        p = prefill_n + step
        pos.fill_(p)
        q_h = rng.standard_normal(qrows).astype(np.float32)
        k_h = rng.standard_normal(Hkv * hd).astype(np.float32)
        v_h = rng.standard_normal(Hkv * hd).astype(np.float32)
        q, k, v = d(q_h), d(k_h), d(v_h)
        got = torch.empty(H * hd, dtype=torch.float32, device="cuda")
        torch.cuda.synchronize()
        free0 = torch.cuda.mem_get_info()[0]
        ops.attn_decode_static(shape, q, k, v, qn, kn, freq, caches[1][0], caches[1][1], pos, err, out=got)
        torch.cuda.synchronize()
        assert torch.cuda.mem_get_info()[0] == free0, "the static entry allocated device memory"
        qm = q_h.reshape(H, -1)
        want_o = ref.attn_decode(qm[:, :hd].copy(), k_h.reshape(Hkv, hd), v_h.reshape(Hkv, hd), kc_o, vc_o, p,
                                 qn_h, kn_h, 1e-6, freq_h, gate=qm[:, hd:].copy() if gated else None).reshape(-1)
        scale = max(1.0, float(np.abs(want_o).max()))
        assert float(np.abs(got.cpu().numpy() - want_o).max()) <= 1e-3 * scale
        if compare_ctx:
            want = ops.attn_decode(ctx, shape, q, k, v, qn, kn, freq, caches[0][0], caches[0][1], pos)
            torch.cuda.synchronize()
            assert float((got - want).abs().max()) <= 1e-3 * scale
            for a, b in zip(caches[0], caches[1]):
                assert torch.equal(a[:p], b[:p]) and torch.equal(a[p + 1:], b[p + 1:])
                assert torch.allclose(a[p].float(), b[p].float(), rtol=1e-3, atol=1e-3)
    assert int(err.item()) == 0


def test_static_attention_matches_context_entry_and_oracle():
    from trixium_b200 import ops
    ctx = ops.Context(0)
    try:
        rng = np.random.default_rng(21)
        _case(ctx, rng, 16, 8, 128, 640, 300, gated=False, compare_ctx=True)
        # Another shape on the same static arrays: the arrival counts left at zero by the first.
        _case(ctx, rng, 12, 4, 64, 900, 517, gated=True, compare_ctx=True)
        assert ctx.errors() == 0
    finally:
        ctx.close()
