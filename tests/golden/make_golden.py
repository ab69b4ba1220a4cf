"""Generate the golden fixtures for the ternary decode path from the reference's own Python.

Run where the TriXium reference tree (read-only) is importable, with TRIXIUM_REF naming its
root directory:

    TRIXIUM_REF=<reference tree> python tests/golden/make_golden.py

It imports the reference's `model.bons` (TensorSpec + encode_rows: the converter's row-packet
bytes, with its per-tensor B/R), `model.bitexact` (matvec_ternary and matvec_q8, the engine's integer specs),
`model.mirror` (_quantize_f_pow2 and _sumsq64), `model.deltanet` (head_step, the integer DeltaNet
head), and writes small .npz files next to this script.  The GPU box never reads the reference: the tests read only these fixtures.

Cases follow the reference's own tests where they exist:
* test/model/test_bitexact.py:36-56 (seed 42, 64x512, uniform scales, uniform x8),
* test/model/test_bitexact.py:58-70 (seed 7, 16x12288 all +1 codes, x8 = 127: the no-overflow
  bound),
plus the benchmark distribution at small sizes, ragged G (K = 128, 640, 2944), negative /
subnormal / zero scales, an all-zero activation, fp32 rounding edges for the quantiser, and
every trit5 byte value.
"""

import os
import sys

import numpy as np

REF = os.environ.get("TRIXIUM_REF")
if not REF:
    sys.exit("set TRIXIUM_REF to the root of the TriXium reference tree")
sys.path.insert(0, REF)

from model import bitexact as bx          # noqa: E402
from model import bons, layout, mirror    # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
f32 = np.float32


def ref_pack(name, scales, codes, kind):
    """The converter's bytes and B/R for one tensor (model/bons.py TensorSpec + encode_rows)."""
    rows, cols = codes.shape
    spec = bons.TensorSpec(name, layout.ROLE_FFN_GATE, 0, layout.KIND_TERNARY, rows, cols,
                           scales=scales, values=codes)
    spec.kind = kind          # write_image(trit5=True) switches the kind the same way.
    packed = bons.encode_rows(spec, 0, rows)
    return packed, spec.bias, spec.rshift


def bench_dist(rng, rows, cols):
    u = rng.random((rows, cols))
    codes = np.where(u < 0.3, 0, np.where(u < 0.7, 1, 2)).astype(np.uint8)
    scales = (np.abs(rng.standard_normal((rows, cols // 128))) * 0.02).astype(np.float16)
    return codes, scales


def matvec_case(name, codes, scales, x=None, x8=None):
    rows, cols = codes.shape
    out = {}
    for kind in (layout.KIND_TERNARY, layout.KIND_TERNARY5):
        packed, B, R = ref_pack(name, scales, codes, kind)
        out[f"packed_k{kind}"] = packed
        out["B"], out["R"] = B, R
        # Round trip through the reference reader.
        entry = {"kind": kind, "cols": cols}
        s2, c2 = bons.decode_rows(entry, packed.tobytes())
        assert np.array_equal(c2, codes) and np.array_equal(s2.view(np.uint16), scales.view(np.uint16))
    if x8 is None:
        x8, e8 = mirror._quantize_f_pow2(np.asarray(x, dtype=f32))
        out["x"] = np.asarray(x, dtype=f32)
    else:
        e8 = 0
    res = bx.matvec_ternary(scales, codes, x8, out["B"], out["R"])
    out.update(rows=rows, cols=cols, scales=scales, codes=codes, x8=x8, e8=e8, y_int=res)
    # The mirror's float result of the quantised projection (model/mirror.py:676-678).
    sc = f32(np.exp2(f32(e8 + out["R"] - out["B"])))
    out["y_f"] = (res.astype(np.int32).astype(f32) * sc).astype(f32)
    # fp64 reference of the fp projection on the same fp32 x (test_bitexact.py:49-56).
    if x is not None:
        w = codes.astype(np.float64).reshape(rows, -1, 128) - 1.0
        gs = np.einsum("rgk,gk->rg", w, np.asarray(x, np.float64).reshape(-1, 128))
        out["y_f64"] = (gs * scales.astype(np.float64)).sum(axis=1)
    np.savez_compressed(os.path.join(HERE, f"matvec_{name}.npz"), **out)
    return out


def q8_case(name, q8w, scales, x8, B=None, R=None):
    """A KIND_Q8 tensor (group 32) through the converter (model/bons.py TensorSpec + encode_rows,
    its B/R from GS_MAX_Q8) and the engine's Q8 row-dot spec (model/bitexact.py:127-144).  B and R
    may be given instead (the K-cache scores of model/mirror.py:243-253 pick their own)."""
    rows, cols = q8w.shape
    spec = bons.TensorSpec(name, layout.ROLE_FFN_GATE, 0, layout.KIND_Q8, rows, cols,
                           scales=scales, values=q8w)
    packed = bons.encode_rows(spec, 0, rows)
    s2, v2 = bons.decode_rows({"kind": layout.KIND_Q8, "cols": cols}, packed.tobytes())
    assert np.array_equal(v2, q8w) and np.array_equal(s2.view(np.uint16), scales.view(np.uint16))
    B = spec.bias if B is None else B
    R = spec.rshift if R is None else R
    res = bx.matvec_q8(scales, q8w, x8, B, R)
    np.savez_compressed(os.path.join(HERE, f"q8_{name}.npz"), packed=packed, B=B, R=R, rows=rows,
                        cols=cols, scales=scales, q8w=q8w, x8=x8, y_int=res)


def q8_cases():
    # 1. The reference's own Q8 accuracy case (test/model/test_bitexact.py:72-86).
    rng = np.random.default_rng(3)
    M, K = 32, 256
    scales = rng.uniform(0.005, 0.02, (M, K // 32)).astype(np.float16)
    q8w = rng.integers(-127, 128, (M, K), dtype=np.int8)
    x8 = rng.integers(-127, 128, K, dtype=np.int8)
    q8_case("refacc_32x256", q8w, scales, x8)
    # 2. Near the int48 bound: every product 127*127, scales spread over 10 octaves (the converter's
    #    B targets the ternary range, so a much wider Q8 row of these overflows the accumulator).
    rng = np.random.default_rng(8)
    M, K = 16, 512
    scales = (np.exp2(rng.uniform(-10, 0, (M, K // 32))) * 0.5).astype(np.float16)
    q8_case("bound_16x512", np.full((M, K), 127, np.int8), scales, np.full(K, 127, np.int8))
    # 3. Ragged group counts (G = 1, 3, 17, 65, 130) with signed, subnormal and zero scales.
    for (rows, cols, seed) in [(5, 32, 20), (9, 96, 21), (33, 544, 22), (40, 2080, 23), (12, 4160, 24)]:
        rng = np.random.default_rng(seed)
        s = rng.standard_normal((rows, cols // 32)) * 0.03
        s[0, 0] = 6e-8                      # fp16 subnormal
        s[min(1, rows - 1), :] = 0.0
        s[rows - 1, ::2] *= -1.0
        q8w = rng.integers(-127, 128, (rows, cols), dtype=np.int8)
        x8 = rng.integers(-127, 128, cols, dtype=np.int8)
        q8_case(f"ragged_{rows}x{cols}", q8w, s.astype(np.float16), x8)
    # 4. K-cache scores as the firmware computes them (model/mirror.py:243-253): one power-of-two
    #    scale per cached row, B = 22 - max exponent, R from the (hd/32)*32*127*127*1024 << 12 bound.
    rng = np.random.default_rng(25)
    hd, n = 128, 77
    ek = rng.integers(-12, -4, n)
    scales = np.repeat(np.exp2(ek.astype(np.float64))[:, None], hd // 32, axis=1).astype(np.float16)
    q8w = rng.integers(-127, 128, (n, hd), dtype=np.int8)
    x8 = rng.integers(-127, 128, hd, dtype=np.int8)
    B = 22 - int(ek.max())
    bound, R = (hd // 32) * 32 * 127 * 127 * 1024 << 12, 0
    while (bound >> R) >= (1 << 31):
        R += 1
    q8_case("kscores_77x128", q8w, scales, x8, B=B, R=R)


def hadamard_case(width, block, seed):
    """The rotation x' = R(s*x) per block as the engine computes it (model/mirror.py:680-690): the
    converter's block tensors (model/convert.py:99-118, called here) and one quantised float
    projection per block (model/mirror.py:664-678 inline: _quantize_f_pow2, matvec_ternary,
    the 2^(e8+R-B) scale)."""
    import types
    from model import convert, golden
    rng = np.random.default_rng(seed)
    signs = np.where(rng.random(width) < 0.5, -1.0, 1.0).astype(f32)
    x = (rng.standard_normal(width) * 2).astype(f32)
    specs = convert._hadamard_specs(types.SimpleNamespace(hadamard_block=block, hadamard_signs={width: signs}))
    y = np.empty(width, f32)
    packed = []
    for b, spec in enumerate(specs):
        codes = spec.get_values()
        packed.append(bons.encode_rows(spec, 0, block))
        x8, e8 = mirror._quantize_f_pow2(x[b * block:(b + 1) * block])
        r = bx.matvec_ternary(spec.scales, codes, x8, spec.bias, spec.rshift)
        y[b * block:(b + 1) * block] = (r.astype(np.int32).astype(f32) *
                                        f32(np.exp2(f32(e8 + spec.rshift - spec.bias)))).astype(f32)
    # The float transform the rotation approximates, times the image's gain (golden.py:265-283).
    y_ref = golden.hadamard_rotate(x, signs, block) * f32(golden.hadamard_image_gain(block))
    np.savez_compressed(os.path.join(HERE, f"hadamard_{width}_{block}.npz"), x=x, signs=signs, block=block,
                        packed=np.concatenate(packed), B=specs[0].bias, R=specs[0].rshift,
                        scale=specs[0].scales[0, 0], y=y, y_ref=y_ref.astype(f32))


def bons_case():
    """A one-layer tiny image from the reference's own generator and writer (model/tinygen.py
    generate -> model/bons.py write_image; 2 channels, trit5, no int16 embedding), stored gzipped,
    with what the reference's reader (model/bons.py:476-525) makes of it: the header fields, the
    entry names, and per matvec tensor the sha256 of its decoded scales and codes and its engine
    matvec on a seeded x8."""
    import dataclasses
    import gzip
    import hashlib
    import shutil
    import tempfile
    from model import tinygen
    cfg = dataclasses.replace(tinygen.BONSAI_TINY, n_layer=1, name="bonsai-tiny-l1")
    with tempfile.TemporaryDirectory() as tmp:
        img, _, _ = tinygen.generate(tmp, n_channels=2, seed=1234, cfg=cfg, trit5=True, emb16=False)
        with open(img, "rb") as src, gzip.GzipFile(os.path.join(HERE, "bons_tiny_l1_t5_n2.img.gz"), "wb",
                                                    compresslevel=9, mtime=0) as dst:
            shutil.copyfileobj(src, dst)
        r = bons.BONSReader(img)
        out = {k: r.header[k] for k in ("n_layer", "n_embd", "n_head", "n_kv_head", "head_dim", "ffn_dim",
                                        "vocab", "n_channels", "n_tensors", "payload_beats")}
        out["names"] = np.array([e["name"] for e in r.entries])
        rng = np.random.default_rng(40)
        for i, e in enumerate(r.entries):
            if e["kind"] not in (layout.KIND_TERNARY, layout.KIND_TERNARY5, layout.KIND_Q8):
                continue
            scales, values = r.tensor(e["name"])
            h = hashlib.sha256(np.ascontiguousarray(scales).tobytes() +
                               np.ascontiguousarray(values).astype(np.int16).tobytes()).hexdigest()
            x8 = rng.integers(-127, 128, e["cols"], dtype=np.int8)
            if e["kind"] == layout.KIND_Q8:
                y = bx.matvec_q8(scales, values, x8, e["bias"], e["rshift"])
            else:
                y = bx.matvec_ternary(scales, values, x8, e["bias"], e["rshift"])
            out[f"e{i}_sha"], out[f"e{i}_x8"], out[f"e{i}_y"] = h, x8, y
    np.savez_compressed(os.path.join(HERE, "bons_tiny_l1_t5_n2.npz"), **out)


def _hybrid_cfg(base, **kw):
    import dataclasses
    return dataclasses.replace(base, **kw)


def _exact_weights(img, e):
    """A matvec tensor as the mirror's exact mode dequantises it (model/mirror.py:648-662)."""
    scales, codes = img.tensor(e["name"])
    if e["kind"] == layout.KIND_F32:
        return np.asarray(codes, dtype=f32).reshape(e["rows"], e["cols"])
    g = 128 if layout.is_ternary(e["kind"]) else 32
    off = 1.0 if layout.is_ternary(e["kind"]) else 0.0
    w = (codes.astype(f32).reshape(e["rows"], -1, g) - f32(off)) * scales.astype(f32)[:, :, None]
    return w.reshape(e["rows"], e["cols"])


def hybrid_kernel_case(name, cfg, n_prompt=8, n_new=4, seed=1234):
    """Kernel-level fixtures for decode attention and the gated-DeltaNet step from the reference's
    firmware mirror (model/mirror.py:594-1044, hybrid27_generate with exact=True: fp32 weights, no
    activation quantisation, the mathematical profile).  The image comes from the reference's own
    tensor inventory and writer (model/tinygen.py make_tiny_hybrid_tensors, model/bons.py
    write_image) with no rotation and the layers' output projections (attn_output, ssm_out)
    replaced by identity matrices (code 2 on the diagonal, 1 elsewhere, scale 1.0), so the traced
    layer outputs ("attn_out", "dn_out", mirror.py:1008-1011) are the attention and DeltaNet
    results themselves.  Stored per (position, layer): the layer's normed input's projections
    (q with its gate; qkv, z, beta and alpha before their activations), computed as the mirror's
    exact mode does (dequantised fp32 weights times the traced "attn_norm" vector), and the
    traced output; per layer the norm weights, conv taps, A and dt bias; the rope frequencies."""
    import tempfile
    from model import tinygen
    import dataclasses
    # The inventory as tinygen makes it (its rotation tensors need a block), then without them.
    tensors = tinygen.make_tiny_hybrid_tensors(dataclasses.replace(cfg, hadamard_block=128), seed)
    tensors = [t for t in tensors if t.role != layout.ROLE_HADAMARD]
    cfg = dataclasses.replace(cfg, hadamard_block=0, hadamard_signs=None)
    E = cfg.n_embd
    for t in tensors:
        if t.role in (layout.ROLE_ATTN_OUT, layout.ROLE_SSM_OUT):
            assert t.rows == E and t.cols == E, (t.name, t.rows, t.cols)
            t.values = (np.eye(E, dtype=np.uint8) + 1).astype(np.uint8)
            t.scales = np.ones((E, E // 128), np.float16)
            t.bias = bx.choose_scale_bias(bx.fp16_decompose(t.scales)[1])
            t.rshift = bx.choose_result_shift(t.scales, t.bias)
    trace = {}
    with tempfile.TemporaryDirectory() as tmp:
        path = os.path.join(tmp, "k.img")
        bons.write_image(cfg, tensors, 1, path, emb16=True)
        img = bons.BONSReader(path)
        h = img.header
        rng = np.random.default_rng(seed + 1)
        prompt = [int(t) for t in rng.integers(0, cfg.vocab, n_prompt)]

        def cb(pos, layer, tag, dtype, values):
            trace[(pos, layer, tag)] = np.asarray(values)
        mirror.hybrid27_generate(img, prompt, n_new, exact=True, trace=cb)
        ent = lambda role, l: next(e for e in img.entries if e["role"] == role and e["layer"] == l)
        f32row = lambda role, l: np.asarray(img.tensor(ent(role, l)["name"])[1], dtype=f32).reshape(-1)
        out = {"n_embd": E, "n_head": h["n_head"], "n_kv": h["n_kv_head"], "head_dim": h["head_dim"],
               "rope_dims": h["rope_dims"] or h["head_dim"], "gated": h["attn_gated"], "eps": f32(h["rms_eps"]),
               "nk": h["dn_num_k_heads"], "hk": h["dn_k_head_dim"], "nv": h["dn_num_v_heads"],
               "hv": h["dn_v_head_dim"], "conv": h["dn_conv_kernel"],
               "layer_types": np.array([1 if t == "deltanet" else 0 for t in h["layer_types"]])}
        rope_n = out["rope_dims"]
        out["rope_freq"] = np.array([f32(np.float32(h["rope_theta"]) ** f32(-2.0 * i / rope_n))
                                     for i in range(rope_n // 2)], dtype=f32)
        npos = n_prompt + n_new - 1
        out["npos"] = npos
        for l, lt in enumerate(h["layer_types"]):
            W = lambda role: _exact_weights(img, ent(role, l))
            hn = np.stack([trace[(p, l, "attn_norm")] for p in range(npos)]).astype(f32)
            if lt == "deltanet":
                for key, role in (("qkv", layout.ROLE_ATTN_QKV), ("z", layout.ROLE_ATTN_ZGATE),
                                  ("beta", layout.ROLE_SSM_BETA), ("alpha", layout.ROLE_SSM_ALPHA)):
                    w = W(role)
                    out[f"l{l}_{key}"] = np.stack([(w @ v).astype(f32) for v in hn])
                out[f"l{l}_out"] = np.stack([trace[(p, l, "dn_out")] for p in range(npos)]).astype(f32)
                out[f"l{l}_conv_w"] = f32row(layout.ROLE_SSM_CONV, l)
                out[f"l{l}_ssm_a"] = f32row(layout.ROLE_SSM_A, l)
                out[f"l{l}_dt_bias"] = f32row(layout.ROLE_SSM_DT, l)
                out[f"l{l}_ssm_norm"] = f32row(layout.ROLE_SSM_NORM, l)
            else:
                for key, role in (("q", layout.ROLE_ATTN_Q), ("k", layout.ROLE_ATTN_K), ("v", layout.ROLE_ATTN_V)):
                    w = W(role)
                    out[f"l{l}_{key}"] = np.stack([(w @ v).astype(f32) for v in hn])
                out[f"l{l}_out"] = np.stack([trace[(p, l, "attn_out")] for p in range(npos)]).astype(f32)
                out[f"l{l}_q_norm"] = f32row(layout.ROLE_ATTN_Q_NORM, l)
                out[f"l{l}_k_norm"] = f32row(layout.ROLE_ATTN_K_NORM, l)
    np.savez_compressed(os.path.join(HERE, f"mirror_layers_{name}.npz"), **out)


def hybrid_tokens_case(name, cfg, trit5, kseg_max, n_prompt=6, n_new=128, seed=1234):
    """End-to-end fixture: a tiny hybrid image from the reference's own generator and writer
    (model/tinygen.py generate: DeltaNet and gated attention layers, the Hadamard-rotated basis,
    Q8 beta/alpha, the int16 embedding table; K-segmented where wider than kseg_max), stored
    gzipped, and the reference mirror's greedy tokens for a seeded prompt in its engine arithmetic
    (model/mirror.py:594-1044, hybrid27_generate with exact=False and the mathematical profile):
    int8 power-of-two activations, the engine's integer matvec.  Per generated step the logits and
    their top-two margin are kept too (where the margin is tiny, fp32 rounding order may flip the
    argmax)."""
    import gzip
    import shutil
    import tempfile
    from model import tinygen
    with tempfile.TemporaryDirectory() as tmp:
        img_path, _, _ = tinygen.generate(tmp, n_channels=2, seed=seed, cfg=cfg, kseg_max=kseg_max, trit5=trit5)
        with open(img_path, "rb") as src, gzip.GzipFile(os.path.join(HERE, f"tokens_{name}.img.gz"), "wb",
                                                         compresslevel=9, mtime=0) as dst:
            shutil.copyfileobj(src, dst)
        img = bons.BONSReader(img_path)
        rng = np.random.default_rng(seed + 2)
        prompt = [int(t) for t in rng.integers(0, cfg.vocab, n_prompt)]
        margins, ckpt, logits = {}, {}, {}

        def cb(pos, layer, tag, dtype, values):
            if tag == "logits":
                v = np.sort(np.asarray(values, dtype=np.float64))
                margins[pos] = v[-1] - v[-2]
                logits[pos] = np.asarray(values, dtype=f32)
            if pos < 3 and tag in ("emb", "attn_res", "ffn_res", "out_norm", "logits"):
                ckpt[f"p{pos}_l{layer}_{tag}"] = np.asarray(values, dtype=f32)
        toks = mirror.hybrid27_generate(img, prompt, n_new, exact=False, silu_mode="mathematical", trace=cb)
    npos = n_prompt + n_new - 1
    steps = range(n_prompt - 1, npos)
    np.savez_compressed(os.path.join(HERE, f"tokens_{name}.npz"), prompt=np.array(prompt), tokens=np.array(toks),
                        margins=np.array([margins[p] for p in steps]),
                        logits=np.stack([logits[p] for p in steps]), **ckpt)


def fastref_case(name):
    """The fp-mode projections of the reference's fast engine (model/fastref.py HybridRef: matmul of
    an entry, proj of (role, layer) with the Hadamard rotation and K-segments) on the reference-made
    image tokens_<name>.img.gz, for seeded X of 5 rows."""
    import gzip
    import shutil
    import tempfile
    from model import fastref
    with tempfile.TemporaryDirectory() as tmp:
        path = os.path.join(tmp, "img")
        with gzip.open(os.path.join(HERE, f"tokens_{name}.img.gz"), "rb") as src, open(path, "wb") as dst:
            shutil.copyfileobj(src, dst)
        img = bons.BONSReader(path)
        ref = fastref.HybridRef(img)
        rng = np.random.default_rng(77)
        out = {}
        roles = [(layout.ROLE_FFN_GATE, 0), (layout.ROLE_FFN_DOWN, 0), (layout.ROLE_FFN_UP, 1), (layout.ROLE_LM_HEAD, 0)]
        for i, (role, l) in enumerate(roles):
            e = ref._entry(role, l)
            cols = sum(t["cols"] for t in ref._ksegs(e))
            X = (rng.standard_normal((5, cols)) * 0.7).astype(f32)
            out[f"proj{i}_role"] = np.int32(role)
            out[f"proj{i}_layer"] = np.int32(l)
            out[f"proj{i}_X"] = X
            out[f"proj{i}_Y"] = ref.proj(role, l, X)
            out[f"proj{i}_M"] = ref.matmul(e, X)   # the same entry without the rotation
        np.savez_compressed(os.path.join(HERE, f"fastref_{name}.npz"), n=np.int32(len(roles)), **out)


def kseg_case(name, rows, cols, kind, seed):
    """A K-segmented projection (model/bons.py:83-113 split_wide: equal column ranges, the whole
    tensor's B/R in each segment) through the converter's row packets and the mirror's float
    projection (model/mirror.py:664-678: one exponent for the whole input, per segment the
    engine's int32 result, their int64 sum wrapped to int32, scaled once)."""
    rng = np.random.default_rng(seed)
    if kind == layout.KIND_Q8:
        values = rng.integers(-127, 128, (rows, cols), dtype=np.int8)
        scales = rng.uniform(0.005, 0.02, (rows, cols // 32)).astype(np.float16)
        spec = bons.TensorSpec(name, layout.ROLE_FFN_DOWN, 0, layout.KIND_Q8, rows, cols, scales=scales,
                               values=values)
        segs = bons.split_wide(spec)
    else:
        values, scales = bench_dist(rng, rows, cols)
        spec = bons.TensorSpec(name, layout.ROLE_FFN_DOWN, 0, layout.KIND_TERNARY, rows, cols, scales=scales,
                               values=values)
        segs = bons.split_wide(spec)
        for t in segs:
            t.kind = kind          # write_image(trit5=True) switches the kind the same way.
    assert len(segs) > 1 and all(t.flags & layout.FLAG_KSEG for t in segs)
    x = rng.standard_normal(cols).astype(f32)
    x8, e8 = mirror._quantize_f_pow2(x)
    res, c0, out = None, 0, {}
    for k, t in enumerate(segs):
        assert (t.bias, t.rshift) == (spec.bias, spec.rshift) and t.kseg == k
        out[f"packed{k}"] = bons.encode_rows(t, 0, rows)
        out[f"cols{k}"] = t.cols
        xs = x8[c0:c0 + t.cols]
        if kind == layout.KIND_Q8:
            r = bx.matvec_q8(t.scales, t.get_values(), xs, t.bias, t.rshift)
        else:
            r = bx.matvec_ternary(t.scales, t.get_values(), xs, t.bias, t.rshift)
        res = r.astype(np.int64) if res is None else res + r.astype(np.int64)
        c0 += t.cols
    y = (res.astype(np.int32).astype(f32) * f32(np.exp2(f32(e8 + spec.rshift - spec.bias)))).astype(f32)
    np.savez_compressed(os.path.join(HERE, f"kseg_{name}.npz"), nseg=len(segs), rows=rows, cols=cols, kind=kind,
                        B=spec.bias, R=spec.rshift, x=x, y=y, **out)


def dn_int_case():
    """The integer DeltaNet head step (model/deltanet.py head_step) over a few tokens per shape, as
    test/model/test_asm.py:554-590 drives it (the state starts at exponent -20 and empty, so the
    first tokens ratchet and the small last one does not).  Token t starts from token t-1's state
    (zero at token 0)."""
    from model import deltanet as dn
    out = {}
    for (hv, hk, seed) in [(64, 64, 1), (128, 128, 2), (128, 128, 3), (32, 64, 4)]:
        rng = np.random.default_rng(seed)
        M = np.zeros((hv, hk), dtype=np.int64)
        eM, maxM = -20, 0
        tag = f"h{hv}x{hk}s{seed}"
        for tok in range(4):
            kk = rng.standard_normal(hk).astype(f32); kk /= np.linalg.norm(kk)
            qh = rng.standard_normal(hk).astype(f32); qh /= np.linalg.norm(qh)
            vh = (rng.standard_normal(hv) * (3.0 if tok < 2 else 0.05)).astype(f32)
            decay, beta = f32(rng.uniform(0.3, 1.0)), f32(rng.uniform(0.2, 1.0))
            o, eM2, maxM2 = dn.head_step(M, eM, kk, qh, vh, decay, beta, maxM=maxM)
            out.update({f"{tag}_t{tok}_eM": np.int32(eM),
                        f"{tag}_t{tok}_maxM": np.int32(maxM), f"{tag}_t{tok}_k": kk, f"{tag}_t{tok}_q": qh,
                        f"{tag}_t{tok}_v": vh, f"{tag}_t{tok}_decay": decay, f"{tag}_t{tok}_beta": beta,
                        f"{tag}_t{tok}_o": o, f"{tag}_t{tok}_M": M.astype(np.int16),
                        f"{tag}_t{tok}_eM2": np.int32(eM2), f"{tag}_t{tok}_maxM2": np.int32(maxM2)})
            eM, maxM = eM2, maxM2
    out["shapes"] = np.array([(64, 64, 1), (128, 128, 2), (128, 128, 3), (32, 64, 4)], dtype=np.int32)
    np.savez_compressed(os.path.join(HERE, "dn_int_steps.npz"), **out)


def main():
    from model import tinygen
    dn_int_case()
    # Decode attention and the DeltaNet step, pinned to the mirror (identity output projections).
    hybrid_kernel_case("hd64", _hybrid_cfg(tinygen.BONSAI_TINY_HYBRID, hadamard_block=0, dn_num_v_heads=4,
                                           name="kernels-hd64"))
    hybrid_kernel_case("hd256", _hybrid_cfg(tinygen.BONSAI_TINY_HYBRID, hadamard_block=0, n_embd=512, n_head=2,
                                            n_kv_head=1, head_dim=256, rope_dims=64, dn_num_k_heads=2,
                                            dn_k_head_dim=128, dn_num_v_heads=4, dn_v_head_dim=128,
                                            ffn_dim=512, name="kernels-hd256"))
    # Greedy tokens of the mirror's engine arithmetic on reference-made images.
    hybrid_tokens_case("hybrid_t5_kseg", tinygen.BONSAI_TINY_HYBRID, trit5=True, kseg_max=256)
    hybrid_tokens_case("hybrid_2b", tinygen.BONSAI_TINY_HYBRID, trit5=False, kseg_max=None)
    # K-segmented projections at the hybrid-27b down projection's width and a wide Q8 tensor.
    fastref_case("hybrid_t5_kseg")
    kseg_case("t5_24x17408", 24, 17408, layout.KIND_TERNARY5, 50)
    kseg_case("2b_40x17408", 40, 17408, layout.KIND_TERNARY, 51)
    kseg_case("q8_20x9216", 20, 9216, layout.KIND_Q8, 52)
    q8_cases()
    bons_case()
    hadamard_case(1024, 512, 30)
    hadamard_case(2048, 1024, 31)
    hadamard_case(512, 128, 32)
    # 1. The reference's own matvec accuracy case (test_bitexact.py:36-47).
    rng = np.random.default_rng(42)
    M, K = 64, 512
    scales = rng.uniform(0.01, 0.08, (M, K // 128)).astype(np.float16)
    codes = rng.integers(0, 3, (M, K), dtype=np.uint8)
    x8 = rng.integers(-127, 128, K, dtype=np.int8)
    matvec_case("refacc_64x512", codes, scales, x8=x8)

    # 2. The reference's no-overflow bound (test_bitexact.py:58-70).
    rng = np.random.default_rng(7)
    M, K = 16, 12288
    scales = (np.exp2(rng.uniform(-10, 0, (M, K // 128))) * 0.5).astype(np.float16)
    codes = np.full((M, K), 2, dtype=np.uint8)
    x8 = np.full(K, 127, dtype=np.int8)
    matvec_case("refbound_16x12288", codes, scales, x8=x8)

    # 3. The benchmark distribution at small/ragged sizes (seeded draws: codes, scales, x).
    for (rows, cols, seed) in [(48, 2048, 0), (33, 640, 1), (7, 128, 2), (64, 4096, 3),
                               (20, 2944, 4), (16, 6144, 5), (3, 17408, 6)]:
        rng = np.random.default_rng(seed)
        codes, scales = bench_dist(rng, rows, cols)
        x = rng.standard_normal(cols).astype(f32)
        matvec_case(f"bench_{rows}x{cols}", codes, scales, x=x)

    # 4. Signed, subnormal and zero scales; one all-zero-codes row (w = -1 everywhere).
    rng = np.random.default_rng(11)
    rows, cols = 24, 1024
    codes = rng.integers(0, 3, (rows, cols), dtype=np.uint8)
    codes[5] = 0
    s = rng.standard_normal((rows, cols // 128)) * 0.05
    s[1, :] = 6e-8                          # fp16 subnormals
    s[2, 3] = 0.0
    s[3, :] = -np.abs(s[3, :])
    scales = s.astype(np.float16)
    x = (rng.standard_normal(cols) * 3).astype(f32)
    matvec_case("signed_24x1024", codes, scales, x=x)

    # 5. An all-zero activation: x8 = 0, e8 = 0 (model/mirror.py:47-49).
    rng = np.random.default_rng(12)
    codes, scales = bench_dist(rng, 8, 256)
    matvec_case("zerox_8x256", codes, scales, x=np.zeros(256, f32))

    # 6. Quantiser edges: values at the fp32 rounding boundaries of floor(x + 0.5).
    rng = np.random.default_rng(13)
    xs = []
    for e in (0, -3, 5):
        base = rng.standard_normal(256).astype(f32) * f32(2.0 ** e)
        base[0] = f32(127.99) * f32(2.0 ** (e - 7 + 7)) if e == 0 else base[0]
        # Values whose scaled magnitude is k + 0.5 - 2**-25 and k + 0.5 exactly.
        amax = np.abs(base).max()
        e8 = int(np.frexp(f32(amax))[1]) - 7
        for i, k in enumerate(range(0, 40)):
            v = f32(k) + f32(0.5)
            base[10 + 2 * i] = f32(np.nextafter(v, f32(0))) * f32(np.exp2(e8)) * (1 if k % 2 else -1)
            base[11 + 2 * i] = v * f32(np.exp2(e8)) * (-1 if k % 2 else 1)
        xs.append(base)
    xq = np.stack(xs)
    q = [mirror._quantize_f_pow2(v) for v in xq]
    np.savez_compressed(os.path.join(HERE, "quantize.npz"), x=xq,
                        x8=np.stack([a for a, _ in q]), e8=np.array([b for _, b in q]))

    # 7. The canonical sum of squares (model/mirror.py:576-591) at the norm widths.
    rng = np.random.default_rng(14)
    sums = {}
    for n in (64, 100, 128, 256, 2048, 4096, 5120):
        v = (rng.standard_normal(n) * 2).astype(f32)
        sums[f"v{n}"] = v
        sums[f"ss{n}"] = np.array(mirror._sumsq64(v), dtype=f32)
    np.savez_compressed(os.path.join(HERE, "sumsq64.npz"), **sums)

    # 8. Every trit5 byte through the reference reader (model/bons.py:125-130).
    g = 10
    body = np.zeros((1, 26 * g), dtype=np.uint8)
    body[0, :256] = np.arange(256, dtype=np.uint8)
    digits = bons.trit5_unpack_rows(body, 128 * g)
    np.savez_compressed(os.path.join(HERE, "trit5_bytes.npz"), body=body, codes=digits)
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
