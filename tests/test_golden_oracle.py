"""The oracle and the host-side packer against the reference's golden vectors (CPU only).

Fixtures: tests/golden/*.npz, made by tests/golden/make_golden.py from the reference's own
model/bons.py (encode_rows, TensorSpec B/R), model/bitexact.py (matvec_ternary) and
model/mirror.py (_quantize_f_pow2, _sumsq64).
"""
import glob
import os

import numpy as np
import pytest

from oracle import ref
from oracle import build as cor
from trixium_b200 import image, layout as L

from conftest import GOLDEN, golden_matvec_files, load, fp_rel_err

FILES = golden_matvec_files()
IDS = [os.path.basename(f)[7:-4] for f in FILES]


@pytest.mark.parametrize("path", FILES, ids=IDS)
@pytest.mark.parametrize("kind", [L.KIND_TERNARY, L.KIND_TERNARY5])
def test_packer_bytes_and_contract(path, kind):
    d = load(path)
    t = image.TernaryTensor(d["scales"], d["codes"], kind=kind)
    assert np.array_equal(t.packed, d[f"packed_k{kind}"])
    assert (t.bias, t.rshift) == (int(d["B"]), int(d["R"]))
    assert t.packed.size == int(d["rows"]) * L.row_bytes(int(d["cols"]), kind)
    s, c = image.unpack_rows(t.packed, t.rows, t.cols, kind)
    assert np.array_equal(c, d["codes"]) and np.array_equal(s.view(np.uint16), d["scales"].view(np.uint16))


@pytest.mark.parametrize("path", FILES, ids=IDS)
@pytest.mark.parametrize("kind", [L.KIND_TERNARY, L.KIND_TERNARY5])
def test_oracle_int_matvec(path, kind):
    d = load(path)
    rows, cols = int(d["rows"]), int(d["cols"])
    s, c = ref.decode_packed(d[f"packed_k{kind}"], rows, cols, kind)
    assert np.array_equal(c, d["codes"])
    y = ref.matvec_int(s, c, d["x8"], int(d["B"]), int(d["R"]))
    assert np.array_equal(y, d["y_int"])
    yc, bad = cor.matvec_int(d[f"packed_k{kind}"], rows, cols, kind, d["x8"], int(d["B"]), int(d["R"]))
    assert bad == 0 and np.array_equal(yc, d["y_int"])


@pytest.mark.parametrize("path", [f for f in FILES if "x" in np.load(f)], ids=lambda p: os.path.basename(p))
def test_oracle_float_projection(path):
    d = load(path)
    rows, cols = int(d["rows"]), int(d["cols"])
    x8, e8 = ref.quantize_pow2(d["x"])
    assert np.array_equal(x8, d["x8"]) and e8 == int(d["e8"])
    for kind in (0, 5):
        s, c = ref.decode_packed(d[f"packed_k{kind}"], rows, cols, kind)
        yf = ref.matvec_f(s, c, d["x"], int(d["B"]), int(d["R"]))
        assert np.array_equal(yf.view(np.uint32), d["y_f"].view(np.uint32))
        yc, bad = cor.matvec_f(d[f"packed_k{kind}"], rows, cols, kind, int(d["B"]), int(d["R"]), d["x"])
        assert bad == 0 and np.array_equal(yc.view(np.uint32), d["y_f"].view(np.uint32))
        if np.any(d["y_f64"]):
            assert fp_rel_err(cor.matvec_fp(d[f"packed_k{kind}"], rows, cols, kind, d["x"]), d["y_f64"]) < 1e-3
            assert fp_rel_err(ref.matvec_fastref(s, c, d["x"])[0], d["y_f64"]) < 1e-3


def test_quantizer_rounding_edges():
    q = load(os.path.join(GOLDEN, "quantize.npz"))
    for x, x8, e8 in zip(q["x"], q["x8"], q["e8"]):
        a, b = ref.quantize_pow2(x)
        assert np.array_equal(a, x8) and b == int(e8)
        a, b = cor.quantize(x)
        assert np.array_equal(a, x8) and b == int(e8)


def test_sumsq64_canonical():
    d = load(os.path.join(GOLDEN, "sumsq64.npz"))
    for n in (64, 100, 128, 256, 2048, 4096, 5120):
        assert ref.sumsq64(d[f"v{n}"]).view(np.uint32) == d[f"ss{n}"].view(np.uint32)


def test_trit5_every_byte():
    d = load(os.path.join(GOLDEN, "trit5_bytes.npz"))
    body, codes = d["body"], d["codes"]
    g = body.shape[1] // 26
    packed = np.zeros((1, L.row_bytes(128 * g, 5)), np.uint8)
    packed[0, L.scale_bytes(128 * g):L.scale_bytes(128 * g) + 26 * g] = body[0]
    _, c = ref.decode_packed(packed.reshape(-1), 1, 128 * g, 5)
    assert np.array_equal(c, codes)
    assert ref.trit5_invalid(packed.reshape(-1), 1, 128 * g) == 13   # bytes 243..255


def test_oracle_raises_where_reference_asserts():
    d = load(os.path.join(GOLDEN, "matvec_refbound_16x12288.npz"))
    s, c = d["scales"], d["codes"]
    with pytest.raises(ref.OverflowError48):
        ref.matvec_int(s, c, d["x8"], int(d["B"]), 0)      # R = 0: the int32 result overflows
    _, bad = cor.matvec_int(d["packed_k5"], 16, 12288, 5, d["x8"], int(d["B"]), 0)
    assert bad == 16


def test_synthetic_distribution():
    rng = np.random.default_rng(0)
    codes, scales = image.synthetic_codes_scales(rng, 512, 2048)
    frac = np.bincount(codes.reshape(-1), minlength=3) / codes.size
    assert abs(frac[1] - 0.4) < 0.01 and abs(frac[0] - 0.3) < 0.01 and abs(frac[2] - 0.3) < 0.01
    assert scales.dtype == np.float16 and np.all(scales >= 0)


Q8_FILES = sorted(glob.glob(os.path.join(GOLDEN, "q8_*.npz")))


@pytest.mark.parametrize("path", Q8_FILES, ids=[os.path.basename(f)[3:-4] for f in Q8_FILES])
def test_q8_packer_and_oracle(path):
    """KIND_Q8: the packer's bytes and B/R equal the converter's (the K-score case carries the
    firmware's own B/R), and the oracle's Q8 row dot equals model/bitexact.py:matvec_q8."""
    d = load(path)
    rows, cols, B, R = int(d["rows"]), int(d["cols"]), int(d["B"]), int(d["R"])
    kscores = "kscores" in path
    t = image.Q8Tensor(d["scales"], d["q8w"], bias=B if kscores else None, rshift=R if kscores else None)
    assert np.array_equal(t.packed, d["packed"])
    assert (t.bias, t.rshift) == (B, R)
    assert t.packed.size == rows * L.q8_row_bytes(cols) == rows * ref.q8_row_bytes(cols)
    assert np.array_equal(ref.q8_pack(d["scales"], d["q8w"]), d["packed"])
    s, w = ref.q8_decode_packed(d["packed"], rows, cols)
    assert np.array_equal(w, d["q8w"]) and np.array_equal(s.view(np.uint16), d["scales"].view(np.uint16))
    assert np.array_equal(ref.matvec_q8(s, w, d["x8"], B, R), d["y_int"])


def test_q8_oracle_raises_where_reference_asserts():
    d = load(os.path.join(GOLDEN, "q8_bound_16x512.npz"))
    with pytest.raises(ref.OverflowError48):
        ref.matvec_q8(d["scales"], d["q8w"], d["x8"], int(d["B"]), 0)        # int32 result
    with pytest.raises(ref.OverflowError48):
        ref.matvec_q8(d["scales"], d["q8w"], d["x8"], int(d["B"]) + 6, 0)    # int48 accumulator


HAD_FILES = sorted(glob.glob(os.path.join(GOLDEN, "hadamard_*.npz")))


@pytest.mark.parametrize("path", HAD_FILES, ids=[os.path.basename(f)[9:-4] for f in HAD_FILES])
def test_hadamard_tensor_and_oracle_rotation(path):
    """The rotation's block tensors equal the converter's bytes and B/R (model/convert.py:99-118),
    and the oracle's blockwise engine rotation equals the reference's (model/mirror.py:680-690)."""
    d = load(path)
    block, B, R = int(d["block"]), int(d["B"]), int(d["R"])
    t = image.hadamard_tensor(d["signs"], block)
    assert np.array_equal(t.packed, d["packed"]) and (t.bias, t.rshift) == (B, R)
    s, c = ref.hadamard_codes(d["signs"], block)
    assert np.array_equal(c, t.codes) and np.array_equal(s.view(np.uint16), t.scales.view(np.uint16))
    y = ref.hadamard_rotate(d["x"], s, c, B, R)
    assert np.array_equal(y.view(np.uint32), d["y"].view(np.uint32))
    # The engine's rotation approximates the float transform (int8 activations): within 2 %.
    assert np.abs(y - d["y_ref"]).max() <= 0.02 * np.abs(d["y_ref"]).max()


# Decode attention and the gated-DeltaNet step against the reference's firmware mirror -------------
# Fixtures mirror_layers_*.npz: model/mirror.py hybrid27_generate (exact=True, mathematical profile)
# on a reference-written hybrid image whose output projections are identities, so its traced layer
# outputs are the attention and DeltaNet results (tests/golden/make_golden.py hybrid_kernel_case).

MIRROR_LAYERS = ["hd64", "hd256"]


def mirror_layers(name):
    return load(os.path.join(GOLDEN, f"mirror_layers_{name}.npz"))


def _scale_err(got, want):
    return float(np.abs(np.asarray(got, np.float64) - want).max() / max(1.0, float(np.abs(want).max())))


@pytest.mark.parametrize("name", MIRROR_LAYERS)
def test_attention_oracle_matches_the_mirror(name):
    """oracle/ref.attn_decode step by step against the mirror's attention (model/mirror.py:945-996):
    with fp32 cache rows the oracle follows the mirror to 1e-5 of the output scale; with the build's
    fp16 cache to 1e-3."""
    d = mirror_layers(name)
    H, Hkv, hd, eps = int(d["n_head"]), int(d["n_kv"]), int(d["head_dim"]), float(d["eps"])
    gated, freq, npos = bool(d["gated"]), d["rope_freq"], int(d["npos"])
    n = 0
    for l, dn in enumerate(d["layer_types"]):
        if dn:
            continue
        qn, kn = d[f"l{l}_q_norm"], d[f"l{l}_k_norm"]
        k32 = np.zeros((npos, Hkv, hd), np.float32)
        v32 = np.zeros_like(k32)
        k16 = np.zeros((npos, Hkv, hd), np.float16)
        v16 = np.zeros_like(k16)
        for p in range(npos):
            qm = d[f"l{l}_q"][p].reshape(H, -1)
            q, gate = qm[:, :hd].copy(), (qm[:, hd:].copy() if gated else None)
            k, v = d[f"l{l}_k"][p].reshape(Hkv, hd), d[f"l{l}_v"][p].reshape(Hkv, hd)
            rows32 = (np.stack([ref.rope_neox(ref.rmsnorm(k[h], kn, eps), p, freq) for h in range(Hkv)]),
                      v.astype(np.float32))
            o32 = ref.attn_decode(q, k, v, k32, v32, p, qn, kn, eps, freq, gate=gate, rows=rows32)
            o16 = ref.attn_decode(q, k, v, k16, v16, p, qn, kn, eps, freq, gate=gate)
            want = d[f"l{l}_out"][p]
            assert _scale_err(o32.reshape(-1), want) <= 1e-5, (l, p)
            assert _scale_err(o16.reshape(-1), want) <= 1e-3, (l, p)
            n += 1
    assert n > 0


@pytest.mark.parametrize("name", MIRROR_LAYERS)
def test_deltanet_oracle_matches_the_mirror(name):
    """oracle/ref.deltanet_step from a zero state, step by step, against the mirror's DeltaNet
    (model/mirror.py:892-943): the grouped-order gated-norm output to 1e-4 of its scale (the mirror
    sums in sequence, the oracle with numpy's matmul)."""
    d = mirror_layers(name)
    nk, hk, nv, hv, K = (int(d[k]) for k in ("nk", "hk", "nv", "hv", "conv"))
    eps = float(d["eps"])
    C = 2 * nk * hk + nv * hv
    n = 0
    for l, dn in enumerate(d["layer_types"]):
        if not dn:
            continue
        win = np.zeros((K - 1, C), np.float32)
        S = np.zeros((nv, hv, hk), np.float32)
        for p in range(int(d["npos"])):
            og = ref.deltanet_step(d[f"l{l}_qkv"][p], d[f"l{l}_z"][p], d[f"l{l}_beta"][p], d[f"l{l}_alpha"][p],
                                   d[f"l{l}_dt_bias"], d[f"l{l}_ssm_a"], d[f"l{l}_conv_w"].reshape(C, K), win, S,
                                   d[f"l{l}_ssm_norm"], eps, nk, hk, nv, hv)
            assert _scale_err(og, d[f"l{l}_out"][p]) <= 1e-4, (l, p)
            n += 1
    assert n > 0


# K-segmented projections (model/bons.py:83-113 split_wide; model/mirror.py:664-678) --------------

KSEG = ["t5_24x17408", "2b_40x17408", "q8_20x9216"]


def kseg_segments(d):
    out = []
    kind, rows = int(d["kind"]), int(d["rows"])
    for k in range(int(d["nseg"])):
        cols = int(d[f"cols{k}"])
        if kind == L.KIND_Q8:
            s, v = ref.q8_decode_packed(d[f"packed{k}"], rows, cols)
        else:
            s, v = ref.decode_packed(d[f"packed{k}"], rows, cols, kind)
        out.append((kind, s, v))
    return out


@pytest.mark.parametrize("name", KSEG)
def test_kseg_oracle_bit_exact(name):
    """The oracle's K-segmented float projection against the mirror's, fp32 bits."""
    d = load(os.path.join(GOLDEN, f"kseg_{name}.npz"))
    y = ref.matvec_f_kseg(kseg_segments(d), d["x"], int(d["B"]), int(d["R"]))
    assert np.array_equal(y.view(np.uint32), d["y"].view(np.uint32))
    # One segment-wide shift per segment is not one shift of the whole sum: the unsegmented
    # projection of the same weights differs in the low bits somewhere.
    if int(d["kind"]) != L.KIND_Q8:
        segs = kseg_segments(d)
        s = np.concatenate([a[1] for a in segs], axis=1)
        c = np.concatenate([a[2] for a in segs], axis=1)
        whole = ref.matvec_f(s, c, d["x"], int(d["B"]), int(d["R"]))
        assert not np.array_equal(whole.view(np.uint32), d["y"].view(np.uint32))


def test_int_deltanet_oracle_pinned():
    """oracle/ref.py dn_head_step against the reference's own head_step (model/deltanet.py:99-147)
    over the token schedule of test/model/test_asm.py:554-590: state, exponent, max and output
    bit-exact, the ratchet firing on the first tokens and not on the last."""
    d = load(os.path.join(GOLDEN, "dn_int_steps.npz"))
    for hv, hk, seed in d["shapes"]:
        tag = f"h{hv}x{hk}s{seed}"
        M = np.zeros((hv, hk), dtype=np.int64)
        for t in range(4):
            g = lambda n: d[f"{tag}_t{t}_{n}"]
            o, eM2, maxM2, bad = ref.dn_head_step(M, int(g("eM")), g("k"), g("q"), g("v"), g("decay"), g("beta"),
                                                  maxM=int(g("maxM")))
            assert not bad
            assert np.array_equal(M, g("M").astype(np.int64)), (tag, t)
            assert (eM2, maxM2) == (int(g("eM2")), int(g("maxM2")))
            assert np.array_equal(o.view(np.uint32), g("o").view(np.uint32))
            if t == 0:
                assert eM2 > -20  # the empty -20 state ratchets on the first update
        assert eM2 == int(d[f"{tag}_t2_eM2"])  # the small last update does not ratchet
