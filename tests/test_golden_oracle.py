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
