"""Host-side packing of ternary tensors into the converter's row-packet layout, and the
per-tensor fixed-point contract (scale bias B, result shift R).

Everything here is the converter's side of the drop-in boundary, written for this package:

* `pack_rows` produces, byte for byte, what `model/bons.py:encode_rows` (:150-175) emits for
  KIND_TERNARY and KIND_TERNARY5 tensors; `unpack_rows` is its inverse
  (`model/bons.py:decode_rows`, :177-200).  Equality with the reference is pinned by the
  golden fixtures in tests/golden.
* `scale_bias` / `result_shift` restate `model/bitexact.py:choose_scale_bias` (:77-80) and
  `choose_result_shift` (:91-97) with `tensor_acc_bound` (:82-89); `model/bons.py:62-65`
  applies them per tensor.
* `synthetic_tensor` draws the benchmark distribution (codes with P(w=0)=0.4, P(+1)=P(-1)=0.3,
  scales |N(0,1)|*0.02 as fp16), one `numpy.random.default_rng(seed)` drawing codes, then
  scales, then the activation.
"""

import numpy as np

from . import layout as L

_POW3 = np.array([1, 3, 9, 27, 81], dtype=np.uint16)


def _trit5_bytes(codes):
    """(rows, cols) digits {0,1,2} -> (rows, 26*G) bytes; lane 5i+k is digit k of byte i."""
    rows, cols = codes.shape
    g = L.groups(cols)
    lanes = np.zeros((rows, g, 130), dtype=np.uint16)
    lanes[:, :, :128] = codes.reshape(rows, g, 128)
    return (lanes.reshape(rows, g, 26, 5) * _POW3).sum(axis=3).astype(np.uint8).reshape(rows, -1)


def _twobit_bytes(codes):
    """(rows, cols) codes -> (rows, cols/4) bytes; code j at bits 2*(j%4) of byte j//4."""
    rows, cols = codes.shape
    c = codes.astype(np.uint8).reshape(rows, cols // 4, 4)
    return (c[..., 0] | (c[..., 1] << 2) | (c[..., 2] << 4) | (c[..., 3] << 6)).astype(np.uint8)


def pack_rows(scales, codes, kind):
    """scales (rows, G) fp16, codes (rows, cols) uint8 in {0,1,2} -> packed uint8
    (rows * row_bytes,)."""
    codes = np.asarray(codes)
    rows, cols = codes.shape
    g = L.groups(cols)
    scales = np.ascontiguousarray(np.asarray(scales, dtype=np.float16).reshape(rows, g))
    rb = L.row_bytes(cols, kind)
    sb = L.scale_bytes(cols)
    out = np.zeros((rows, rb), dtype=np.uint8)
    out[:, :2 * g] = scales.view(np.uint8).reshape(rows, 2 * g)
    body = _trit5_bytes(codes) if kind == L.KIND_TERNARY5 else _twobit_bytes(codes)
    out[:, sb:sb + body.shape[1]] = body
    return out.reshape(-1)


def unpack_rows(packed, rows, cols, kind):
    """Inverse of pack_rows -> (scales fp16 (rows, G), codes uint8 (rows, cols)).
    Invalid trit5 bytes (> 242) decode digit by digit like the reference reader does."""
    g = L.groups(cols)
    rb = L.row_bytes(cols, kind)
    data = np.asarray(packed, dtype=np.uint8).reshape(rows, rb)
    scales = data[:, :2 * g].copy().view(np.float16)
    body = data[:, L.scale_bytes(cols):]
    if kind == L.KIND_TERNARY5:
        b = body[:, :26 * g].astype(np.uint16).reshape(rows, g, 26, 1)
        d = (b // _POW3) % 3
        codes = d.reshape(rows, g, 130)[:, :, :128].reshape(rows, cols).astype(np.uint8)
    else:
        q = body[:, :cols // 4]
        codes = np.stack([(q >> (2 * j)) & 3 for j in range(4)], axis=-1).reshape(rows, cols)
    return scales, codes.astype(np.uint8)


# Fixed-point contract ---------------------------------------------------------------------------

def fp16_split(scales):
    """fp16 -> (m11, e16) with value = m11 * 2**e16 exactly (model/bitexact.py:56-68).
    Normal: m11 = +-(1024 + frac), e16 = E - 25; subnormal/zero: m11 = +-frac, e16 = -24."""
    bits = np.asarray(scales, dtype=np.float16).view(np.uint16).astype(np.int64)
    E = (bits >> 10) & 0x1F
    if np.any(E == 0x1F):
        raise ValueError("fp16 inf/nan in scales")
    frac = bits & 0x3FF
    mag = np.where(E > 0, frac + 1024, frac)
    m11 = np.where(bits & 0x8000, -mag, mag)
    e16 = np.where(E > 0, E - 25, -24)
    return m11, e16


def scale_bias(scales, target_top=12):
    _, e16 = fp16_split(scales)
    return int(target_top - e16.max())


def result_shift(scales, bias, gs_max=128 * 127):
    """Smallest R with (worst-case |acc|) >> R inside int32."""
    m11, e16 = fp16_split(scales)
    per_group = np.abs(m11).astype(np.float64) * gs_max * np.exp2((e16 + bias).astype(np.float64))
    bound = np.ceil(per_group).sum(axis=-1).max()
    r = 0
    while bound / float(1 << r) >= 2.0 ** 31:
        r += 1
    return r


class TernaryTensor:
    """One packed ternary tensor: its bytes and the entry fields the kernels need
    (the BONS entry's kind/rows/cols/bias/rshift, model/layout.py:311-333)."""

    def __init__(self, scales, codes, kind=L.KIND_TERNARY5, bias=None, rshift=None):
        codes = np.asarray(codes, dtype=np.uint8)
        self.rows, self.cols = codes.shape
        self.kind = kind
        self.scales = np.asarray(scales, dtype=np.float16).reshape(self.rows, -1)
        self.codes = codes
        self.bias = scale_bias(self.scales) if bias is None else int(bias)
        self.rshift = result_shift(self.scales, self.bias) if rshift is None else int(rshift)
        self.packed = pack_rows(self.scales, codes, kind)

    @property
    def row_bytes(self):
        return L.row_bytes(self.cols, self.kind)

    def as_kind(self, kind):
        return TernaryTensor(self.scales, self.codes, kind, self.bias, self.rshift)


GS_MAX_Q8 = 32 * 127 * 127   # max |group sum| of a Q8 row dot (model/bitexact.py:73)


def pack_q8_rows(scales, q8w):
    """scales (rows, cols/32) fp16, q8w (rows, cols) int8 -> KIND_Q8 row packets (uint8), byte for
    byte model/bons.py:encode_rows (:150-154, :167-169)."""
    q8w = np.asarray(q8w, dtype=np.int8)
    rows, cols = q8w.shape
    g = L.q8_groups(cols)
    sb = L.ceil_div(g, L.SCALES_PER_BEAT) * L.BEAT_BYTES
    out = np.zeros((rows, L.q8_row_bytes(cols)), dtype=np.uint8)
    sc = np.ascontiguousarray(np.asarray(scales, dtype=np.float16).reshape(rows, g))
    out[:, :2 * g] = sc.view(np.uint8).reshape(rows, 2 * g)
    out[:, sb:] = np.ascontiguousarray(q8w).view(np.uint8)
    return out.reshape(-1)


class Q8Tensor:
    """One packed KIND_Q8 tensor (group 32, w = q * scale): its bytes and entry fields.  B and R
    follow the converter (model/bons.py:56-65 with GS_MAX_Q8) unless given."""

    def __init__(self, scales, q8w, bias=None, rshift=None):
        q8w = np.asarray(q8w, dtype=np.int8)
        self.rows, self.cols = q8w.shape
        self.kind = L.KIND_Q8
        self.scales = np.asarray(scales, dtype=np.float16).reshape(self.rows, -1)
        self.q8w = q8w
        self.bias = scale_bias(self.scales) if bias is None else int(bias)
        self.rshift = result_shift(self.scales, self.bias, GS_MAX_Q8) if rshift is None else int(rshift)
        self.packed = pack_q8_rows(self.scales, q8w)

    @property
    def row_bytes(self):
        return L.q8_row_bytes(self.cols)


def hadamard_tensor(signs, block, kind=L.KIND_TERNARY):
    """The rotation x' = R(s*x) per block (PrismML's basis) as the converter stores it
    (model/convert.py:99-118): per block b a block x block ternary tensor with codes
    H[i, j]*s[b*block + j] + 1, H the +-1 Sylvester-Hadamard matrix ((-1)^popcount(i & j),
    model/golden.py:256-263) and every scale 2^-floor(log2(block)/2) (model/golden.py:271-278).
    The blocks are stacked into one TernaryTensor of width rows (every block has the same scales,
    so the converter's B and R are the same for all of them)."""
    signs = np.asarray(signs)
    width = signs.size
    if block & (block - 1) or block < L.GROUP or width % block:
        raise ValueError(f"block {block} must be a power of two >= {L.GROUP} dividing width {width}")
    i = np.arange(block)
    par = np.bitwise_and(i[:, None], i[None, :])
    odd = np.zeros_like(par)
    while par.any():
        odd ^= par & 1
        par >>= 1
    H = (1 - 2 * odd).astype(np.int16)
    s = np.where(signs.reshape(-1, block) < 0, -1, 1).astype(np.int16)
    codes = (H[None, :, :] * s[:, None, :] + 1).reshape(width, block).astype(np.uint8)
    k = block.bit_length() - 1
    scales = np.full((width, block // L.GROUP), 2.0 ** -(k // 2), dtype=np.float16)
    return TernaryTensor(scales, codes, kind=kind)


def synthetic_codes_scales(rng, rows, cols, p_zero=0.4, scale_sigma=0.02):
    """Codes {0,1,2} with P(code 1, w=0)=p_zero and P(code 0)=P(code 2)=(1-p_zero)/2, then
    fp16 scales |N(0,1)|*scale_sigma per 128-group."""
    u = rng.random((rows, cols))
    half = (1.0 - p_zero) / 2.0
    codes = np.where(u < half, 0, np.where(u < half + p_zero, 1, 2)).astype(np.uint8)
    scales = (np.abs(rng.standard_normal((rows, cols // L.GROUP))) * scale_sigma).astype(np.float16)
    return codes, scales


def synthetic_matvec_case(rows, cols, seed=0, kind=L.KIND_TERNARY5):
    """The single-matvec benchmark case: (TernaryTensor, x fp32)."""
    rng = np.random.default_rng(seed)
    codes, scales = synthetic_codes_scales(rng, rows, cols)
    x = rng.standard_normal(cols).astype(np.float32)
    return TernaryTensor(scales, codes, kind), x


# Device-side generation (benchmark set-up; not on the timed path) --------------------------------

def pack_rows_torch(scales, codes, kind):
    """torch version of pack_rows for CUDA tensors: scales (rows, G) fp16, codes (rows, cols)
    uint8 -> packed uint8 (rows * row_bytes,) on the same device.  Byte-identical to pack_rows."""
    import torch
    rows, cols = codes.shape
    g = L.groups(cols)
    rb, sb = L.row_bytes(cols, kind), L.scale_bytes(cols)
    out = torch.zeros(rows, rb, dtype=torch.uint8, device=codes.device)
    out[:, :2 * g] = scales.contiguous().view(torch.uint8).reshape(rows, 2 * g)
    if kind == L.KIND_TERNARY5:
        lanes = torch.zeros(rows, g, 130, dtype=torch.int16, device=codes.device)
        lanes[:, :, :128] = codes.reshape(rows, g, 128).to(torch.int16)
        pw = torch.tensor([1, 3, 9, 27, 81], dtype=torch.int16, device=codes.device)
        body = (lanes.reshape(rows, g, 26, 5) * pw).sum(dim=3).to(torch.uint8).reshape(rows, 26 * g)
    else:
        c = codes.reshape(rows, cols // 4, 4).to(torch.uint8)
        body = c[..., 0] | (c[..., 1] << 2) | (c[..., 2] << 4) | (c[..., 3] << 6)
    out[:, sb:sb + body.shape[1]] = body
    return out.reshape(-1)


def synthetic_codes_scales_torch(gen, rows, cols, device, p_zero=0.4, scale_sigma=0.02):
    """Device draw of the benchmark distribution (torch.Generator `gen`)."""
    import torch
    u = torch.rand(rows, cols, generator=gen, device=device)
    half = (1.0 - p_zero) / 2.0
    codes = torch.where(u < half, 0, torch.where(u < half + p_zero, 1, 2)).to(torch.uint8)
    scales = (torch.randn(rows, cols // L.GROUP, generator=gen, device=device).abs() * scale_sigma).to(torch.float16)
    return codes, scales
