"""numpy restatement of the reference's ternary decode-path numerics.  TEST INFRASTRUCTURE ONLY.

Each function cites the reference lines it restates (paths relative to the TriXium tree).
Nothing on the product path may import this module.
"""

import numpy as np

f32 = np.float32
POW3 = np.array([1, 3, 9, 27, 81], dtype=np.int64)


# Row packets ------------------------------------------------------------------------------------

def row_bytes(cols, kind):
    """model/layout.py:189-217: ceil(G/16) scale beats + code beats (trit5: 26 B/group, padded)."""
    g = cols // 128
    sb = -(-g // 16) * 32
    cb = 26 * g if kind == 5 else 32 * g
    return sb + -(-cb // 32) * 32


def decode_packed(packed, rows, cols, kind):
    """model/bons.py:177-200 (decode_rows) with trit5_unpack_rows (:125-130):
    packed bytes -> (scales fp16 (rows,G), codes uint8 (rows,cols))."""
    g = cols // 128
    rb = row_bytes(cols, kind)
    d = np.frombuffer(np.asarray(packed, dtype=np.uint8).tobytes(), dtype=np.uint8).reshape(rows, rb)
    scales = d[:, :2 * g].copy().view(np.float16)
    body = d[:, -(-g // 16) * 32:].astype(np.int64)
    if kind == 5:
        b = body[:, :26 * g].reshape(rows, g, 26, 1)
        digits = (b // POW3) % 3
        codes = digits.reshape(rows, g, 130)[:, :, :128].reshape(rows, cols)
    else:
        q = body[:, :cols // 4]
        codes = np.stack([(q >> s) & 3 for s in (0, 2, 4, 6)], axis=-1).reshape(rows, cols)
    return scales, codes.astype(np.uint8)


def trit5_invalid(packed, rows, cols):
    """Bytes above 242 in the code groups (gateware/core/trit5.py:37-39 flags them)."""
    g = cols // 128
    rb = row_bytes(cols, 5)
    d = np.asarray(packed, dtype=np.uint8).reshape(rows, rb)
    body = d[:, -(-g // 16) * 32:][:, :26 * g]
    return int((body > 242).sum())


# Integer engine ---------------------------------------------------------------------------------

def fp16_parts(s):
    """model/bitexact.py:56-68: fp16 = m11 * 2**e16 exactly."""
    u = np.asarray(s, dtype=np.float16).view(np.uint16).astype(np.int64)
    e = (u >> 10) & 31
    assert not np.any(e == 31), "fp16 inf/nan in scales"
    m = np.where(e > 0, (u & 1023) | 1024, u & 1023)
    return np.where(u >> 15, -m, m), np.where(e > 0, e - 25, -24)


class OverflowError48(ArithmeticError):
    pass


def matvec_int(scales, codes, x8, B, R):
    """model/bitexact.py:101-119 (matvec_ternary): exact group sums of (code-1)*x8, each times
    m11 and shifted by e16+B (floor shift when negative), summed in int64, then >> R.
    Raises OverflowError48 where the reference asserts (:116, :118)."""
    rows, cols = codes.shape
    g = cols // 128
    w = codes.astype(np.int64).reshape(rows, g, 128) - 1
    gs = np.einsum("rgk,gk->rg", w, np.asarray(x8, dtype=np.int64).reshape(g, 128))
    m11, e16 = fp16_parts(scales)
    sh = e16 + B
    prod = gs * m11
    contrib = np.where(sh >= 0, prod << np.clip(sh, 0, 63), prod >> np.clip(-sh, 0, 63))
    acc = contrib.sum(axis=1)
    if np.any(np.abs(acc) >= 2 ** 47):
        raise OverflowError48("int48 accumulator overflow")
    res = acc >> R
    if np.any(np.abs(res) >= 2 ** 31):
        raise OverflowError48("int32 result overflow")
    return res.astype(np.int32)


def q8_row_bytes(cols):
    """model/layout.py:189-217 for KIND_Q8: ceil(G/16) scale beats + G code beats, G = cols/32."""
    g = cols // 32
    return -(-g // 16) * 32 + 32 * g


def q8_decode_packed(packed, rows, cols):
    """model/bons.py:177-200 (decode_rows) for KIND_Q8 -> (scales fp16 (rows,G), q8w int8)."""
    g = cols // 32
    d = np.asarray(packed, dtype=np.uint8).reshape(rows, q8_row_bytes(cols))
    return d[:, :2 * g].copy().view(np.float16), d[:, -(-g // 16) * 32:].copy().view(np.int8)


def q8_pack(scales, q8w):
    """model/bons.py:132-160 (encode_rows) for KIND_Q8: scales then the int8 weights per row."""
    rows, cols = q8w.shape
    g = cols // 32
    out = np.zeros((rows, q8_row_bytes(cols)), dtype=np.uint8)
    out[:, :2 * g] = np.ascontiguousarray(np.asarray(scales, np.float16)).view(np.uint8).reshape(rows, 2 * g)
    out[:, -(-g // 16) * 32:] = np.asarray(q8w, np.int8).view(np.uint8)
    return out.reshape(-1)


def matvec_q8(scales, q8w, x8, B, R):
    """model/bitexact.py:127-144 (matvec_q8): exact sums of q8w*x8 over groups of 32, each times
    m11 and shifted by e16+B (floor shift when negative), summed in int64, then >> R.
    Raises OverflowError48 where the reference asserts (:141, :143)."""
    rows, cols = q8w.shape
    g = cols // 32
    gs = np.einsum("rgk,gk->rg", np.asarray(q8w, np.int64).reshape(rows, g, 32),
                   np.asarray(x8, dtype=np.int64).reshape(g, 32))
    m11, e16 = fp16_parts(scales)
    sh = e16 + B
    prod = gs * m11
    acc = np.where(sh >= 0, prod << np.clip(sh, 0, 63), prod >> np.clip(-sh, 0, 63)).sum(axis=1)
    if np.any(np.abs(acc) >= 2 ** 47):
        raise OverflowError48("int48 accumulator overflow")
    res = acc >> R
    if np.any(np.abs(res) >= 2 ** 31):
        raise OverflowError48("int32 result overflow")
    return res.astype(np.int32)


def group_sums(codes, x8):
    """The exact per-(row, group) sums gs (model/bitexact.py:108)."""
    rows, cols = codes.shape
    g = cols // 128
    w = codes.astype(np.int64).reshape(rows, g, 128) - 1
    return np.einsum("rgk,gk->rg", w, np.asarray(x8, dtype=np.int64).reshape(g, 128))


# Activation quantisation ------------------------------------------------------------------------

def lround_mirror(x):
    """model/mirror.py:34-35 (_lroundf) on fp32 input: floor(x + 0.5) for x >= 0 and
    ceil(x - 0.5) below, the +-0.5 added IN FP32 (numpy keeps the fp32 dtype), so x = 0.5-2**-25
    rounds to 1."""
    x = np.asarray(x, dtype=f32)
    up = np.floor((x + f32(0.5)).astype(f32))
    dn = np.ceil((x - f32(0.5)).astype(f32))
    return np.where(x >= 0, up, dn).astype(np.int64)


def quantize_pow2(x):
    """model/mirror.py:45-51 (_quantize_f_pow2) = firmware f32_quant_e8/f32_pack_q8x4
    (firmware/infer_internal.h:60-124): e8 = frexp(amax)[1] - 7, q = clip(lround(x*2**-e8))."""
    x = np.asarray(x, dtype=f32)
    amax = np.abs(x).max() if x.size else f32(0)
    if amax == 0:
        return np.zeros(x.shape, dtype=np.int8), 0
    e8 = int(np.frexp(f32(amax))[1]) - 7
    q = lround_mirror((x * f32(np.exp2(-e8))).astype(f32))
    return np.clip(q, -127, 127).astype(np.int8), e8


def matvec_f(scales, codes, x, B, R):
    """model/mirror.py:648-678 (matvec_f, quantised mode, one K-segment): quantise x, the
    engine's int32 result, scaled by fp32 2**(e8+R-B)."""
    x8, e8 = quantize_pow2(x)
    res = matvec_int(scales, codes, x8, B, R)
    sc = f32(np.exp2(f32(e8 + R - B)))
    return (res.astype(f32) * sc).astype(f32)


def matvec_q8_f(scales, q8w, x, B, R):
    """model/mirror.py:664-678 for a KIND_Q8 tensor (the :672-675 branch, one K-segment): quantise
    x, the engine's Q8 int32 result, scaled by fp32 2**(e8+R-B)."""
    x8, e8 = quantize_pow2(x)
    res = matvec_q8(scales, q8w, x8, B, R)
    return (res.astype(f32) * f32(np.exp2(f32(e8 + R - B)))).astype(f32)


def matvec_f_kseg(segments, x, B, R):
    """model/mirror.py:664-678 over K-segments (FLAG_KSEG, model/bons.py:83-113): quantise the whole
    x once, per segment the engine's int32 result on its column range (segments: (kind, scales,
    values) in order; ternary codes or Q8 weights), the int64 sum wrapped to int32, times
    fp32 2**(e8+R-B)."""
    x8, e8 = quantize_pow2(x)
    res, c0 = np.zeros(segments[0][2].shape[0], dtype=np.int64), 0
    for kind, scales, values in segments:
        cols = values.shape[1]
        xs = x8[c0:c0 + cols]
        r = matvec_q8(scales, values, xs, B, R) if kind == 1 else matvec_int(scales, values, xs, B, R)
        res += r.astype(np.int64)
        c0 += cols
    return (res.astype(np.int32).astype(f32) * f32(np.exp2(f32(e8 + R - B)))).astype(f32)


def hadamard_codes(signs, block):
    """model/convert.py:99-118 with model/golden.py:256-263: block tensor b of the rotation has
    codes H[i, j] * s[b*block + j] + 1, H[i, j] = (-1)^popcount(i & j); its scales are all
    2^-floor(log2(block)/2) (model/golden.py:271-278).  Returns (scales, codes) of all blocks
    stacked: (width, block/128) fp16 and (width, block) uint8."""
    i = np.arange(block)
    par = i[:, None] & i[None, :]
    bits = np.zeros_like(par)
    while par.any():
        bits ^= par & 1
        par >>= 1
    H = np.where(bits & 1, -1, 1).astype(np.int64)
    s = np.asarray(signs).astype(np.int64).reshape(-1, block)
    codes = (H[None, :, :] * s[:, None, :] + 1).reshape(-1, block).astype(np.uint8)
    k = block.bit_length() - 1
    scales = np.full((codes.shape[0], block // 128), 2.0 ** -(k // 2), np.float16)
    return scales, codes


def hadamard_rotate(x, scales, codes, B, R):
    """model/mirror.py:680-690 (rotate): block b of x' = matvec_f(block tensor b, x[b-th block])."""
    block = codes.shape[1]
    return np.concatenate([matvec_f(scales[b:b + block], codes[b:b + block], x[b:b + block], B, R)
                           for b in range(0, len(x), block)])


def matvec_f64(scales, codes, x):
    """fp64 reference of the fp projection: sum over groups of scale * sum((code-1)*x)
    (the float reference of test/model/test_bitexact.py:49-56, and model/fastref.py:119-125
    without its fp32 rounding)."""
    rows, cols = codes.shape
    g = cols // 128
    w = codes.astype(np.float64).reshape(rows, g, 128) - 1.0
    gs = np.einsum("rgk,gk->rg", w, np.asarray(x, dtype=np.float64).reshape(g, 128))
    return (gs * np.asarray(scales, dtype=np.float64)).sum(axis=1)


def matvec_fastref(scales, codes, X):
    """model/fastref.py:103-125: fp16 weight cache (code-1)*scale, X @ W.T in fp32."""
    rows, cols = codes.shape
    W = ((codes.astype(f32).reshape(rows, -1, 128) - f32(1.0))
         * np.asarray(scales, dtype=np.float16).astype(f32)[:, :, None]).reshape(rows, cols)
    W = W.astype(np.float16).astype(f32)
    return np.atleast_2d(np.asarray(X, dtype=f32)) @ W.T


# Canonical reductions (model/mirror.py:576-591, doc/units.md canonical sum64) -------------------

def sumsq64(v):
    """model/mirror.py:576-591: 64 strided fp32 partials, then the halving tree."""
    v = np.asarray(v, dtype=f32)
    sq = (v * v).astype(f32)
    n = len(sq)
    P = np.zeros(64, dtype=f32)
    full = n // 64 * 64
    for r in range(0, full, 64):
        P = (P + sq[r:r + 64]).astype(f32)
    if n - full:
        P[:n - full] = (P[:n - full] + sq[full:]).astype(f32)
    w = 32
    while w:
        P[:w] = (P[:w] + P[w:2 * w]).astype(f32)
        w //= 2
    return P[0]


def rmsnorm(x, w, eps):
    """model/mirror.py:697-700: r = 1/sqrt(ss/n + eps) (fp32 ops), (x*r)*w."""
    x = np.asarray(x, dtype=f32)
    ss = sumsq64(x)
    r = f32(1.0) / f32(np.sqrt(f32(f32(ss / f32(len(x))) + f32(eps))))
    return ((x * r).astype(f32) * np.asarray(w, dtype=f32)).astype(f32)


def l2norm(x, eps):
    """model/mirror.py:702-705: x * (1/max(sqrt(ss), eps))."""
    x = np.asarray(x, dtype=f32)
    nrm = f32(np.sqrt(sumsq64(x)))
    nrm = max(nrm, f32(eps))
    return (x * f32(f32(1) / nrm)).astype(f32)


def silu(x):
    """model/mirror.py:713 (mathematical profile): x / (1 + exp(-x)) in fp32."""
    x = np.asarray(x, dtype=f32)
    return (x / (f32(1.0) + np.exp(-x, dtype=f32))).astype(f32)


def sigmoid(x):
    x = np.asarray(x, dtype=f32)
    return (f32(1.0) / (f32(1.0) + np.exp(-x, dtype=f32))).astype(f32)


def argmax_first(v):
    """Greedy argmax, ties to the smallest index (doc/units.md:149)."""
    return int(np.argmax(np.asarray(v)))


# Decode attention --------------------------------------------------------------------------------

def rope_freq(rope_n, theta):
    """model/mirror.py:754: theta^(-2i/rope_n) per pair, in fp32."""
    return np.array([f32(f32(theta) ** f32(-2.0 * i / rope_n)) for i in range(rope_n // 2)], dtype=f32)


def rope_neox(vh, pos, freq):
    """model/mirror.py:956-961: neox pairs (i, i + rope_n/2) over the first rope_n dims, cos/sin of
    fp32(pos * freq) in fp32; the rest passes through."""
    vh = np.array(vh, dtype=f32)
    half = len(freq)
    ang = (f32(pos) * freq).astype(f32)
    c, s = np.cos(ang, dtype=f32), np.sin(ang, dtype=f32)
    x0, x1 = vh[:half].copy(), vh[half:2 * half].copy()
    vh[:half] = (x0 * c - x1 * s).astype(f32)
    vh[half:2 * half] = (x0 * s + x1 * c).astype(f32)
    return vh


def attn_new_rows(k, v, pos, kn_w, eps, freq):
    """model/mirror.py:963-965: this token's cache rows, RMSNorm'd and RoPE'd k and v, rounded to
    fp16 (the build's cache type)."""
    kn = np.stack([rope_neox(rmsnorm(k[h], kn_w, eps), pos, freq) for h in range(k.shape[0])])
    return kn.astype(np.float16), np.asarray(v, dtype=f32).astype(np.float16)


def attn_decode(q, k, v, kcache, vcache, pos, qn_w, kn_w, eps, freq, gate=None, rows=None):
    """One decode step of GQA attention (model/mirror.py:945-996; model/golden.py:361-398).

    q (H, hd), k/v (Hkv, hd) fp32: this token's projections (gate (H, hd) or None).
    kcache/vcache (T, Hkv, hd) fp16: positions [0, pos) already filled; this step writes
    position pos (attn_new_rows, or `rows` = (k_row, v_row) given).
    Returns out (H, hd) fp32; kcache/vcache updated in place."""
    H, hd = q.shape
    Hkv = k.shape[0]
    rep = H // Hkv
    qn = np.stack([rope_neox(rmsnorm(q[h], qn_w, eps), pos, freq) for h in range(H)])
    kcache[pos], vcache[pos] = rows if rows is not None else attn_new_rows(k, v, pos, kn_w, eps, freq)
    T = pos + 1
    K = kcache[:T].astype(f32)
    V = vcache[:T].astype(f32)
    scale = f32(1.0 / np.sqrt(hd))
    out = np.zeros((H, hd), dtype=f32)
    for h in range(H):
        kvh = h // rep
        sc = ((K[:, kvh, :] @ qn[h]).astype(f32) * scale).astype(f32)
        ex = np.exp((sc - sc.max()).astype(f32), dtype=f32)
        inv = f32(f32(1) / ex.sum(dtype=f32))
        o = ((ex * inv).astype(f32) @ V[:, kvh, :]).astype(f32)
        if gate is not None:
            o = (o * sigmoid(gate[h])).astype(f32)
        out[h] = o
    return out


# Gated DeltaNet step -----------------------------------------------------------------------------

def softplus(x):
    """model/mirror.py:714: x for x > 20, else log1p(exp(x)), in fp32."""
    x = np.asarray(x, dtype=f32)
    return np.where(x > 20, x, np.log1p(np.exp(x, dtype=f32), dtype=f32)).astype(f32)


def deltanet_step(qkv, z, beta_raw, alpha, dt_bias, ssm_a, conv_w, win, S, norm_w, eps, nk, hk, nv, hv):
    """One decode step of a gated-DeltaNet layer after its projections (model/mirror.py:892-943,
    mathematical profile; model/golden.py:400-434).

    qkv (2*nk*hk + nv*hv), z (nv*hv), beta_raw/alpha (nv) fp32: this token's projections;
    dt_bias, ssm_a (nv); conv_w (C, K); win (K-1, C): the previous K-1 conv inputs, oldest
    first; S (nv, hv, hk): the recurrent state.  win and S are updated in place.
    Returns og (nv*hv): RMSNorm(o_h)*silu(z_h) per value head, in the grouped head order
    (value head h at position (h % nk)*(nv/nk) + h // nk, mirror.py:941-942)."""
    nq = nk * hk
    C = 2 * nq + nv * hv
    K = conv_w.shape[1]
    beta = sigmoid(np.asarray(beta_raw, dtype=f32))
    g = (softplus(np.asarray(alpha, dtype=f32) + np.asarray(dt_bias, dtype=f32)) * np.asarray(ssm_a, dtype=f32)).astype(f32)
    conv = np.empty(C, dtype=f32)
    for c in range(C):
        acc = f32(0.0)
        for i in range(K - 1):
            acc = f32(acc + f32(conv_w[c, i] * win[i, c]))
        conv[c] = f32(acc + f32(conv_w[c, K - 1] * qkv[c]))
    conv = silu(conv)
    win[:-1] = win[1:]
    win[-1] = qkv
    q = conv[:nq].copy()
    k = conv[nq:2 * nq].copy()
    v = conv[2 * nq:].copy()
    for h in range(nk):
        q[h * hk:(h + 1) * hk] = l2norm(q[h * hk:(h + 1) * hk], eps)
        k[h * hk:(h + 1) * hk] = l2norm(k[h * hk:(h + 1) * hk], eps)
    rep = nv // nk
    scale = f32(1.0 / np.sqrt(hk))
    og = np.zeros(nv * hv, dtype=f32)
    for h in range(nv):
        kh = h % nk
        qh, kk, vh = q[kh * hk:(kh + 1) * hk], k[kh * hk:(kh + 1) * hk], v[h * hv:(h + 1) * hv]
        decay = f32(np.exp(f32(g[h]), dtype=f32))
        M = S[h]
        M *= decay
        delta = ((vh - (M @ kk).astype(f32)).astype(f32) * f32(beta[h])).astype(f32)
        M += (delta[:, None] * kk[None, :]).astype(f32)
        oh = ((M @ qh).astype(f32) * scale).astype(f32)
        gpos = kh * rep + h // nk
        og[gpos * hv:(gpos + 1) * hv] = (rmsnorm(oh, norm_w, eps) * silu(z[h * hv:(h + 1) * hv])).astype(f32)
    return og


# Integer DeltaNet head step (model/deltanet.py) ----------------------------------------------------

DN_DELTA_FRAC = 19            # model/deltanet.py:49 (delta, -v and the decayed dot in units of 2^-19)
DN_O_SHIFT = 8                # model/deltanet.py:50
DN_STATE_LIM = (1 << 15) - 4  # model/deltanet.py:51


def lroundf64(x):
    """Round half away from zero on float64 values (model/deltanet.py:55-58)."""
    x = np.asarray(x, dtype=np.float64)
    return np.where(x >= 0, np.floor(x + 0.5), np.ceil(x - 0.5)).astype(np.int64)


def q16_head(x):
    """model/deltanet.py:60-68: int16 mantissas, one exponent (|m| in [2^14, 2^15) at the max)."""
    x = np.asarray(x, dtype=f32)
    amax = np.abs(x).max()
    if amax == 0:
        return np.zeros(len(x), dtype=np.int64), 0
    e = int(np.frexp(f32(amax))[1]) - 15
    return np.clip(lroundf64(x * f32(np.exp2(-e))), -32767, 32767), e


def q15(x):
    """model/deltanet.py:70-72."""
    return int(np.clip(lroundf64(f32(x) * f32(32768.0)), 0, 32767))


def rne_shift(v, k):
    """model/bitexact.py:35-45: round-to-nearest-even right shift."""
    v = np.asarray(v, dtype=np.int64)
    if k == 0:
        return v.copy()
    q = v >> k
    rnd = (v >> (k - 1)) & 1
    sticky = (v & ((1 << (k - 1)) - 1)) != 0 if k > 1 else np.zeros_like(v, dtype=bool)
    return q + (rnd & (sticky | ((q & 1) == 1)).astype(np.int64))


def arith_shift(v, k):
    """model/bitexact.py:47-50: left if k >= 0, floor right otherwise."""
    v = np.asarray(v, dtype=np.int64)
    return v << k if k >= 0 else v >> (-k)


def dn_ratchet(maxM, maxD, eM, ek, k16max, decay):
    """model/deltanet.py:82-89."""
    kmax = float(k16max) * float(np.exp2(ek))
    t = (maxM * float(decay) + maxD * float(np.exp2(-DN_DELTA_FRAC)) * kmax * float(np.exp2(-eM))) / float(DN_STATE_LIM)
    return 0 if t <= 1.0 else int(np.ceil(np.log2(t)))


def dn_head_step(M, eM, kk, qh, vh, decay, beta, maxM=None):
    """model/deltanet.py:99-147 (head_step): one head, one token.  M int64 (hv, hk) updated in
    place; returns (o float32 (hv,), eM2, maxM2, bad) with bad set where the reference asserts."""
    bad = False
    k16, ek = q16_head(kk)
    q16, eq = q16_head(qh)
    if maxM is None:
        maxM = int(np.abs(M).max())
    shift_a = DN_DELTA_FRAC + eM + ek                                  # :77-79
    d15, nbq = q15(decay), -q15(beta)
    dot = M.astype(np.int64) @ k16.astype(np.int64)                   # pass A
    dot_r = arith_shift(dot, shift_a)
    bad |= bool(np.abs(dot_r).max() >= (1 << 31))
    ddr = (dot_r * d15) >> 15
    nv = -lroundf64(np.asarray(vh, dtype=f32).astype(np.float64) * float(1 << DN_DELTA_FRAC))   # :75-80
    bad |= bool(np.abs(nv).max() >= (1 << 31))
    delta = ((ddr + nv) * nbq) >> 15
    maxD = int(np.abs(delta).max())
    n = dn_ratchet(maxM, maxD, eM, ek, int(np.abs(k16).max()), decay)  # the CPU's algebra
    eM2 = eM + n
    sh = eM2 + 7 - ek                                                  # :91-97
    d15n = int(np.clip(lroundf64(f32(decay) * f32(np.exp2(15 - n))), 0, 32767))
    rnd = (1 << (sh - 1)) if sh > 0 else 0
    d8 = 8 * delta                                                     # pass B
    bad |= bool(np.abs(d8 + rnd).max() >= (1 << 31))
    delta_s = arith_shift(d8 + rnd, -sh)
    bad |= bool(np.abs(delta_s).max() >= (1 << 16))
    newM = rne_shift(M.astype(np.int64) * d15n + np.outer(delta_s, k16.astype(np.int64)), 15)
    bad |= bool(np.abs(newM).max() > 32767)
    M[:] = newM
    maxM2 = int(np.abs(newM).max())
    o_r = (newM @ q16.astype(np.int64)) >> DN_O_SHIFT
    bad |= bool(np.abs(o_r).max() >= (1 << 31))
    of = (o_r.astype(np.float64) * float(np.exp2(eM2 + eq + DN_O_SHIFT))).astype(f32)
    return of, eM2, maxM2, bad
