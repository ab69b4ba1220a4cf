"""Device-side ops on torch CUDA tensors, through the C ABI.

torch provides device memory and the current stream; every computation is a kernel of
libtrixium_b200.so.  Tensors are passed as raw pointers, so inputs must be contiguous CUDA
tensors of the stated dtype on the context's device.
"""

import ctypes

import numpy as np
import torch

from . import _lib
from . import layout as L
from .image import TernaryTensor

_entry_cache = {}


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _need(t, dtype, name):
    if not (t.is_cuda and t.dtype == dtype and t.is_contiguous()):
        raise ValueError(f"{name}: expected a contiguous CUDA {dtype} tensor, got {t.dtype} "
                         f"on {t.device} (contiguous={t.is_contiguous()})")


def _need_x(x, tp):
    """A matvec input: float32, or tagged 64-bit words (int64) when the exchange reads a tagged input."""
    _need(x, torch.int64 if (tp is not None and tp.tag_points and tp.tag_in >= 0) else torch.float32, "x")


class Context:
    """One per device: the library context (device error word, the trit5 LUT)."""

    def __init__(self, device=0):
        self.device = torch.device("cuda", device) if isinstance(device, int) else torch.device(device)
        torch.cuda.set_device(self.device)
        h = ctypes.c_void_p()
        _lib.check(_lib.lib().trx_create(ctypes.byref(h), self.device.index or 0), "trx_create")
        self.h = h

    def errors(self):
        """Synchronise the current stream and return (and clear) the device error bits."""
        bits = ctypes.c_uint32(0)
        _lib.check(_lib.lib().trx_get_error(self.h, _stream(), ctypes.byref(bits)), "trx_get_error")
        return bits.value

    def raise_on_error(self):
        bits = self.errors()
        if bits:
            raise _lib.TrxDeviceError(bits)

    def close(self):
        if self.h:
            _lib.lib().trx_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


_default = {}


def default_context(device=None):
    dev = torch.cuda.current_device() if device is None else device
    if dev not in _default:
        _default[dev] = Context(dev)
    return _default[dev]


class DeviceTensor:
    """A packed tensor (ternary, or KIND_Q8 from image.Q8Tensor) resident on the device, with its
    BONS entry fields."""

    def __init__(self, t: TernaryTensor, device=None):
        dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        self.rows, self.cols, self.kind = t.rows, t.cols, t.kind
        self.bias, self.rshift = t.bias, t.rshift
        self.data = torch.from_numpy(np.ascontiguousarray(t.packed)).to(dev)
        self.entry = _lib.Entry(self.rows, self.cols, self.kind, self.bias, self.rshift)

    @classmethod
    def from_packed(cls, packed, rows, cols, kind, bias, rshift, device=None):
        self = cls.__new__(cls)
        self.rows, self.cols, self.kind, self.bias, self.rshift = rows, cols, kind, bias, rshift
        if isinstance(packed, torch.Tensor):
            self.data = packed
        else:
            dev = torch.device("cuda", torch.cuda.current_device()) if device is None else device
            self.data = torch.from_numpy(np.ascontiguousarray(packed)).to(dev)
        self.entry = _lib.Entry(rows, cols, kind, bias, rshift)
        return self

    @property
    def nbytes(self):
        return self.data.numel()


def matvec_i8(ctx, w: DeviceTensor, x8, out=None):
    _need(x8, torch.int8, "x8")
    if out is None:
        out = torch.empty(w.rows, dtype=torch.int32, device=x8.device)
    _lib.check(_lib.lib().trx_matvec_i8(ctx.h, ctypes.byref(w.entry), _ptr(w.data), _ptr(x8), _ptr(out),
                                        _stream()), "trx_matvec_i8")
    return out


def matvec_q8(ctx, w: DeviceTensor, x8, out=None):
    """Q8 row dot of a KIND_Q8 tensor (model/bitexact.py:127-144): int32 (rows,)."""
    if w.kind != L.KIND_Q8:
        raise ValueError(f"matvec_q8 needs a KIND_Q8 tensor, got kind {w.kind}")
    _need(x8, torch.int8, "x8")
    if out is None:
        out = torch.empty(w.rows, dtype=torch.int32, device=x8.device)
    _lib.check(_lib.lib().trx_matvec_q8(ctx.h, ctypes.byref(w.entry), _ptr(w.data), _ptr(x8), _ptr(out),
                                        _stream()), "trx_matvec_q8")
    return out


def matvec_q8_f(ctx, w: DeviceTensor, x, out=None):
    """Float projection of a KIND_Q8 tensor (model/mirror.py:664-678, Q8 branch): fp32 (rows,)."""
    if w.kind != L.KIND_Q8:
        raise ValueError(f"matvec_q8_f needs a KIND_Q8 tensor, got kind {w.kind}")
    _need(x, torch.float32, "x")
    if out is None:
        out = torch.empty(w.rows, dtype=torch.float32, device=x.device)
    _lib.check(_lib.lib().trx_matvec_q8_f(ctx.h, ctypes.byref(w.entry), _ptr(w.data), _ptr(x), _ptr(out),
                                          _stream()), "trx_matvec_q8_f")
    return out


def matvec_i8_rows(ctx, w: DeviceTensor, x8rows, out=None):
    _need(x8rows, torch.int8, "x8rows")
    nb = x8rows.shape[0]
    if out is None:
        out = torch.empty(nb, w.rows, dtype=torch.int32, device=x8rows.device)
    _lib.check(_lib.lib().trx_matvec_i8_rows(ctx.h, ctypes.byref(w.entry), _ptr(w.data), _ptr(x8rows), nb,
                                             _ptr(out), _stream()), "trx_matvec_i8_rows")
    return out


def matvec_f_rows(ctx, w: DeviceTensor, xrows, out=None, resid=None):
    """Batched float projection (trx_matvec_f_rows): xrows [nb, K] float32 (nb <= 32), each row
    quantised with its own exponent, on the tensor cores; returns [nb, rows] float32 (plus resid)."""
    _need(xrows, torch.float32, "xrows")
    nb = xrows.shape[0]
    if out is None:
        out = torch.empty(nb, w.rows, dtype=torch.float32, device=xrows.device)
    if resid is not None:
        _need(resid, torch.float32, "resid")
    _lib.check(_lib.lib().trx_matvec_f_rows(ctx.h, ctypes.byref(w.entry), _ptr(w.data), _ptr(xrows), nb, _ptr(resid),
                                            _ptr(out), _stream()), "trx_matvec_f_rows")
    return out


def matvec_f_rows_kseg(ctx, segs, xrows, out=None, resid=None):
    """Batched float projection of a K-segmented tensor (trx_matvec_f_rows_kseg): segs, the two
    segments' DeviceTensors in column order; xrows [nb, K] float32 (nb <= 32), each row quantised
    with one exponent over all K; returns [nb, rows] float32 (plus resid)."""
    _need(xrows, torch.float32, "xrows")
    nb, n = xrows.shape[0], len(segs)
    if out is None:
        out = torch.empty(nb, segs[0].rows, dtype=torch.float32, device=xrows.device)
    if resid is not None:
        _need(resid, torch.float32, "resid")
    arr = (_lib.Entry * n)(*[t.entry for t in segs])
    ptrs = (ctypes.c_void_p * n)(*[t.data.data_ptr() for t in segs])
    _lib.check(_lib.lib().trx_matvec_f_rows_kseg(ctx.h, arr, n, ptrs, _ptr(xrows), nb, _ptr(resid), _ptr(out),
                                                 _stream()), "trx_matvec_f_rows_kseg")
    return out


def embed_lookup_rows(ctx, table, tokens, x):
    """x[r] = table[tokens[r]] for every row r (fp16 or fp32 table [vocab, dim])."""
    _need(tokens, torch.int32, "tokens")
    _need(x, torch.float32, "x")
    f16 = table.dtype == torch.float16
    _lib.check(_lib.lib().trx_embed_lookup_rows(ctx.h, _ptr(table), table.shape[0], table.shape[1], 1 if f16 else 0,
                                                _ptr(tokens), tokens.numel(), _ptr(x), _stream()),
               "trx_embed_lookup_rows")
    return x


def rmsnorm_rows(ctx, x, w, eps=1e-6, y=None):
    """Row-wise RMSNorm of x [nrows, n] (trx_rmsnorm_rows)."""
    _need(x, torch.float32, "x")
    if y is None:
        y = torch.empty_like(x)
    _lib.check(_lib.lib().trx_rmsnorm_rows(ctx.h, _ptr(x), _ptr(w), x.shape[-1], x.numel() // x.shape[-1],
                                           ctypes.c_float(eps), _ptr(y), _stream()), "trx_rmsnorm_rows")
    return y


def silu_mul(ctx, g, u, act=None):
    if act is None:
        act = torch.empty_like(g)
    _lib.check(_lib.lib().trx_silu_mul(ctx.h, _ptr(g), _ptr(u), g.numel(), _ptr(act), _stream()), "trx_silu_mul")
    return act


def argmax_rows(ctx, logits, tokens):
    _need(logits, torch.float32, "logits")
    _lib.check(_lib.lib().trx_argmax_rows(ctx.h, _ptr(logits), logits.shape[-1], logits.numel() // logits.shape[-1],
                                          _ptr(tokens), _stream()), "trx_argmax_rows")
    return tokens


def advance_positions(ctx, pos, n=1):
    _need(pos, torch.int32, "pos")
    _lib.check(_lib.lib().trx_advance_positions(ctx.h, _ptr(pos), pos.numel(), n, _stream()), "trx_advance_positions")


def attn_decode_rows(ctx, shape, q, k, v, q_norm, k_norm, rope_freq, kcache, vcache, pos, out=None):
    """Decode attention for a batch of independent sequences (trx_attn_decode_rows): q [nseq, ...],
    caches [nseq, max_pos, n_kv, hd] fp16, pos [nseq] int32."""
    nseq = pos.numel()
    _need(kcache, torch.float16, "kcache")
    if out is None:
        out = torch.empty(nseq, shape.n_head * shape.head_dim, dtype=torch.float32, device=q.device)
    _lib.check(_lib.lib().trx_attn_decode_rows(ctx.h, ctypes.byref(shape), nseq, _ptr(q), _ptr(k), _ptr(v),
                                               _ptr(q_norm), _ptr(k_norm), _ptr(rope_freq), _ptr(kcache),
                                               _ptr(vcache), _ptr(pos), _ptr(out), _stream()), "trx_attn_decode_rows")
    return out


def quantize_pow2(ctx, x, x8=None, e8=None):
    _need(x, torch.float32, "x")
    if x8 is None:
        x8 = torch.empty(x.numel(), dtype=torch.int8, device=x.device)
    if e8 is None:
        e8 = torch.empty(1, dtype=torch.int32, device=x.device)
    _lib.check(_lib.lib().trx_quantize_pow2(ctx.h, _ptr(x), x.numel(), _ptr(x8), _ptr(e8), _stream()),
               "trx_quantize_pow2")
    return x8, e8


def matvec_f(ctx, w: DeviceTensor, x, y=None, norm_w=None, eps=1e-6, resid=None, tp=None):
    _need_x(x, tp)
    if norm_w is not None:
        _need(norm_w, torch.float32, "norm_w")
    if resid is not None:
        _need(resid, torch.float32, "resid")
    if y is None:
        y = torch.empty(w.rows, dtype=torch.float32, device=x.device)
    if tp is not None:  # tensor-parallel exchange (a _lib.TpXfer)
        _lib.check(_lib.lib().trx_matvec_f_tp(ctx.h, ctypes.byref(w.entry), _ptr(w.data), _ptr(x), _ptr(norm_w),
                                              ctypes.c_float(eps), _ptr(resid), _ptr(y), ctypes.byref(tp),
                                              _stream()), "trx_matvec_f_tp")
        return y
    _lib.check(_lib.lib().trx_matvec_f(ctx.h, ctypes.byref(w.entry), _ptr(w.data), _ptr(x), _ptr(norm_w),
                                       ctypes.c_float(eps), _ptr(resid), _ptr(y), _stream()), "trx_matvec_f")
    return y


def matvec_fp(ctx, w: DeviceTensor, x, y=None):
    _need(x, torch.float32, "x")
    if y is None:
        y = torch.empty(w.rows, dtype=torch.float32, device=x.device)
    _lib.check(_lib.lib().trx_matvec_fp(ctx.h, ctypes.byref(w.entry), _ptr(w.data), _ptr(x), _ptr(y),
                                        _stream()), "trx_matvec_fp")
    return y


def matvec_swiglu(ctx, gate: DeviceTensor, up: DeviceTensor, x, act=None, norm_w=None, eps=1e-6, tp=None):
    _need_x(x, tp)
    if act is None:
        act = torch.empty(gate.rows, dtype=torch.float32, device=x.device)
    if tp is not None:
        _lib.check(_lib.lib().trx_matvec_swiglu_tp(ctx.h, ctypes.byref(gate.entry), _ptr(gate.data),
                                                   ctypes.byref(up.entry), _ptr(up.data), _ptr(x), _ptr(norm_w),
                                                   ctypes.c_float(eps), _ptr(act), ctypes.byref(tp), _stream()),
                   "trx_matvec_swiglu_tp")
        return act
    _lib.check(_lib.lib().trx_matvec_swiglu(ctx.h, ctypes.byref(gate.entry), _ptr(gate.data),
                                            ctypes.byref(up.entry), _ptr(up.data), _ptr(x), _ptr(norm_w),
                                            ctypes.c_float(eps), _ptr(act), _stream()), "trx_matvec_swiglu")
    return act


def validate_packed(ctx, w: DeviceTensor):
    _lib.check(_lib.lib().trx_validate_packed(ctx.h, ctypes.byref(w.entry), _ptr(w.data), _stream()),
               "trx_validate_packed")


def matvec_f_batch(ctx, w: DeviceTensor, w_stride, x, x_stride, y, y_stride, njobs):
    """njobs projections in one launch: tensor j at w.data + j*w_stride bytes, input x[j], output y[j]."""
    _lib.check(_lib.lib().trx_matvec_f_batch(ctx.h, ctypes.byref(w.entry), _ptr(w.data), w_stride, _ptr(x),
                                             x_stride, _ptr(y), y_stride, njobs, _stream()),
               "trx_matvec_f_batch")
    return y


def hadamard_rotate(ctx, had: DeviceTensor, x, out=None):
    """The engine's blockwise rotation (model/mirror.py:680-690): block b of the output is the
    quantised float projection of block tensor b against x[b*block:(b+1)*block], all blocks in one
    trx_matvec_f_batch launch.  had: the stacked block tensors (image.hadamard_tensor), width rows of
    block columns; x, out: width floats."""
    block, width = had.cols, had.rows
    _need(x, torch.float32, "x")
    if x.numel() != width:
        raise ValueError(f"x has {x.numel()} elements, the rotation is {width} wide")
    if out is None:
        out = torch.empty(width, dtype=torch.float32, device=x.device)
    one = DeviceTensor.from_packed(had.data, block, block, had.kind, had.bias, had.rshift)
    return matvec_f_batch(ctx, one, block * L.row_bytes(block, had.kind), x, block, out, block, width // block)


def attn_decode(ctx, shape, q, k, v, q_norm, k_norm, rope_freq, kcache, vcache, pos, out=None, tp=None):
    """One decode step of GQA attention (trx_attn_decode).  shape: _lib.AttnShape; q (H*(1+gated)*hd),
    k/v (n_kv*hd) float32; caches [max_pos, n_kv, hd] float16 (or float32: trx_attn_decode_f32cache,
    the reference mirror's cache type); pos: int32 device tensor of one element (the position
    written and attended up to)."""
    for t, n in ((q, "q"), (k, "k"), (v, "v"), (q_norm, "q_norm"), (k_norm, "k_norm")):
        _need(t, torch.float32, n)
    if kcache.dtype == torch.float32:
        _need(vcache, torch.float32, "vcache")
        _need(pos, torch.int32, "pos")
        if tp is not None:
            raise ValueError("the fp32-cache attention has no tensor-parallel exchange")
        if out is None:
            out = torch.empty(shape.n_head * shape.head_dim, dtype=torch.float32, device=q.device)
        _lib.check(_lib.lib().trx_attn_decode_f32cache(ctx.h, ctypes.byref(shape), _ptr(q), _ptr(k), _ptr(v),
                                                       _ptr(q_norm), _ptr(k_norm), _ptr(rope_freq), _ptr(kcache),
                                                       _ptr(vcache), _ptr(pos), _ptr(out), _stream()),
                   "trx_attn_decode_f32cache")
        return out
    _need(kcache, torch.float16, "kcache")
    _need(vcache, torch.float16, "vcache")
    _need(pos, torch.int32, "pos")
    if rope_freq is not None:
        _need(rope_freq, torch.float32, "rope_freq")
    if out is None:
        out = torch.empty(shape.n_head * shape.head_dim, dtype=torch.float32, device=q.device)
    if tp is not None:
        _lib.check(_lib.lib().trx_attn_decode_tp(ctx.h, ctypes.byref(shape), _ptr(q), _ptr(k), _ptr(v),
                                                 _ptr(q_norm), _ptr(k_norm), _ptr(rope_freq), _ptr(kcache),
                                                 _ptr(vcache), _ptr(pos), _ptr(out), ctypes.byref(tp), _stream()),
                   "trx_attn_decode_tp")
        return out
    _lib.check(_lib.lib().trx_attn_decode(ctx.h, ctypes.byref(shape), _ptr(q), _ptr(k), _ptr(v), _ptr(q_norm),
                                          _ptr(k_norm), _ptr(rope_freq), _ptr(kcache), _ptr(vcache), _ptr(pos),
                                          _ptr(out), _stream()), "trx_attn_decode")
    return out


def attn_decode_static(shape, q, k, v, q_norm, k_norm, rope_freq, kcache, vcache, pos, err, out=None):
    """trx_attn_decode without a context (the library's static scratch; nothing allocated by the
    library).  err: a caller-owned int32 device word receiving the device error bits."""
    for t, n in ((q, "q"), (k, "k"), (v, "v"), (q_norm, "q_norm"), (k_norm, "k_norm")):
        _need(t, torch.float32, n)
    _need(kcache, torch.float16, "kcache")
    _need(vcache, torch.float16, "vcache")
    _need(pos, torch.int32, "pos")
    _need(err, torch.int32, "err")
    if out is None:
        out = torch.empty(shape.n_head * shape.head_dim, dtype=torch.float32, device=q.device)
    _lib.check(_lib.lib().trx_attn_decode_static(ctypes.byref(shape), _ptr(q), _ptr(k), _ptr(v), _ptr(q_norm),
                                                 _ptr(k_norm), _ptr(rope_freq), _ptr(kcache), _ptr(vcache),
                                                 _ptr(pos), _ptr(out), _ptr(err), _stream()),
               "trx_attn_decode_static")
    return out


def attn_shape(n_head, n_kv, head_dim, max_pos, rope_dims=None, gated=False, eps=1e-6):
    return _lib.AttnShape(n_head, n_kv, head_dim, head_dim if rope_dims is None else rope_dims, max_pos,
                          1 if gated else 0, eps)


def matvec_f_multi(ctx, entries, packed, x, ys, norm_w=None, eps=1e-6, resids=None, tp=None):
    """Segments sharing one input (trx_matvec_f_multi): entries (list of _lib.Entry), packed (their row
    packets back to back, uint8 CUDA tensor), ys (one float32 output per segment)."""
    n = len(entries)
    _need_x(x, tp)
    arr = (_lib.Entry * n)(*entries)
    yp = (ctypes.c_void_p * n)(*[y.data_ptr() for y in ys])
    rp = None
    if resids is not None:
        rp = (ctypes.c_void_p * n)(*[(r.data_ptr() if r is not None else None) for r in resids])
    if tp is not None:
        _lib.check(_lib.lib().trx_matvec_f_multi_tp(ctx.h, arr, n, _ptr(packed), _ptr(x), _ptr(norm_w),
                                                    ctypes.c_float(eps), yp, rp, ctypes.byref(tp), _stream()),
                   "trx_matvec_f_multi_tp")
        return ys
    _lib.check(_lib.lib().trx_matvec_f_multi(ctx.h, arr, n, _ptr(packed), _ptr(x), _ptr(norm_w), ctypes.c_float(eps),
                                             yp, rp, _stream()), "trx_matvec_f_multi")
    return ys


def matvec_f_rows_multi(ctx, entries, packed, xrows, ys, norm_w=None, eps=1e-6, resids=None):
    """The batched form of matvec_f_multi (trx_matvec_f_rows_multi): up to 4 tensors packed back to
    back on the same activation rows xrows [nb, cols] (optionally RMS-normalised per row first); ys:
    one [nb, rows_i] float32 output per tensor, resids the same or None."""
    n = len(entries)
    _need(xrows, torch.float32, "xrows")
    arr = (_lib.Entry * n)(*entries)
    yp = (ctypes.c_void_p * n)(*[y.data_ptr() for y in ys])
    rp = None
    if resids is not None:
        rp = (ctypes.c_void_p * n)(*[(r.data_ptr() if r is not None else None) for r in resids])
    _lib.check(_lib.lib().trx_matvec_f_rows_multi(ctx.h, arr, n, _ptr(packed), _ptr(xrows), xrows.shape[0],
                                                  _ptr(norm_w), ctypes.c_float(eps), yp, rp, _stream()),
               "trx_matvec_f_rows_multi")
    return ys


def embed_lookup(ctx, table, token, x):
    """x = table[token] (float16 or float32 table [vocab, dim]; token: int32 device tensor)."""
    _need(token, torch.int32, "token")
    _need(x, torch.float32, "x")
    f16 = table.dtype == torch.float16
    _need(table, torch.float16 if f16 else torch.float32, "table")
    _lib.check(_lib.lib().trx_embed_lookup(ctx.h, _ptr(table), table.shape[0], table.shape[1], 1 if f16 else 0,
                                           _ptr(token), _ptr(x), _stream()), "trx_embed_lookup")
    return x


def embed_lookup_bfp16(ctx, mant, exps, token, x):
    """x = mant[token] * 2^exps[token] (an image's int16 embedding table: mant int16 [vocab, dim],
    exps int32 [vocab]; token: int32 device tensor of one element)."""
    _need(mant, torch.int16, "mant")
    _need(exps, torch.int32, "exps")
    _need(token, torch.int32, "token")
    _need(x, torch.float32, "x")
    _lib.check(_lib.lib().trx_embed_lookup_bfp16(ctx.h, _ptr(mant), _ptr(exps), mant.shape[0], mant.shape[1],
                                                 _ptr(token), _ptr(x), _stream()), "trx_embed_lookup_bfp16")
    return x


def rmsnorm(ctx, x, w, eps=1e-6, y=None):
    """y = RMSNorm(x) * w with the canonical 64-partial sum of squares (trx_rmsnorm)."""
    _need(x, torch.float32, "x")
    _need(w, torch.float32, "w")
    if y is None:
        y = torch.empty_like(x)
    _lib.check(_lib.lib().trx_rmsnorm(ctx.h, _ptr(x), _ptr(w), x.numel(), ctypes.c_float(eps), _ptr(y), _stream()),
               "trx_rmsnorm")
    return y


def matvec_f_kseg(ctx, segs, x, y=None, resid=None, tp=None):
    """Float projection of a K-segmented tensor (trx_matvec_f_kseg): segs, the segments' DeviceTensors
    in column order (ternary or KIND_Q8, the tensor's B/R in each); x: the full input.  tp: a
    _lib.TpXfer of tagged words (trx_matvec_f_kseg_tp)."""
    _need_x(x, tp)
    n = len(segs)
    arr = (_lib.Entry * n)(*[t.entry for t in segs])
    ptrs = (ctypes.c_void_p * n)(*[t.data.data_ptr() for t in segs])
    if y is None:
        y = torch.empty(segs[0].rows, dtype=torch.float32, device=x.device)
    if tp is not None:
        _lib.check(_lib.lib().trx_matvec_f_kseg_tp(ctx.h, arr, n, ptrs, _ptr(x), _ptr(resid), _ptr(y),
                                                   ctypes.byref(tp), _stream()), "trx_matvec_f_kseg_tp")
        return y
    _lib.check(_lib.lib().trx_matvec_f_kseg(ctx.h, arr, n, ptrs, _ptr(x), _ptr(resid), _ptr(y), _stream()),
               "trx_matvec_f_kseg")
    return y


def advance_position(ctx, pos, n=1):
    _need(pos, torch.int32, "pos")
    _lib.check(_lib.lib().trx_advance_position(ctx.h, _ptr(pos), n, _stream()), "trx_advance_position")


def lmhead_argmax(ctx, w: DeviceTensor, x, token=None, logits=None, norm_w=None, eps=1e-6):
    """Greedy token of the LM head (trx_lmhead_argmax): token (int32 device tensor of one
    element) = argmax over rows of the float projection of (optionally RMS-normalised) x."""
    _need(x, torch.float32, "x")
    if token is None:
        token = torch.empty(1, dtype=torch.int32, device=x.device)
    _need(token, torch.int32, "token")
    if logits is not None:
        _need(logits, torch.float32, "logits")
    if norm_w is not None:
        _need(norm_w, torch.float32, "norm_w")
    _lib.check(_lib.lib().trx_lmhead_argmax(ctx.h, ctypes.byref(w.entry), _ptr(w.data), _ptr(x), _ptr(norm_w),
                                            ctypes.c_float(eps), _ptr(logits), _ptr(token), _stream()),
               "trx_lmhead_argmax")
    return token


def lmhead_argmax_key(ctx, w: DeviceTensor, x, key, row_offset=0, logits=None, norm_w=None, eps=1e-6, tp=None):
    """One shard of a row-sharded LM head: key (int64 device tensor of one element) = the shard's
    argmax key with global row = local row + row_offset (trx_lmhead_argmax_key)."""
    _need_x(x, tp)
    _need(key, torch.int64, "key")
    if tp is not None:
        _lib.check(_lib.lib().trx_lmhead_argmax_key_tp(ctx.h, ctypes.byref(w.entry), _ptr(w.data), _ptr(x),
                                                       _ptr(norm_w), ctypes.c_float(eps), int(row_offset),
                                                       _ptr(logits), _ptr(key), ctypes.byref(tp), _stream()),
                   "trx_lmhead_argmax_key_tp")
        return key
    _lib.check(_lib.lib().trx_lmhead_argmax_key(ctx.h, ctypes.byref(w.entry), _ptr(w.data), _ptr(x), _ptr(norm_w),
                                                ctypes.c_float(eps), int(row_offset), _ptr(logits), _ptr(key),
                                                _stream()), "trx_lmhead_argmax_key")
    return key


def argmax_token(ctx, keys, token, tp=None):
    """token = the row of the largest key in `keys` (int64 device tensor of gathered shard keys)."""
    _need(keys, torch.int64, "keys")
    _need(token, torch.int32, "token")
    if tp is not None:
        _lib.check(_lib.lib().trx_argmax_token_tp(ctx.h, _ptr(keys), keys.numel(), _ptr(token), ctypes.byref(tp),
                                                  _stream()), "trx_argmax_token_tp")
        return token
    _lib.check(_lib.lib().trx_argmax_token(ctx.h, _ptr(keys), keys.numel(), _ptr(token), _stream()),
               "trx_argmax_token")
    return token


def deltanet_shape(n_k_heads, k_head_dim, n_v_heads, v_head_dim, conv_kernel=4, eps=1e-6):
    return _lib.DeltaNetShape(n_k_heads, k_head_dim, n_v_heads, v_head_dim, conv_kernel, eps)


def deltanet_step(ctx, shape, qkv, z, beta, alpha, dt_bias, ssm_a, conv_w, norm_w, conv_ring, state, pos, out=None,
                  tp=None):
    """One gated-DeltaNet decode step (trx_deltanet_step); conv_ring [K, C] and state [nv, hv, hk]
    float32 are updated in place; pos: int32 device tensor of one element.  tp: a _lib.TpXfer whose
    tagged output receives the grouped output too (trx_deltanet_step_tp)."""
    for t, n in ((qkv, "qkv"), (z, "z"), (beta, "beta"), (alpha, "alpha"), (dt_bias, "dt_bias"), (ssm_a, "ssm_a"),
                 (conv_w, "conv_w"), (norm_w, "norm_w"), (conv_ring, "conv_ring"), (state, "state")):
        _need(t, torch.float32, n)
    _need(pos, torch.int32, "pos")
    if out is None:
        out = torch.empty(shape.n_v_heads * shape.v_head_dim, dtype=torch.float32, device=qkv.device)
    if tp is not None:
        _lib.check(_lib.lib().trx_deltanet_step_tp(ctx.h, ctypes.byref(shape), _ptr(qkv), _ptr(z), _ptr(beta),
                                                   _ptr(alpha), _ptr(dt_bias), _ptr(ssm_a), _ptr(conv_w),
                                                   _ptr(norm_w), _ptr(conv_ring), _ptr(state), _ptr(pos), _ptr(out),
                                                   ctypes.byref(tp), _stream()), "trx_deltanet_step_tp")
        return out
    _lib.check(_lib.lib().trx_deltanet_step(ctx.h, ctypes.byref(shape), _ptr(qkv), _ptr(z), _ptr(beta), _ptr(alpha),
                                            _ptr(dt_bias), _ptr(ssm_a), _ptr(conv_w), _ptr(norm_w), _ptr(conv_ring),
                                            _ptr(state), _ptr(pos), _ptr(out), _stream()), "trx_deltanet_step")
    return out


def deltanet_step_rows(ctx, shape, qkv, z, beta, alpha, dt_bias, ssm_a, conv_w, norm_w, conv_ring, state, pos,
                       out=None):
    """The gated-DeltaNet step of a batch of sequences (trx_deltanet_step_rows): every per-sequence
    tensor has a leading sequence dimension; pos [nseq] int32."""
    nseq = pos.numel()
    if out is None:
        out = torch.empty(nseq, shape.n_v_heads * shape.v_head_dim, dtype=torch.float32, device=qkv.device)
    _lib.check(_lib.lib().trx_deltanet_step_rows(ctx.h, ctypes.byref(shape), nseq, _ptr(qkv), _ptr(z), _ptr(beta),
                                                 _ptr(alpha), _ptr(dt_bias), _ptr(ssm_a), _ptr(conv_w), _ptr(norm_w),
                                                 _ptr(conv_ring), _ptr(state), _ptr(pos), _ptr(out), _stream()),
               "trx_deltanet_step_rows")
    return out


def matvec_fp_rows(ctx, w: DeviceTensor, X, out=None, resid=None):
    """fp-mode projection of the rows of X [T, cols] float32 (trx_matvec_fp_rows,
    model/fastref.py:119-125): returns [T, rows] float32 (plus resid)."""
    _need(X, torch.float32, "X")
    T = X.shape[0]
    if out is None:
        out = torch.empty(T, w.rows, dtype=torch.float32, device=X.device)
    if resid is not None:
        _need(resid, torch.float32, "resid")
    _lib.check(_lib.lib().trx_matvec_fp_rows(ctx.h, ctypes.byref(w.entry), _ptr(w.data), _ptr(X), T, _ptr(resid),
                                             _ptr(out), _stream()), "trx_matvec_fp_rows")
    return out


def deltanet_int_step(ctx, state, exp, maxabs, k, q, v, decay, beta, out=None):
    """The integer DeltaNet head step of nheads heads (trx_deltanet_int_step, model/deltanet.py:99-147):
    state int16 [nheads, hv, hk], exp and maxabs int32 [nheads] (maxabs < 0: computed), k, q float32
    [nheads, hk], v [nheads, hv], decay, beta [nheads].  Updates state, exp and maxabs in place and
    returns o [nheads, hv] float32."""
    nh, hv, hk = state.shape
    _need(state, torch.int16, "state")
    _need(exp, torch.int32, "exp")
    _need(maxabs, torch.int32, "maxabs")
    for t, n in ((k, "k"), (q, "q"), (v, "v"), (decay, "decay"), (beta, "beta")):
        _need(t, torch.float32, n)
    if out is None:
        out = torch.empty(nh, hv, dtype=torch.float32, device=state.device)
    _lib.check(_lib.lib().trx_deltanet_int_step(ctx.h, nh, hv, hk, _ptr(state), _ptr(exp), _ptr(maxabs), _ptr(k),
                                                _ptr(q), _ptr(v), _ptr(decay), _ptr(beta), _ptr(out), _stream()),
               "trx_deltanet_int_step")
    return out


def row_bytes(cols, kind):
    return int(_lib.lib().trx_row_bytes(cols, kind))


__all__ = ["Context", "default_context", "DeviceTensor", "matvec_i8", "matvec_q8", "matvec_q8_f", "matvec_i8_rows", "quantize_pow2",
           "matvec_f", "matvec_fp", "matvec_swiglu", "hadamard_rotate", "validate_packed", "matvec_f_batch", "attn_decode", "attn_decode_static", "attn_shape",
           "deltanet_shape", "deltanet_step", "lmhead_argmax", "lmhead_argmax_key", "argmax_token", "matvec_f_multi", "embed_lookup",
           "advance_position", "row_bytes", "L"]
