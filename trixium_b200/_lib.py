"""ctypes binding of libtrixium_b200.so (the C ABI declared in include/trixium_b200.h).

The library is loaded from this package directory only; there is no fallback: if it is missing
or fails to load, importing the ops raises.
"""

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libtrixium_b200.so")

TRX_OK = 0
ERRORS = {
    -1: "TRX_ERR_ARG", -2: "TRX_ERR_LAYOUT", -3: "TRX_ERR_OVERFLOW", -4: "TRX_ERR_CUDA",
    -5: "TRX_ERR_TIMEOUT", -6: "TRX_ERR_UNSUPPORTED",
}
DEV_OVERFLOW, DEV_BADBYTE, DEV_TIMEOUT, DEV_INTERNAL, DEV_RANGE = 0x1, 0x2, 0x4, 0x8, 0x10

# Every symbol the header declares (tests check the library exports all of them).
SYMBOLS = (
    "trx_create", "trx_destroy", "trx_get_error", "trx_last_cuda_error", "trx_row_bytes", "trx_matvec_i8", "trx_matvec_q8", "trx_matvec_q8_f",
    "trx_matvec_i8_rows", "trx_quantize_pow2", "trx_matvec_f", "trx_matvec_fp",
    "trx_matvec_swiglu", "trx_validate_packed", "trx_matvec_f_batch", "trx_attn_decode",
    "trx_deltanet_step", "trx_lmhead_argmax", "trx_matvec_f_multi", "trx_embed_lookup", "trx_advance_position",
    "trx_attn_decode_static", "trx_lmhead_argmax_key", "trx_argmax_token", "trx_matvec_f_tp",
    "trx_matvec_f_multi_tp", "trx_matvec_swiglu_tp", "trx_lmhead_argmax_key_tp", "trx_argmax_token_tp",
    "trx_attn_decode_tp", "trx_embed_lookup_bfp16", "trx_rmsnorm", "trx_matvec_f_kseg",
    "trx_attn_decode_f32cache", "trx_matvec_f_rows", "trx_embed_lookup_rows", "trx_rmsnorm_rows", "trx_silu_mul",
    "trx_argmax_rows", "trx_advance_positions", "trx_attn_decode_rows", "trx_deltanet_step_rows",
    "trx_deltanet_int_step", "trx_matvec_fp_rows", "trx_matvec_f_rows_multi", "trx_deltanet_step_tp",
    "trx_matvec_f_kseg_tp", "trx_matvec_f_rows_kseg",
)

TP_MAX = 8
# Device error-word bits (trx_get_error).
TRX_DEV_OVERFLOW, TRX_DEV_BADBYTE, TRX_DEV_TIMEOUT, TRX_DEV_INTERNAL, TRX_DEV_RANGE = 0x1, 0x2, 0x4, 0x8, 0x10


class TrxError(RuntimeError):
    def __init__(self, status, where=""):
        self.status = status
        super().__init__(f"{where}: {ERRORS.get(status, status)}")


class TrxDeviceError(RuntimeError):
    def __init__(self, bits):
        self.bits = bits
        names = [n for b, n in ((DEV_OVERFLOW, "overflow"), (DEV_BADBYTE, "invalid trit5 byte"),
                                (DEV_TIMEOUT, "bounded wait timed out"),
                                (DEV_INTERNAL, "shared-memory layout mismatch"),
                                (DEV_RANGE, "device-side index out of range")) if bits & b]
        super().__init__("device error: " + ", ".join(names or [hex(bits)]))


class AttnShape(ctypes.Structure):
    """trx_attn_shape: one attention layer's geometry."""
    _fields_ = [("n_head", ctypes.c_uint32), ("n_kv", ctypes.c_uint32), ("head_dim", ctypes.c_uint32),
                ("rope_dims", ctypes.c_uint32), ("max_pos", ctypes.c_uint32), ("gated", ctypes.c_int32),
                ("eps", ctypes.c_float)]


class DeltaNetShape(ctypes.Structure):
    """trx_deltanet_shape: one gated-DeltaNet layer's geometry."""
    _fields_ = [("n_k_heads", ctypes.c_uint32), ("k_head_dim", ctypes.c_uint32), ("n_v_heads", ctypes.c_uint32),
                ("v_head_dim", ctypes.c_uint32), ("conv_kernel", ctypes.c_uint32), ("eps", ctypes.c_float)]


class TpXfer(ctypes.Structure):
    """trx_tp_xfer: a launch's tensor-parallel exchange over peer memory."""
    _fields_ = [("world", ctypes.c_uint32), ("rank", ctypes.c_uint32), ("dst", ctypes.c_void_p * TP_MAX),
                ("offset", ctypes.c_uint32), ("signal", ctypes.c_void_p * TP_MAX), ("wait", ctypes.c_void_p),
                ("step", ctypes.c_void_p), ("arrive", ctypes.c_void_p), ("tag_points", ctypes.c_uint32),
                ("tag_out", ctypes.c_int32), ("tag_in", ctypes.c_int32)]

    def __init__(self, *a, **k):
        super().__init__(*a, **k)
        if "tag_out" not in k:
            self.tag_out = -1
        if "tag_in" not in k:
            self.tag_in = -1


class Entry(ctypes.Structure):
    """trx_entry: the BONS entry fields a matvec needs."""
    _fields_ = [("rows", ctypes.c_uint32), ("cols", ctypes.c_uint32), ("kind", ctypes.c_int32),
                ("bias", ctypes.c_int32), ("rshift", ctypes.c_int32)]


_vp = ctypes.c_void_p
_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is not built (python -m trixium_b200.build)")
        L = ctypes.CDLL(LIB_PATH)
        E = ctypes.POINTER(Entry)
        T = ctypes.POINTER(TpXfer)
        sig = {
            "trx_create": ([ctypes.POINTER(_vp), ctypes.c_int], ctypes.c_int),
            "trx_destroy": ([_vp], ctypes.c_int),
            "trx_get_error": ([_vp, _vp, ctypes.POINTER(ctypes.c_uint32)], ctypes.c_int),
            "trx_row_bytes": ([ctypes.c_uint32, ctypes.c_int32], ctypes.c_uint64),
            "trx_last_cuda_error": ([], ctypes.c_char_p),
            "trx_matvec_i8": ([_vp, E, _vp, _vp, _vp, _vp], ctypes.c_int),
            "trx_matvec_q8": ([_vp, E, _vp, _vp, _vp, _vp], ctypes.c_int),
            "trx_matvec_q8_f": ([_vp, E, _vp, _vp, _vp, _vp], ctypes.c_int),
            "trx_matvec_i8_rows": ([_vp, E, _vp, _vp, ctypes.c_int, _vp, _vp], ctypes.c_int),
            "trx_quantize_pow2": ([_vp, _vp, ctypes.c_uint32, _vp, _vp, _vp], ctypes.c_int),
            "trx_matvec_f": ([_vp, E, _vp, _vp, _vp, ctypes.c_float, _vp, _vp, _vp], ctypes.c_int),
            "trx_matvec_fp": ([_vp, E, _vp, _vp, _vp, _vp], ctypes.c_int),
            "trx_matvec_swiglu": ([_vp, E, _vp, E, _vp, _vp, _vp, ctypes.c_float, _vp, _vp], ctypes.c_int),
            "trx_validate_packed": ([_vp, E, _vp, _vp], ctypes.c_int),
            "trx_matvec_f_batch": ([_vp, E, _vp, ctypes.c_uint64, _vp, ctypes.c_uint64, _vp,
                                    ctypes.c_uint64, ctypes.c_int, _vp], ctypes.c_int),
            "trx_attn_decode": ([_vp, ctypes.POINTER(AttnShape)] + [_vp] * 11, ctypes.c_int),
            "trx_deltanet_step": ([_vp, ctypes.POINTER(DeltaNetShape)] + [_vp] * 13, ctypes.c_int),
            "trx_lmhead_argmax": ([_vp, E, _vp, _vp, _vp, ctypes.c_float, _vp, _vp, _vp], ctypes.c_int),
            "trx_matvec_f_multi": ([_vp, E, ctypes.c_int, _vp, _vp, _vp, ctypes.c_float, _vp, _vp, _vp],
                                   ctypes.c_int),
            "trx_embed_lookup": ([_vp, _vp, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_int32, _vp, _vp, _vp],
                                 ctypes.c_int),
            "trx_advance_position": ([_vp, _vp, ctypes.c_int32, _vp], ctypes.c_int),
            "trx_attn_decode_static": ([ctypes.POINTER(AttnShape)] + [_vp] * 12, ctypes.c_int),
            "trx_lmhead_argmax_key": ([_vp, E, _vp, _vp, _vp, ctypes.c_float, ctypes.c_uint32, _vp, _vp, _vp],
                                      ctypes.c_int),
            "trx_argmax_token": ([_vp, _vp, ctypes.c_int32, _vp, _vp], ctypes.c_int),
            "trx_matvec_f_tp": ([_vp, E, _vp, _vp, _vp, ctypes.c_float, _vp, _vp, T, _vp], ctypes.c_int),
            "trx_matvec_f_multi_tp": ([_vp, E, ctypes.c_int, _vp, _vp, _vp, ctypes.c_float, _vp, _vp, T, _vp],
                                      ctypes.c_int),
            "trx_matvec_swiglu_tp": ([_vp, E, _vp, E, _vp, _vp, _vp, ctypes.c_float, _vp, T, _vp], ctypes.c_int),
            "trx_lmhead_argmax_key_tp": ([_vp, E, _vp, _vp, _vp, ctypes.c_float, ctypes.c_uint32, _vp, _vp, T, _vp],
                                         ctypes.c_int),
            "trx_argmax_token_tp": ([_vp, _vp, ctypes.c_int32, _vp, T, _vp], ctypes.c_int),
            "trx_attn_decode_tp": ([_vp, ctypes.POINTER(AttnShape)] + [_vp] * 10 + [T, _vp], ctypes.c_int),
            "trx_embed_lookup_bfp16": ([_vp, _vp, _vp, ctypes.c_uint32, ctypes.c_uint32, _vp, _vp, _vp],
                                       ctypes.c_int),
            "trx_rmsnorm": ([_vp, _vp, _vp, ctypes.c_uint32, ctypes.c_float, _vp, _vp], ctypes.c_int),
            "trx_matvec_f_kseg": ([_vp, E, ctypes.c_int, _vp, _vp, _vp, _vp, _vp], ctypes.c_int),
            "trx_matvec_f_kseg_tp": ([_vp, E, ctypes.c_int, _vp, _vp, _vp, _vp, T, _vp], ctypes.c_int),
            "trx_matvec_f_rows_kseg": ([_vp, E, ctypes.c_int, _vp, _vp, ctypes.c_int, _vp, _vp, _vp], ctypes.c_int),
            "trx_deltanet_step_tp": ([_vp, ctypes.POINTER(DeltaNetShape)] + [_vp] * 12 + [T, _vp], ctypes.c_int),
            "trx_attn_decode_f32cache": ([_vp, ctypes.POINTER(AttnShape)] + [_vp] * 11, ctypes.c_int),
            "trx_matvec_f_rows": ([_vp, E, _vp, _vp, ctypes.c_int, _vp, _vp, _vp], ctypes.c_int),
            "trx_embed_lookup_rows": ([_vp, _vp, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_int32, _vp, ctypes.c_int32,
                                       _vp, _vp], ctypes.c_int),
            "trx_rmsnorm_rows": ([_vp, _vp, _vp, ctypes.c_uint32, ctypes.c_int32, ctypes.c_float, _vp, _vp],
                                 ctypes.c_int),
            "trx_silu_mul": ([_vp, _vp, _vp, ctypes.c_uint64, _vp, _vp], ctypes.c_int),
            "trx_argmax_rows": ([_vp, _vp, ctypes.c_uint32, ctypes.c_int32, _vp, _vp], ctypes.c_int),
            "trx_advance_positions": ([_vp, _vp, ctypes.c_int32, ctypes.c_int32, _vp], ctypes.c_int),
            "trx_attn_decode_rows": ([_vp, ctypes.POINTER(AttnShape), ctypes.c_int32] + [_vp] * 11, ctypes.c_int),
            "trx_deltanet_step_rows": ([_vp, ctypes.POINTER(DeltaNetShape), ctypes.c_int32] + [_vp] * 13,
                                       ctypes.c_int),
            "trx_deltanet_int_step": ([_vp, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32] + [_vp] * 10,
                                      ctypes.c_int),
            "trx_matvec_fp_rows": ([_vp, E, _vp, _vp, ctypes.c_int32, _vp, _vp, _vp], ctypes.c_int),
            "trx_matvec_f_rows_multi": ([_vp, E, ctypes.c_int, _vp, _vp, ctypes.c_int, _vp, ctypes.c_float, _vp, _vp,
                                         _vp], ctypes.c_int),
        }
        for name, (args, res) in sig.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = res
        _lib = L
    return _lib


def check(status, where=""):
    if status != TRX_OK:
        if status == -4 and _lib is not None:
            where = f"{where} ({_lib.trx_last_cuda_error().decode(errors='replace')})"
        raise TrxError(status, where)
