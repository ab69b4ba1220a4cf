"""Build the C oracle (oracle/trx_oracle.c) into oracle/_build/libtrx_oracle.so.

TEST INFRASTRUCTURE ONLY.  gcc -O2 -fopenmp, no -march flags (the GPU box's host CPU may differ
from the build machine's) and no -ffast-math (the quantiser's fp32 rounding must stay exact).
"""

import ctypes
import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "trx_oracle.c")
OUT_DIR = os.path.join(HERE, "_build")
LIB = os.path.join(OUT_DIR, "libtrx_oracle.so")


def build(force=False):
    os.makedirs(OUT_DIR, exist_ok=True)
    if force or not os.path.exists(LIB) or os.path.getmtime(LIB) < os.path.getmtime(SRC):
        subprocess.run(["gcc", "-O2", "-fopenmp", "-fPIC", "-shared", "-fno-fast-math", "-ffp-contract=off",
                        "-o", LIB, SRC, "-lm"], check=True)
    return LIB


_lib = None


def lib():
    global _lib
    if _lib is None:
        L = ctypes.CDLL(build())
        vp, i = ctypes.c_void_p, ctypes.c_int
        L.trxo_matvec_int.argtypes = [vp, i, i, i, vp, i, i, vp]
        L.trxo_matvec_int.restype = i
        L.trxo_quantize.argtypes = [vp, i, vp]
        L.trxo_quantize.restype = i
        L.trxo_matvec_f.argtypes = [vp, i, i, i, i, i, vp, vp, vp, vp]
        L.trxo_matvec_f.restype = i
        L.trxo_matvec_fp.argtypes = [vp, i, i, i, vp, vp]
        L.trxo_matvec_fp.restype = None
        L.trxo_threads.restype = i
        L.trxo_set_threads.argtypes = [i]
        L.trxo_row_bytes.argtypes = [i, i]
        L.trxo_row_bytes.restype = ctypes.c_long
        _lib = L
    return _lib


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def matvec_int(packed, rows, cols, kind, x8, B, R):
    import numpy as np
    out = np.empty(rows, dtype=np.int32)
    bad = lib().trxo_matvec_int(_p(packed), rows, cols, kind, _p(np.ascontiguousarray(x8, dtype=np.int8)),
                                B, R, _p(out))
    return out, bad


def matvec_f(packed, rows, cols, kind, B, R, x):
    import numpy as np
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty(rows, dtype=np.float32)
    x8 = np.empty(cols, dtype=np.int8)
    scratch = np.empty(rows, dtype=np.int32)
    bad = lib().trxo_matvec_f(_p(packed), rows, cols, kind, B, R, _p(x), _p(y), _p(x8), _p(scratch))
    return y, bad


def quantize(x):
    import numpy as np
    x = np.ascontiguousarray(x, dtype=np.float32)
    x8 = np.empty(x.size, dtype=np.int8)
    e8 = lib().trxo_quantize(_p(x), x.size, _p(x8))
    return x8, e8


def matvec_fp(packed, rows, cols, kind, x):
    import numpy as np
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty(rows, dtype=np.float32)
    lib().trxo_matvec_fp(_p(packed), rows, cols, kind, _p(x), _p(y))
    return y


if __name__ == "__main__":
    print(build(force=True))
