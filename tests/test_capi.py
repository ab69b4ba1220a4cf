"""The C-ABI library loads and exports every entry point include/trixium_b200.h declares.

No compute runs here (no GPU in the build container): only symbol lookup and the host-only
geometry helper.
"""
import os
import re

import pytest

from oracle import ref

from trixium_b200 import _lib, layout as L

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    src = open(os.path.join(ROOT, "include", "trixium_b200.h")).read()
    return sorted(set(re.findall(r"^\s*(?:trx_status|uint64_t|const char \*)\s*(trx_\w+)\s*\(", src, re.M)))


def test_header_and_binding_agree():
    assert declared_symbols() == sorted(_lib.SYMBOLS)


def test_library_exports_every_symbol():
    lib = _lib.lib()
    for name in declared_symbols():
        assert hasattr(lib, name), name


@pytest.mark.parametrize("cols", [128, 256, 640, 2048, 2944, 4096, 5120, 6144, 12288, 17408])
@pytest.mark.parametrize("kind", [L.KIND_TERNARY, L.KIND_TERNARY5])
def test_row_bytes(cols, kind):
    assert _lib.lib().trx_row_bytes(cols, kind) == L.row_bytes(cols, kind)


@pytest.mark.parametrize("cols", [32, 96, 512, 544, 4160, 32768])
def test_row_bytes_q8(cols):
    assert _lib.lib().trx_row_bytes(cols, L.KIND_Q8) == L.q8_row_bytes(cols) == ref.q8_row_bytes(cols)


def test_row_bytes_rejects_bad_layouts():
    assert _lib.lib().trx_row_bytes(48, L.KIND_Q8) == 0
    assert _lib.lib().trx_row_bytes(100, 5) == 0
    assert _lib.lib().trx_row_bytes(128, 3) == 0


def test_bindings_match_header_arity():
    """Every ctypes binding takes as many arguments as its prototype in the header declares."""
    import re
    from trixium_b200 import _lib
    h = open(os.path.join(ROOT, "include", "trixium_b200.h")).read()
    L = _lib.lib()
    protos = re.findall(r"trx_status\s+(trx_\w+)\s*\(([^;]*)\);", h)
    assert protos
    for name, args in protos:
        fn = getattr(L, name)
        assert fn.argtypes is not None, name
        assert len(fn.argtypes) == len([a for a in args.split(",") if a.strip()]), name


def test_static_attention_rejects_shapes_beyond_its_arrays():
    """trx_attn_decode_static checks its fixed limits on the host before any CUDA call: more than
    64 kv heads, or partials beyond 2^20 floats, return TRX_ERR_UNSUPPORTED (the pointers here are
    never dereferenced)."""
    import ctypes
    lib = _lib.lib()
    fake = ctypes.c_void_p(0x1000)  # 16-byte aligned, never touched
    args = [fake] * 11 + [ctypes.c_void_p(0)]
    too_many_kv = _lib.AttnShape(128, 128, 64, 64, 512, 0, 1e-6)
    assert lib.trx_attn_decode_static(ctypes.byref(too_many_kv), *args) == -6
    # 64 kv heads x 16 splits x 8 heads per kv head x (128 + 2) floats > 2^20.
    too_many_partials = _lib.AttnShape(512, 64, 128, 128, 4096, 0, 1e-6)
    assert lib.trx_attn_decode_static(ctypes.byref(too_many_partials), *args) == -6
