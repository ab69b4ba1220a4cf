"""trixium_b200: the TriXium ternary decode path on NVIDIA B200 (sm_100a).

* `layout`, `image`: the converter's row-packet layout and the per-tensor fixed point (host).
* `ops`: device ops on torch CUDA tensors through libtrixium_b200.so (C ABI:
  include/trixium_b200.h).
* `bitexact`: the reference engine's call surface (model/bitexact.py) on the GPU.

The CUDA library is required: importing `ops` raises if libtrixium_b200.so is missing.
"""

from . import layout, image  # noqa: F401

__all__ = ["layout", "image"]
