"""The fp-mode projections of the reference's fast engine (model/fastref.py:46-140, HybridRef) on the
B200, over a BONS image.

`HybridRef(img).matmul(entry, X)` is model/fastref.py:119-125: X [T, cols] float32 times the entry's
dequantised matrix W = (code - 1) * scale (the reference's fp16 weight cache holds exactly these
values), in fp32, returning [T, rows]; a K-segmented tensor (FLAG_KSEG, model/fastref.py:95-100)
accumulates its segments over their column ranges.  `proj(role, l, X)` is model/fastref.py:137-140:
the entry of (role, layer), with the image's blockwise Hadamard rotation applied to X first when the
image has one (model/fastref.py:127-135, each block one matmul of its rotation entry).  Every product
is trx_matvec_fp_rows on the device; X may be a numpy array (copied in, the result copied back) or a
CUDA float32 tensor (the result stays on the device).  Ternary entries only: the reference's Q8
tensors are the engine's integer path (trx_matvec_q8_f).
"""

import numpy as np
import torch

from . import bons as Bn
from . import layout as L
from . import ops


class HybridRef:
    def __init__(self, img, ctx=None):
        self.img = img
        self.ctx = ctx or ops.default_context()
        h = img.header
        self.B = h.get("hadamard_block", 0) or 0
        self.widths = list(h.get("hadamard_widths", ()))
        self._dev = {}

    def _tensor(self, e):
        if e["name"] not in self._dev:
            if e["kind"] not in L.TERNARY_KINDS:
                raise TypeError(f"{e['name']}: the fp-mode projection takes ternary entries (kind {e['kind']})")
            self._dev[e["name"]] = self.img.device_tensor(e, device=self.ctx.device)
        return self._dev[e["name"]]

    def _segments(self, e):
        if e["flags"] & Bn.FLAG_KSEG:
            return self.img.matvec_entries(e["role"], e["layer"])
        return [e]

    def matmul(self, e, X):
        """X [T, cols] -> [T, rows] (model/fastref.py:119-125)."""
        host = not isinstance(X, torch.Tensor)
        Xd = torch.as_tensor(np.ascontiguousarray(X, dtype=np.float32) if host else X).to(
            self.ctx.device, torch.float32).contiguous()
        segs = self._segments(e)
        y, c0 = None, 0
        for s in segs:
            t = self._tensor(s)
            xs = Xd[:, c0:c0 + t.cols].contiguous() if len(segs) > 1 else Xd
            y = ops.matvec_fp_rows(self.ctx, t, xs, out=y, resid=y)
            c0 += t.cols
        return y.cpu().numpy() if host else y

    def rotate(self, X, width):
        """model/fastref.py:127-135: the blockwise rotation of X's columns (identity without one)."""
        if not self.B:
            return X
        wi = self.widths.index(width)
        host = not isinstance(X, torch.Tensor)
        Xd = torch.as_tensor(np.ascontiguousarray(X, dtype=np.float32) if host else X).to(self.ctx.device)
        out = torch.empty_like(Xd)
        for b in range(width // self.B):
            e = self.img.find(role=Bn.ROLE_HADAMARD, layer=Bn.hadamard_layer(wi, b))
            out[:, b * self.B:(b + 1) * self.B] = self.matmul(e, Xd[:, b * self.B:(b + 1) * self.B].contiguous())
        return out.cpu().numpy() if host else out

    def proj(self, role, l, X):
        """model/fastref.py:137-140."""
        e = self.img.matvec_entries(role, l)[0]
        cols = sum(s["cols"] for s in self._segments(e))
        return self.matmul(e, self.rotate(X, cols) if self.B else X)


__all__ = ["HybridRef"]
