"""Time one kernel of the library on synthetic data (a CUDA device is required).

    python -m trixium_b200.microbench rows --rows 12288 --cols 4096 --kind 0 --batch 16
    python -m trixium_b200.microbench dn_int --heads 48 --hv 128 --hk 128

`rows`: the batched projection (trx_matvec_f_rows, tcgen05 kind::i8) of `batch` activation rows
against one `rows` x `cols` tensor of the benchmark distribution, `copies` distinct tensors used in
turn.  `dn_int`: the integer DeltaNet head step (trx_deltanet_int_step) over `heads` heads.  Prints
one JSON line with the mean time per launch (CUDA events) and the weight (or state) bytes per second.
"""

import argparse
import json

import numpy as np
import torch

from . import image, layout as L, ops


def rows(a):
    ctx = ops.Context(0)
    gen = torch.Generator(device="cuda").manual_seed(77)
    t0, _ = image.synthetic_matvec_case(256, a.cols, seed=0, kind=a.kind)
    rb = L.row_bytes(a.cols, a.kind)
    ws = []
    for _ in range(a.copies):
        c, s = image.synthetic_codes_scales_torch(gen, a.rows, a.cols, "cuda")
        ws.append(ops.DeviceTensor.from_packed(image.pack_rows_torch(s, c, a.kind), a.rows, a.cols, a.kind, t0.bias,
                                               t0.rshift))
    X = torch.randn(a.batch, a.cols, generator=gen, device="cuda")
    Y = torch.empty(a.batch, a.rows, device="cuda")
    for i in range(a.warmup):
        ops.matvec_f_rows(ctx, ws[i % a.copies], X, Y)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(a.launches):
        ops.matvec_f_rows(ctx, ws[i % a.copies], X, Y)
    e1.record()
    torch.cuda.synchronize()
    ctx.raise_on_error()
    ms = e0.elapsed_time(e1) / a.launches
    alg = L.algorithmic_bytes(a.rows, a.cols, a.kind)
    return {"kernel": "rows_kernel", "rows": a.rows, "cols": a.cols, "kind": a.kind, "batch": a.batch,
            "us_per_launch": round(ms * 1e3, 2), "weight_GBps": round(alg / (ms * 1e-3) / 1e9, 1),
            "weight_bytes": alg, "note": "includes the rows' quantisation launch"}


def dn_int(a):
    ctx = ops.Context(0)
    g = torch.Generator(device="cuda").manual_seed(5)
    nh, hv, hk = a.heads, a.hv, a.hk
    st = torch.zeros(nh, hv, hk, dtype=torch.int16, device="cuda")
    ex = torch.full((nh,), -20, dtype=torch.int32, device="cuda")
    mx = torch.zeros(nh, dtype=torch.int32, device="cuda")
    k = torch.nn.functional.normalize(torch.randn(nh, hk, generator=g, device="cuda"), dim=1)
    q = torch.nn.functional.normalize(torch.randn(nh, hk, generator=g, device="cuda"), dim=1)
    v = torch.randn(nh, hv, generator=g, device="cuda") * 0.5
    decay = torch.rand(nh, generator=g, device="cuda") * 0.5 + 0.5
    beta = torch.rand(nh, generator=g, device="cuda") * 0.5 + 0.3
    for _ in range(a.warmup):
        ops.deltanet_int_step(ctx, st, ex, mx, k, q, v, decay, beta)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(a.launches):
        ops.deltanet_int_step(ctx, st, ex, mx, k, q, v, decay, beta)
    e1.record()
    torch.cuda.synchronize()
    ctx.raise_on_error()
    ms = e0.elapsed_time(e1) / a.launches
    state = nh * hv * hk * 2 * 2  # int16 state read and written
    return {"kernel": "dn_int_kernel", "heads": nh, "hv": hv, "hk": hk, "us_per_launch": round(ms * 1e3, 2),
            "state_GBps": round(state / (ms * 1e-3) / 1e9, 1), "state_bytes": state}


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    sub = ap.add_subparsers(dest="what", required=True)
    r = sub.add_parser("rows")
    r.add_argument("--rows", type=int, default=12288)
    r.add_argument("--cols", type=int, default=4096)
    r.add_argument("--kind", type=int, default=L.KIND_TERNARY, choices=[L.KIND_TERNARY, L.KIND_TERNARY5])
    r.add_argument("--batch", type=int, default=16)
    r.add_argument("--copies", type=int, default=2)
    d = sub.add_parser("dn_int")
    d.add_argument("--heads", type=int, default=48)
    d.add_argument("--hv", type=int, default=128)
    d.add_argument("--hk", type=int, default=128)
    for p in (r, d):
        p.add_argument("--launches", type=int, default=20)
        p.add_argument("--warmup", type=int, default=3)
    a = ap.parse_args(argv)
    print(json.dumps(rows(a) if a.what == "rows" else dn_int(a)))


if __name__ == "__main__":
    main()
