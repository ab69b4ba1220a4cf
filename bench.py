"""Benchmark of the B200 ternary decode path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--kind 5|0]

Workload: the group-128 ternary matvec at the Qwen3-1.7B MLP gate/up shape,
K=2048, N=6144, trit5 codes (kind 5; --kind 0 for the 2-bit image), weights drawn i.i.d. with
P(w=0)=0.4, P(+-1)=0.3, fp16 scales |N(0,1)|*0.02, x ~ N(0,1).  Copy 0 is the exact seed-0 draw of
the reference's generator; the other copies are independent device draws of the same
distribution.  One step = one launch over `--copies` distinct weight copies (96 copies = 264 MB,
more than the 126 MB L2, so every step streams from HBM) and as many distinct activations:
each copy is quantised (the firmware's pow-2 int8), multiplied in the engine's exact integer
arithmetic and scaled to fp32 (firmware/infer_float.c:398 infer_matvec_f).

`value`: whole-job GB/s of algorithmic bytes (scales + codes, no row padding, plus x and y) with
inputs resident in HBM; `e2e`: the same through the public API with x copied host->device and y
device->host every step; `roofline`: the matvec kernel's achieved bandwidth against the
measured HBM copy peak; `cpu_baseline`: the C oracle on this host's cores.

Multi-GPU (torchrun): every rank runs its own copies (weak scaling, no collective on the data
path); the time is the max over ranks.
"""

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

# Symmetric (peer-mapped) buffers of the tensor-parallel leg without NVLink multicast objects.
os.environ.setdefault("TORCH_SYMM_MEM_DISABLE_MULTICAST", "1")
# The tensor-parallel decode leg's exchange (TRX_TP_EXCHANGE): "peer", the kernels over peer
# memory, or "nccl", NCCL all-gathers.
TP_PEER_EXCHANGE = os.environ.get("TRX_TP_EXCHANGE", "peer") == "peer"

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

K_COLS, N_ROWS = 2048, 6144
NOMINAL_HBM_GBS = 8000.0


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


# DRAM traffic (dram__bytes_read.sum + dram__bytes_write.sum) of one 96-copy batch launch of the
# matvec kernel, per kind, from the ncu capture summarised in profiles/matvec_config0_traffic.md,
# with the sha256 of the kernel sources it was captured from.  When the sources have changed since,
# the figure no longer describes the kernel and the line reports null.
KERNEL_TRAFFIC = {
    5: (267236608, "eae26433eef9aaa685f48c62a261732b400e1a9b09d00a734678f71f3be39b8c"),
    0: (323869696, "eae26433eef9aaa685f48c62a261732b400e1a9b09d00a734678f71f3be39b8c"),
}
KERNEL_SOURCES = ("trixium_b200/csrc/trx_matvec.cu", "trixium_b200/csrc/trx_common.cuh")


def kernel_sources_sha():
    import hashlib
    h = hashlib.sha256()
    for f in KERNEL_SOURCES:
        with open(os.path.join(ROOT, f), "rb") as fh:
            h.update(fh.read())
    return h.hexdigest()


def measured_traffic(kind, copies=96):
    """The captured figure, for the 96-copy launch it was captured on and the sources it describes."""
    t = KERNEL_TRAFFIC.get(kind)
    return float(t[0]) if t and copies == 96 and t[1] == kernel_sources_sha() else None


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled while the timed region runs."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "20"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def host_cores():
    """The host threads this process may run on (its CPU affinity, else the machine's count)."""
    try:
        return len(os.sched_getaffinity(0))
    except (AttributeError, OSError):
        return os.cpu_count() or 1


def cpu_baseline(kind, seconds=10.0, threads=None):
    """The C oracle (oracle/trx_oracle.c) on this host: repeated config-0 float projections, on
    every host core (the OpenMP thread count set explicitly: under torchrun OMP_NUM_THREADS is 1)."""
    from oracle import build as cor
    from trixium_b200 import image, layout as L
    lib = cor.lib()
    lib.trxo_set_threads(int(threads or host_cores()))
    t, x = image.synthetic_matvec_case(N_ROWS, K_COLS, seed=0, kind=kind)
    alg = L.algorithmic_bytes(N_ROWS, K_COLS, kind) + 4 * (K_COLS + N_ROWS)
    cor.matvec_f(t.packed, N_ROWS, K_COLS, kind, t.bias, t.rshift, x)   # warm-up
    n, t0 = 0, time.perf_counter()
    while True:
        cor.matvec_f(t.packed, N_ROWS, K_COLS, kind, t.bias, t.rshift, x)
        n += 1
        dt = time.perf_counter() - t0
        if dt >= seconds:
            break
    return {"value": alg * n / dt / 1e9, "unit": "GB/s", "cores": int(lib.trxo_threads()), "kind": "port",
            "sample": f"{n} config-0 float projections (K=2048, N=6144, kind {kind}) in {dt:.1f} s, "
                      f"C oracle oracle/trx_oracle.c, OpenMP over rows"}


def run_reference(args, rank, world):
    """--impl reference: the reference algorithm on the host cores (the C port of the oracle;
    the reference itself is Python that does not travel to the GPU box)."""
    if rank != 0:
        return
    from oracle import build as cor
    from trixium_b200 import image, layout as L
    lib = cor.lib()
    lib.trxo_set_threads(host_cores())  # every host core, also under torchrun (OMP_NUM_THREADS=1)
    t, x = image.synthetic_matvec_case(N_ROWS, K_COLS, seed=0, kind=args.kind)
    alg = L.algorithmic_bytes(N_ROWS, K_COLS, args.kind) + 4 * (K_COLS + N_ROWS)
    for _ in range(args.warmup):
        cor.matvec_f(t.packed, N_ROWS, K_COLS, args.kind, t.bias, t.rshift, x)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        cor.matvec_f(t.packed, N_ROWS, K_COLS, args.kind, t.bias, t.rshift, x)
    dt = time.perf_counter() - t0
    value = alg * args.steps / dt / 1e9
    cores = int(lib.trxo_threads())
    print(json.dumps({
        "impl": "reference", "metric": metric_name(args.kind), "value": value, "unit": "GB/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": dt / args.steps * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "i8", "data": "synthetic",
        "config": workload_config(args),
        "cpu_baseline": {"value": value, "unit": "GB/s", "cores": cores, "kind": "port",
                         "sample": "one config-0 float projection per step (C oracle, OpenMP)"},
        "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def make_batch(ctx, kind, C, dev, rank):
    """The benchmark's weights and inputs on the device: C copies of the config-0 tensor (copy 0 the
    reference generator's seed-0 draw, copies 1..C-1 device draws of the same distribution) with one
    (B, R) for all, C activations; copy 0's float projection checked bit-exact against the C oracle.
    Returns (tensor, job stride, weights, x, y, parity)."""
    import torch
    from trixium_b200 import image, layout as L, ops
    from oracle import build as cor
    t0, x0 = image.synthetic_matvec_case(N_ROWS, K_COLS, seed=0, kind=kind)
    gen = torch.Generator(device=dev)
    gen.manual_seed(1000 + rank)
    scales_all = [torch.from_numpy(t0.scales).to(dev)]
    codes_all = [torch.from_numpy(t0.codes).to(dev)]
    for _ in range(1, C):
        c, s = image.synthetic_codes_scales_torch(gen, N_ROWS, K_COLS, dev)
        codes_all.append(c)
        scales_all.append(s)
    # One (B, R) for every copy so a single entry describes them (max over the copies).
    smax = max(float(s.float().abs().max()) for s in scales_all)
    B = image.scale_bias(np.array([smax], dtype=np.float16))
    R = max(image.result_shift(s.cpu().numpy(), B) for s in scales_all)
    rb = L.row_bytes(K_COLS, kind)
    wstride = N_ROWS * rb
    W = torch.empty(C * wstride, dtype=torch.uint8, device=dev)
    for j in range(C):
        W[j * wstride:(j + 1) * wstride] = image.pack_rows_torch(scales_all[j], codes_all[j], kind)
    del codes_all, scales_all
    X = torch.randn(C, K_COLS, generator=gen, device=dev)
    X[0] = torch.from_numpy(x0).to(dev)
    Y = torch.empty(C, N_ROWS, dtype=torch.float32, device=dev)
    wt = ops.DeviceTensor.from_packed(W, N_ROWS, K_COLS, kind, B, R)
    ops.matvec_f_batch(ctx, wt, wstride, X, K_COLS, Y, N_ROWS, C)
    ctx.raise_on_error()
    y_or, bad = cor.matvec_f(t0.packed if (t0.bias, t0.rshift) == (B, R) else
                             image.pack_rows(t0.scales, t0.codes, kind), N_ROWS, K_COLS, kind, B, R, x0)
    parity = bool(bad == 0 and np.array_equal(Y[0].cpu().numpy().view(np.uint32), y_or.view(np.uint32)))
    return wt, wstride, W, X, Y, parity


def other_kind_leg(ctx, kind, C, steps, warmup, dev, rank, peak):
    """The config-0 batch in the other code image (2-bit beside trit5, or trit5 beside 2-bit): the
    same timing, inputs resident, its own roofline figures."""
    import torch
    from trixium_b200 import layout as L, ops
    wt, wstride, W, X, Y, parity = make_batch(ctx, kind, C, dev, rank)
    for _ in range(warmup):
        ops.matvec_f_batch(ctx, wt, wstride, X, K_COLS, Y, N_ROWS, C)
    torch.cuda.synchronize()
    st = torch.cuda.current_stream()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(st)
    for _ in range(steps):
        ops.matvec_f_batch(ctx, wt, wstride, X, K_COLS, Y, N_ROWS, C)
    b.record(st)
    torch.cuda.synchronize()
    ctx.raise_on_error()
    launch_ms = a.elapsed_time(b) / steps
    alg = (L.algorithmic_bytes(N_ROWS, K_COLS, kind) + 4 * (K_COLS + N_ROWS)) * C
    achieved = alg / (launch_ms * 1e-3) / 1e9
    del wt, W, X, Y
    torch.cuda.empty_cache()
    return {"metric": metric_name(kind), "value": round(achieved, 1), "unit": "GB/s", "ms_per_launch": launch_ms,
            "parity_copy0_bitexact": parity,
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "traffic": measured_traffic(kind, C),
                         "algorithmic_bytes_per_launch": alg}}


def metric_name(kind):
    return f"ternary matvec HBM GB/s (config 0: K=2048 N=6144, {'trit5' if kind == 5 else '2-bit'})"


def workload_config(args):
    return {"workload": f"config0 ternary matvec K={K_COLS} N={N_ROWS} kind={args.kind}, "
                        f"{args.copies} distinct weight copies + activations per step",
            "l2": f"inputs larger than L2 ({args.copies} copies per step)",
            "global_batch": 1, "seq_len": 1, "parallelism": f"replicas{args.gpus}"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--kind", type=int, default=5, choices=[0, 5])
    ap.add_argument("--copies", type=int, default=96)
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-extra", action="store_true", help="skip the per-launch graph and e2e legs")
    ap.add_argument("--no-decode", action="store_true", help="skip the decoder tok/s legs")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        run_reference(args, rank, world)
        return

    import torch
    import torch.distributed as dist
    from trixium_b200 import image, layout as L, ops

    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120))
    dev = torch.device("cuda", local)
    ctx = ops.Context(local)

    kind, C = args.kind, args.copies
    wt, wstride, W, X, Y, parity = make_batch(ctx, kind, C, dev, rank)
    B, R = wt.bias, wt.rshift
    alg_per_copy = L.algorithmic_bytes(N_ROWS, K_COLS, kind) + 4 * (K_COLS + N_ROWS)
    alg_per_step = alg_per_copy * C

    def step():
        ops.matvec_f_batch(ctx, wt, wstride, X, K_COLS, Y, N_ROWS, C)

    sampler = ClockSampler(local)
    sampler.start()
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    # Back-to-back launches between two events: a launch's average duration is the timed region
    # over K (events between launches would serialise each launch's start behind its predecessor's
    # end, which programmatic dependent launch otherwise overlaps).
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(args.steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clocks = sampler.stop()
    ms = e0.elapsed_time(e1)
    launch_ms = ms / args.steps
    ctx.raise_on_error()

    # Per-launch variant: one launch per copy (a single 2.75 MB matvec per kernel), in a CUDA graph.
    single_ms = None
    try:
        if args.no_extra:
            raise RuntimeError("skipped (--no-extra)")
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for _ in range(2):
                for j in range(C):
                    ops.matvec_f(ctx, per_copy(ops, wt, W, j, wstride, kind, B, R), X[j], Y[j])
            torch.cuda.synchronize()
            with torch.cuda.graph(g, stream=s):
                for j in range(C):
                    ops.matvec_f(ctx, per_copy(ops, wt, W, j, wstride, kind, B, R), X[j], Y[j])
        torch.cuda.synchronize()
        for _ in range(3):
            g.replay()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(10):
            g.replay()
        b.record()
        torch.cuda.synchronize()
        single_ms = a.elapsed_time(b) / 10
        del g
    except Exception as exc:  # reported, not fatal
        single_ms = None
        print(f"per-launch graph variant failed: {exc}", file=sys.stderr)

    # e2e: public API with host buffers (pinned), H2D of x and D2H of y inside the timed region.
    Xh = X.cpu().pin_memory()
    Yh = torch.empty(C, N_ROWS, dtype=torch.float32).pin_memory()
    Xd = torch.empty_like(X)

    def e2e_step():
        Xd.copy_(Xh, non_blocking=True)
        ops.matvec_f_batch(ctx, wt, wstride, Xd, K_COLS, Y, N_ROWS, C)
        Yh.copy_(Y, non_blocking=True)

    e2e_steps = 0 if args.no_extra else args.steps
    for _ in range(0 if args.no_extra else args.warmup):
        e2e_step()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    b.record(stream)
    torch.cuda.synchronize()
    e2e_ms = max(a.elapsed_time(b), 1e-9) if e2e_steps else 0.0  # 0: leg skipped (--no-extra)

    if world > 1:
        t = torch.tensor([ms, e2e_ms, launch_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, e2e_ms, launch_ms = t.tolist()
        pt = torch.tensor([1 if parity else 0], device=dev)
        dist.all_reduce(pt, op=dist.ReduceOp.MIN)
        parity = bool(pt.item())

    peak, peak_src = measured_peaks()
    achieved = alg_per_step / (launch_ms * 1e-3) / 1e9
    value = alg_per_step * args.steps * world / (ms * 1e-3) / 1e9
    out = {
        "metric": metric_name(kind), "value": round(value, 1), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "i8",
        "data": "synthetic", "config": workload_config(args),
        "parity_copy0_bitexact": parity,
        "frac_of_8tbs_nominal": round(value / world / NOMINAL_HBM_GBS, 4),
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "peak_source": peak_src,
                     "traffic": measured_traffic(kind, C), "kernel_sources_sha256": kernel_sources_sha(),
                     "algorithmic_bytes_per_launch": alg_per_step,
                     "kernel": "trx::tmv_kernel (trx_matvec_f_batch)"},
        "per_launch_single_matvec": None if single_ms is None else {
            "ms_per_matvec": single_ms / C, "gbs": round(alg_per_copy * C / (single_ms * 1e-3) / 1e9, 1)},
        "e2e": {"value": round(alg_per_step * args.steps * world / (e2e_ms * 1e-3) / 1e9, 1) if e2e_ms > 0 else None,
                "unit": "GB/s",
                "h2d_bytes_per_step": C * K_COLS * 4, "d2h_bytes_per_step": C * N_ROWS * 4},
        "gpu_launches": args.steps,
        "clocks": clocks,
    }
    if world == 1 and not args.no_extra:
        out["other_kind"] = other_kind_leg(ctx, 0 if kind == 5 else 5, C, args.steps, args.warmup, dev, rank, peak)
    if world > 1 and not args.no_decode:
        # Tensor-parallel batch-1 decode: config 2, and config 4 (4 kv heads: replicated above 4 GPUs;
        # the down projection K-segmented) at 4096 of context.
        out["decode"] = {"qwen3-8b": tp_decode_leg(ctx, "qwen3-8b", 1024, 64, 5, rank, world, dev),
                         "hybrid-27b": tp_decode_leg(ctx, "hybrid-27b", 4096, 32, 3, rank, world, dev)}
    if world == 1 and not args.no_decode:
        # The metric's second half: 8B-shape batch-1 decode tok/s (config 2), and config 1.
        out["decode"] = {"qwen3-8b": decode_leg(ctx, "qwen3-8b", 1024, 128, 8),
                         "qwen3-1.7b": decode_leg(ctx, "qwen3-1.7b", 512, 128, 8),
                         # BASELINE configs 3 and 4 at batch 1: 256 tokens after 2048 of context;
                         # 128 tokens at 4096 of context (the down projection K-segmented).
                         "hybrid-2b": decode_leg(ctx, "hybrid-2b", 2048, 256, 8),
                         "hybrid-27b": decode_leg(ctx, "hybrid-27b", 4096, 128, 8)}
        # Config 2 at batch 16: 16 sequences in lockstep on the tensor-core rows projection.
        # Config 4 at batch 32: 32 sequences at 4096 of context, the K-segmented down projection on
        # the tensor cores (trx_matvec_f_rows_kseg).
        out["decode_batch"] = {"qwen3-8b": batch_decode_leg(ctx, "qwen3-8b", 16, 1024, 16, 3),
                               "hybrid-27b": batch_decode_leg(ctx, "hybrid-27b", 32, 4096, 8, 3)}
    if world == 1 and not args.no_decode:
        out["q8_matvec"] = q8_leg(ctx, peak)
        out["batched_rows"] = [rows_leg(ctx, peak, k, nb) for k in (5, 0) for nb in (16, 32)]
    if rank == 0 and world == 1 and not args.no_cpu:
        out["cpu_baseline"] = cpu_baseline(kind, args.cpu_seconds)
    if rank == 0:
        print(json.dumps(out), flush=True)
    ctx.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def q8_leg(ctx, peak, rows=16384, cols=8192, launches=20, warmup=3):
    """The Q8 row-dot matvec (trx_matvec_q8, model/bitexact.py:127-144) on a KIND_Q8 tensor of
    rows x cols int8 weights with fp16 group-32 scales, two copies used in turn (272 MB, above
    L2).  Algorithmic bytes per launch: the weights, the scales, x8 and the int32 results."""
    import numpy as np
    import torch
    from trixium_b200 import image, layout as L, ops
    rng = np.random.default_rng(21)
    G = cols // 32
    s = rng.uniform(0.005, 0.02, (rows, G)).astype(np.float16)
    B = image.scale_bias(s)
    R = image.result_shift(s, B, image.GS_MAX_Q8)
    sb = L.ceil_div(G, L.SCALES_PER_BEAT) * L.BEAT_BYTES
    gen = torch.Generator(device="cuda").manual_seed(21)
    tensors = []
    for _ in range(2):
        packed = torch.zeros(rows, L.q8_row_bytes(cols), dtype=torch.uint8, device="cuda")
        packed[:, :2 * G] = torch.from_numpy(s).cuda().view(torch.uint8)
        packed[:, sb:] = torch.randint(-127, 128, (rows, cols), dtype=torch.int8, device="cuda",
                                       generator=gen).view(torch.uint8)
        tensors.append(ops.DeviceTensor.from_packed(packed.reshape(-1), rows, cols, L.KIND_Q8, B, R))
    x8 = torch.randint(-127, 128, (cols,), dtype=torch.int8, device="cuda", generator=gen)
    y = torch.empty(rows, dtype=torch.int32, device="cuda")
    for i in range(warmup):
        ops.matvec_q8(ctx, tensors[i % 2], x8, y)
    torch.cuda.synchronize()
    st = torch.cuda.current_stream()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(st)
    for i in range(launches):
        ops.matvec_q8(ctx, tensors[i % 2], x8, y)
    b.record(st)
    torch.cuda.synchronize()
    ctx.raise_on_error()
    ms = a.elapsed_time(b) / launches
    alg = rows * (cols + 2 * G) + cols + 4 * rows
    gbs = alg / (ms * 1e-3) / 1e9
    del tensors
    torch.cuda.empty_cache()
    return {"kernel": "trx::q8_matvec_kernel (trx_matvec_q8)", "rows": rows, "cols": cols,
            "launches_timed": launches, "ms_per_launch": round(ms, 4),
            "algorithmic_bytes_per_launch": alg, "achieved_GBps": round(gbs, 1),
            "frac": round(gbs / peak, 4), "inputs": "two tensors in turn, 272 MB > L2"}


def rows_leg(ctx, peak, kind, nb, launches=20, copies=48, warmup=3):
    """The batched path (trx_matvec_f_rows, tcgen05 kind::i8): nb activation rows against one pass
    over a config-0 tensor (K=2048, N=6144), `copies` distinct tensors used in turn (above L2).
    Reports the weight stream (GB/s of algorithmic bytes, as the matvec) and rows x rows per second
    (batched projections)."""
    import torch
    from trixium_b200 import image, layout as L, ops
    gen = torch.Generator(device="cuda").manual_seed(77)
    rb = L.row_bytes(K_COLS, kind)
    tensors = []
    W = torch.empty(copies * N_ROWS * rb, dtype=torch.uint8, device="cuda")
    t0, _ = image.synthetic_matvec_case(N_ROWS, K_COLS, seed=0, kind=kind)
    for j in range(copies):
        c, s = image.synthetic_codes_scales_torch(gen, N_ROWS, K_COLS, "cuda")
        W[j * N_ROWS * rb:(j + 1) * N_ROWS * rb] = image.pack_rows_torch(s, c, kind)
        tensors.append(ops.DeviceTensor.from_packed(W[j * N_ROWS * rb:(j + 1) * N_ROWS * rb], N_ROWS, K_COLS, kind,
                                                    t0.bias, t0.rshift))
    X = torch.randn(nb, K_COLS, generator=gen, device="cuda")
    Y = torch.empty(nb, N_ROWS, device="cuda")
    for i in range(warmup):
        ops.matvec_f_rows(ctx, tensors[i % copies], X, Y)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for i in range(launches):
        ops.matvec_f_rows(ctx, tensors[i % copies], X, Y)
    b.record()
    torch.cuda.synchronize()
    ctx.raise_on_error()
    ms = a.elapsed_time(b) / launches
    alg = L.algorithmic_bytes(N_ROWS, K_COLS, kind) + 4 * nb * (K_COLS + N_ROWS)
    del tensors, W
    torch.cuda.empty_cache()
    return {"kernel": "trx::rows_kernel (trx_matvec_f_rows: tcgen05.mma kind::i8, TMEM accumulators)",
            "kind": "trit5" if kind == 5 else "2-bit", "rows": N_ROWS, "cols": K_COLS, "batch": nb,
            "ms_per_launch": round(ms, 4), "weight_GBps": round(alg / (ms * 1e-3) / 1e9, 1),
            "frac": round(alg / (ms * 1e-3) / 1e9 / peak, 4),
            "row_projections_per_s": round(nb / (ms * 1e-3), 1),
            "inputs": f"{copies} tensors in turn ({copies * N_ROWS * rb / 1e6:.0f} MB > L2), includes the rows' quantisation launch"}


def decode_leg(ctx, name, ctx_len, n_tokens, warmup):
    """Batch-1 greedy decode tok/s of a BASELINE decoder config on synthetic random-init weights:
    one CUDA graph per token (trixium_b200.decoder), `ctx_len` positions of synthetic context in
    the caches, the token fed back on the device.  `e2e_tok_s` runs the public generate() API
    (prompt from the host, token ids back to the host)."""
    import torch
    from trixium_b200 import decoder as D
    cfg = D.CONFIGS[name]
    w = D.SyntheticWeights(cfg, seed=0)
    dec = D.Decoder(w, ctx=ctx, max_pos=ctx_len + 2 * n_tokens + warmup + 8)
    dec.set_states(1)
    dec.fill_context(ctx_len)
    dec.tok.fill_(7)
    dec.capture()
    for _ in range(warmup):
        dec.graph.replay()
    torch.cuda.synchronize()
    dec.fill_context(ctx_len)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(n_tokens):
        dec.graph.replay()
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / n_tokens
    ctx.raise_on_error()
    dec.fill_context(ctx_len)
    t0 = time.perf_counter()
    toks = dec.generate([7], n_tokens)
    e2e_s = time.perf_counter() - t0
    wb = cfg.weight_bytes_per_token()
    out = {"config": name, "kind": "trit5" if cfg.kind == 5 else "2-bit", "context": ctx_len, "batch": 1,
           "tokens_timed": n_tokens, "ms_per_token": round(ms, 4), "tok_s": round(1000.0 / ms, 1),
           "e2e_tok_s": round(n_tokens / e2e_s, 1), "weight_bytes_per_token": wb,
           "weight_GBps": round(wb / (ms * 1e-3) / 1e9, 1), "launches_per_token": dec.launches_per_step(),
           "distinct_tokens": len(set(toks))}
    del dec, w
    torch.cuda.empty_cache()
    return out


def batch_decode_leg(ctx, name, nseq, ctx_len, n_tokens, warmup):
    """Batched greedy decode (trixium_b200.decoder.BatchDecoder; BASELINE config 2 at batch 16, config 4
    at batch 32):
    nseq sequences in lockstep, every projection one tensor-core launch over their rows, one CUDA
    graph per step.  tok_s counts every sequence's tokens."""
    import torch
    from trixium_b200 import decoder as D
    cfg = D.CONFIGS[name]
    w = D.SyntheticWeights(cfg, seed=0)
    dec = D.BatchDecoder(w, nseq, ctx=ctx, max_pos=ctx_len + n_tokens + warmup + 8)
    dec.fill_context(ctx_len)
    dec.tok.copy_(torch.arange(7, 7 + nseq, dtype=torch.int32))
    dec.capture()
    for _ in range(warmup):
        dec.graph.replay()
    torch.cuda.synchronize()
    dec.fill_context(ctx_len)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(n_tokens):
        dec.graph.replay()
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / n_tokens
    ctx.raise_on_error()
    wb = cfg.weight_bytes_per_token()
    out = {"config": name, "kind": "trit5" if cfg.kind == 5 else "2-bit", "context": ctx_len, "batch": nseq,
           "steps_timed": n_tokens, "ms_per_step": round(ms, 4), "tok_s": round(nseq * 1000.0 / ms, 1),
           "weight_bytes_per_step": wb, "weight_GBps": round(wb / (ms * 1e-3) / 1e9, 1),
           "kernel": "trx::rows_kernel (tcgen05.mma kind::i8) for every projection"}
    del dec, w
    torch.cuda.empty_cache()
    return out


def tp_decode_leg(ctx, name, ctx_len, n_tokens, warmup, rank, world, dev):
    """Tensor-parallel batch-1 decode tok/s over `world` GPUs (trixium_b200.tp): every rank draws the
    same synthetic image and keeps its row shard; one CUDA graph per token holds the kernels, which
    exchange the sharded vectors themselves over peer memory as tagged words (TRX_TP_EXCHANGE=nccl:
    NCCL all-gathers instead); the time is the max over ranks."""
    import torch
    import torch.distributed as dist
    from trixium_b200 import decoder as D, tp
    cfg = D.CONFIGS[name]
    full = D.SyntheticWeights(cfg, seed=0)
    dec = tp.TPDecoder(tp.TPWeights(full, rank, world), ctx=ctx, max_pos=ctx_len + n_tokens + warmup + 8, p2p=TP_PEER_EXCHANGE)
    del full
    torch.cuda.empty_cache()
    dec.set_states(1)
    dec.fill_context(ctx_len)
    dec.tok.fill_(7)
    dec.capture()
    for _ in range(warmup):
        dec.graph.replay()
    torch.cuda.synchronize()
    dec.fill_context(ctx_len)
    dist.barrier()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(n_tokens):
        dec.graph.replay()
    b.record()
    torch.cuda.synchronize()
    t = torch.tensor([a.elapsed_time(b) / n_tokens], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    ctx.raise_on_error()
    dec.release()
    wb = cfg.weight_bytes_per_token()
    out = {"config": name, "kind": "trit5" if cfg.kind == 5 else "2-bit", "context": ctx_len, "batch": 1,
           "tensor_parallel": world, "scaling": "strong", "tokens_timed": n_tokens, "ms_per_token": round(ms, 4),
           "tok_s": round(1000.0 / ms, 1), "weight_bytes_per_token": wb,
           "weight_GBps_all_gpus": round(wb / (ms * 1e-3) / 1e9, 1),
           "exchange": "peer memory (kernels)" if dec.p2p else "nccl all-gather",
           "collectives_per_token": dec.collectives_per_step()}
    del dec
    torch.cuda.empty_cache()
    return out


_pc_cache = {}


def per_copy(ops, wt, W, j, wstride, kind, B, R):
    key = j
    if key not in _pc_cache:
        _pc_cache[key] = ops.DeviceTensor.from_packed(W[j * wstride:(j + 1) * wstride], N_ROWS, K_COLS, kind, B, R)
    return _pc_cache[key]


if __name__ == "__main__":
    main()
