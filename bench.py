"""Benchmark: GPTQ-INT4 rot-256 Mparams quantized/s (BASELINE.json metric, config 3).

A "step" quantizes one synthetic DiT linear set -- qkv [12288,4096],
proj [4096,4096], mlp_up [16384,4096], mlp_down [4096,16384] (201.3 M params)
-- through the whole per-layer hot path: rotate W (fp16 in HBM) and its
Hessian, row scales / zero-points, damping, tensor-core inverse, GPTQ column
loop with the lazy tensor-core update, INT4 packing and the verify statistics.
Each layer's Hessian is H = X^T X / 8192 with X rows N(0, diag(s^2)),
s ~ LogNormal(0, 1) (seeded, generated on the device before timing).  Sets are
resident in HBM (~1.7 GB each, far larger than L2) and cycled, so no step
reads a warm input.

Modes:
  python bench.py [--gpus N --steps K --warmup W]      B200 path (one process per GPU)
  python bench.py --impl reference ...                 the reference's CPU algorithm (oracle
                                                       restatement) on the host cores
Layers are issued on four CUDA streams (LayerStreams), so consecutive steps
overlap; the default 24 steps measure that steady state.
Multi-GPU: each rank quantizes its own sets (layers are independent, weak
scaling); timing is the max over ranks of the device-event time.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

from int_crush_converter_b200.sharding import max_over_ranks  # noqa: E402

# (name, out_features, in_features) of one DiT linear set (config 3)
LAYERS = [("qkv", 12288, 4096), ("proj", 4096, 4096), ("mlp_up", 16384, 4096), ("mlp_down", 4096, 16384)]
PARAMS_PER_SET = sum(m * n for _, m, n in LAYERS)
BLOCK_COLS = 128
# algorithmic flop of one set: GPTQ trailing updates 2*M*N*(N-B) + the inverse N^3
# (Cholesky, triangular inverse and U*U^T at N^3/3 each)
FLOP_PER_SET = sum(2 * m * n * (n - BLOCK_COLS) + n ** 3 for _, m, n in LAYERS)
N_SAMPLES = 8192
ROT, BLOCK, DAMP = 256, 128, 0.01
METRIC = "GPTQ-INT4 rot256 Mparams quantized/s"
CONFIG = {"workload": "config 3: GPTQ INT4 rot256, block 128, damping 0.01; one step = one synthetic DiT linear "
                      "set qkv[12288,4096] proj[4096,4096] mlp_up[16384,4096] mlp_down[4096,16384] (201.3M params), "
                      "fp16 W ~ N(0,0.02^2), H = X^T X/8192 with X rows N(0, diag(s^2)), s ~ LogNormal(0,1)",
          "rot_size": ROT, "block_size": BLOCK, "damping": DAMP, "int_bits": 4,
          "l2": "inputs larger than L2 (each set ~1.7 GB, sets cycled)"}


def make_set(seed: int, dev: torch.device):
    """One synthetic linear set on the device: fp16 W ~ N(0, 0.02^2), H = X^T X / 8192."""
    g = torch.Generator(device=dev).manual_seed(seed)
    out = []
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    for li, (name, m, n) in enumerate(LAYERS):
        W = (torch.randn(m, n, generator=g, device=dev) * 0.02).half()
        s = torch.exp(torch.randn(n, generator=g, device=dev))  # LogNormal(0, 1) channel scales
        H = torch.zeros(n, n, device=dev)
        for c0 in range(0, N_SAMPLES, 2048):  # X in chunks to bound the temporary
            X = torch.randn(min(2048, N_SAMPLES - c0), n, generator=g, device=dev) * s
            H.addmm_(X.T, X)
            del X
        H.div_(N_SAMPLES)
        H = 0.5 * (H + H.T)
        out.append((name, W, H))
    torch.backends.cuda.matmul.allow_tf32 = prev
    return out


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.lines: list[str] = []
        self.t = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.idx), f"--query-gpu={self.QUERY}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = max(mx, float(f[2]))
            except ValueError:
                continue
            for nm, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx or None,
                "reasons": sorted(reasons), "samples": len(sm)}


# ----------------------------------------------------------------------------- reference (CPU) arm
REF_DIR = os.path.join(ROOT, "baseline", "_ref")


def _reference_converter():
    """The unmodified reference package installed under baseline/_ref (pip --target),
    with its Triton path switched off through its own switch (gptq.py:24) so that
    it runs its CPU PyTorch code; None when it is not installed."""
    os.environ["GPTQ_DISABLE_TRITON"] = "1"
    if not os.path.isdir(os.path.join(REF_DIR, "converter")):
        return None
    if REF_DIR not in sys.path:
        sys.path.insert(0, REF_DIR)
    import importlib
    return {m: importlib.import_module(f"converter.{m}") for m in ("rotation", "gptq", "packing")}


def cpu_layer_inputs(name: str, m: int, n: int, seed: int):
    """Seeded CPU inputs of one layer with the bench's distributions (fp16-valued
    W upcast to fp32 as pipeline.py:524 does; H = X^T X / 8192)."""
    g = torch.Generator().manual_seed(seed)
    W = (torch.randn(m, n, generator=g) * 0.02).half().float()
    s = torch.exp(torch.randn(n, generator=g))
    H = torch.zeros(n, n)
    for c0 in range(0, N_SAMPLES, 2048):
        X = torch.randn(min(2048, N_SAMPLES - c0), n, generator=g) * s
        H.addmm_(X.T, X)
    H.div_(N_SAMPLES)
    return W, 0.5 * (H + H.T)


def reference_layer_seconds(ref, W, H) -> float:
    """One layer through the reference's own per-layer calls, as pipeline.py:547-559,
    702-789 and 1010-1013 make them: rotate_weights -> rotate_hessian ->
    gptq_quantize_layer -> pack_int4 (CPU tensors)."""
    t0 = time.perf_counter()
    Wr = ref["rotation"].rotate_weights(W, ROT)
    Hr = ref["rotation"].rotate_hessian(H, ROT)
    r = ref["gptq"].gptq_quantize_layer(Wr, Hr, block_size=BLOCK, damping=DAMP, int_bits=4)
    ref["packing"].pack_int4(r.quantized_W)
    return time.perf_counter() - t0


def cpu_sample_seconds(reps: int = 1):
    """The reference's CPU path on the proj layer [4096, 4096] of a seeded set
    (baseline/_ref when installed, else the oracle restatement); returns
    (seconds per rep, params, kind)."""
    name, m, n = LAYERS[1]
    ref = _reference_converter()
    if ref is not None:
        W, H = cpu_layer_inputs(name, m, n, 4321)
        return [reference_layer_seconds(ref, W, H) for _ in range(reps)], m * n, "reference"
    from oracle import cpu_ref as R
    from tests.golden import inputs as gi
    W = gi.weight_outlier_cols(1234, m, n, frac=0.0005, mult=1.0)
    H = gi.hessian_lognormal(4321, n, N_SAMPLES)
    ts = []
    for _ in range(reps):
        t0 = time.perf_counter()
        r = R.gptq_quantize_layer(R.rotate_weights(W, ROT), R.rotate_hessian(H, ROT), BLOCK, DAMP, 4)
        R.pack_int4(r["quantized_W"])
        ts.append(time.perf_counter() - t0)
    return ts, m * n, "port"


def cpu_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def run_reference(args, rank: int, world: int) -> None:
    """The reference's own CPU implementation on the B200 arm's config: one step =
    one DiT linear set (qkv, proj, mlp_up, mlp_down) through its per-layer calls,
    all host threads.  A set takes about a minute of CPU, so the timed steps stop
    at --ref-budget seconds (after at least one whole set); `steps` reports the
    sets actually timed.  Warm-up steps run the proj layer only."""
    if rank != 0:
        return
    ref = _reference_converter()
    if ref is None:
        print(json.dumps({"impl": "reference", "unavailable": "reference not installed under baseline/_ref "
                                                               "(pip install --target baseline/_ref)"}), flush=True)
        return
    torch.set_num_threads(cpu_cores())
    inputs = {name: cpu_layer_inputs(name, m, n, 77 + i) for i, (name, m, n) in enumerate(LAYERS)}
    for _ in range(args.warmup):
        reference_layer_seconds(ref, *inputs["proj"])
    per_layer: dict[str, list[float]] = {name: [] for name, _, _ in LAYERS}
    total, sets = 0.0, 0
    t_start = time.perf_counter()
    while sets < args.steps:
        for name, _, _ in LAYERS:
            per_layer[name].append(reference_layer_seconds(ref, *inputs[name]))
        sets += 1
        if time.perf_counter() - t_start > args.ref_budget:
            break
    total = sum(sum(v) for v in per_layer.values())
    val = PARAMS_PER_SET * sets / total / 1e6
    sample = (f"{sets} whole set(s) of 4 layers through the reference's own converter.rotation.rotate_weights -> "
              f"rotate_hessian -> gptq.gptq_quantize_layer -> packing.pack_int4 on CPU tensors "
              f"(baseline/_ref, GPTQ_DISABLE_TRITON=1), torch threads {torch.get_num_threads()}")
    line = {
        "impl": "reference", "metric": METRIC, "value": round(val, 4), "unit": "Mparams/s", "n_gpus": world,
        "steps": sets, "steps_requested": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1e3 * total / sets, 2),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": dict(CONFIG, parallelism="host cores"),
        "per_layer_s": {k: round(sum(v) / len(v), 3) for k, v in per_layer.items()},
        "cpu_baseline": {"value": round(val, 4), "unit": "Mparams/s", "cores": torch.get_num_threads(),
                         "kind": "reference", "sample": sample},
        "e2e": {"value": round(val, 4), "unit": "Mparams/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------- B200 arm
def dominant_gemm_tflops(dev: torch.device, n: int = 16384, reps: int = 3) -> tuple[float, float]:
    """The dominant kernel (3xTF32 tcgen05 GEMM) at the largest shape a step runs
    (the n x n x n product H^-1 = U U^T of the mlp_down inverse), timed with CUDA
    events on the launching stream.  Returns (algorithmic TFLOP/s, ms per launch)."""
    from int_crush_converter_b200 import _native as nat
    lib = nat.load()
    g = torch.Generator(device=dev).manual_seed(7)
    hi = torch.randn(n, n, generator=g, device=dev)
    lo = torch.zeros_like(hi)
    out_hi = torch.empty_like(hi)
    out_lo = torch.empty_like(hi)
    st = nat.stream_ptr(dev)

    def go():
        nat.check(lib.ic_gemm_tn(n, n, n, 1.0, hi.data_ptr(), lo.data_ptr(), n, hi.data_ptr(), lo.data_ptr(), n,
                                 0.0, None, None, n, out_hi.data_ptr(), out_lo.data_ptr(), n, 3, st), "gemm")
    go()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        go()
    e1.record()
    torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1) / reps
    del hi, lo, out_hi, out_lo
    return 2.0 * n ** 3 / (ms * 1e-3) / 1e12, ms


def run_device(args, rank: int, world: int) -> None:
    import int_crush_converter_b200 as B
    from int_crush_converter_b200 import _native as nat

    local = int(os.environ.get("LOCAL_RANK", 0))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    nat.require_device(dev)
    n_sets = max(1, min(args.sets, args.steps))
    sets = [make_set(1000 * rank + i, dev) for i in range(n_sets)]
    pool = B.LayerStreams(args.streams, dev)

    def step(i):
        for name, W, H in sets[i % n_sets]:
            pool.submit(W, H, rot_size=ROT, block_size=BLOCK, damping=DAMP)

    with pool:
        for i in range(args.warmup):
            step(i)
    torch.cuda.synchronize(dev)
    if world > 1:
        torch.distributed.barrier()
    lib = nat.load()
    cvd = os.environ.get("CUDA_VISIBLE_DEVICES", "")
    phys = int(cvd.split(",")[local]) if cvd and cvd.split(",")[local].strip().isdigit() else local
    with ClockSampler(phys) as clk:
        l0 = lib.ic_launch_count()
        g0 = lib.ic_inverse_graph_count()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize(dev)
        e0.record()
        pool.fork()
        for i in range(args.steps):
            step(i)
        pool.join()
        e1.record()
        torch.cuda.synchronize(dev)
        launches = lib.ic_launch_count() - l0
        graphs = lib.ic_inverse_graph_count() - g0
    pool.check()
    if world > 1:
        torch.distributed.barrier()
    ms_max = max_over_ranks(e0.elapsed_time(e1), dev)
    value = PARAMS_PER_SET * args.steps * world / (ms_max * 1e-3) / 1e6
    del sets
    torch.cuda.empty_cache()

    e2e = run_e2e(args, dev, pool, world)
    if rank != 0:
        return
    achieved, gemm_ms = dominant_gemm_tflops(dev)
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except (OSError, ValueError):
        pass
    bf16 = peaks.get("bf16_tflops", 1590.0)
    peak = bf16 / 2.0 / 3.0  # TF32 runs at half the bf16 rate; 3xTF32 issues three products
    cpu_ts, cpu_params, cpu_kind = cpu_sample_seconds(1)
    cpu_val = cpu_params / cpu_ts[0] / 1e6
    line = {
        "metric": METRIC, "value": round(value, 3), "unit": "Mparams/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_max / args.steps, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32 (3xTF32 inverse; TF32 products with fp32 accumulation for the GPTQ trailing update)", "data": "synthetic",
        "config": dict(CONFIG, parallelism=f"layer sets sharded over {world} GPU(s), no collective",
                       streams=args.streams),
        "e2e": e2e,
        "gpu_launches": int(launches),
        "inverse_graphs_instantiated_in_timed_region": int(graphs),
        "roofline": {"bound": "tensor", "achieved": round(achieved, 2), "peak": round(peak, 2), "unit": "TFLOP/s",
                     "frac": round(achieved / peak, 4), "traffic": TRAFFIC_BYTES,
                     "kernel": "gemm_tn_kernel<128,3> (3xTF32), 16384^3 product of the mlp_down inverse, "
                               f"{gemm_ms:.2f} ms/launch",
                     "peak_basis": ("measured bf16 burst / 2 (TF32 rate) / 3 (3xTF32 products), of measured"
                                    if "bf16_tflops" in peaks else "fallback 1.59 PF bf16 / 2 / 3, of fallback")},
        "step_roofline": {"bound": "tensor", "flop_per_step": FLOP_PER_SET,
                          "target_ms": round(FLOP_PER_SET / (peak * 1e12) * 1e3, 3),
                          "ms_per_step": round(ms_max / args.steps, 3),
                          "frac": round(FLOP_PER_SET / (peak * 1e12) * 1e3 / (ms_max / args.steps), 4),
                          "note": "whole step's algorithmic flop over the 3xTF32 peak, of measured"},
        "cpu_baseline": {"value": round(cpu_val, 4), "unit": "Mparams/s", "cores": torch.get_num_threads(),
                         "kind": cpu_kind,
                         "sample": "one proj layer [4096,4096] through the reference's CPU calls (rotate_weights, "
                                   "rotate_hessian, gptq_quantize_layer, pack_int4; baseline/_ref) or, when it "
                                   "is not installed, oracle/cpu_ref.py"},
        "clocks": clk.summary(),
    }
    print(json.dumps(line), flush=True)


# DRAM bytes (read + write) of the 16384^3 3xTF32 product timed by dominant_gemm_tflops (its four
# K-slab launches together), from the ncu capture in profiles/gemm_tn_3xtf32_16384_traffic.md
TRAFFIC_BYTES = 77_440_000_000


def run_e2e(args, dev: torch.device, pool, world: int) -> dict:
    """Same metric through the public API with HOST buffers: every step copies one
    set's fp16 weights and fp32 Hessians from pinned host memory, quantizes, and
    reads back the packed codes, scales and zero-points."""
    host = []
    for name, W, H in make_set(99, dev):
        host.append((name, W.cpu().pin_memory(), H.cpu().pin_memory()))
    torch.cuda.empty_cache()
    res = {}
    for name, m, n in LAYERS:
        res[name] = (torch.empty(m, n // 2, dtype=torch.uint8).pin_memory(),
                     torch.empty(m, 1, dtype=torch.float16).pin_memory(),
                     torch.empty(m, 1, dtype=torch.int8).pin_memory())
    h2d = sum(W.numel() * 2 + H.numel() * 4 for _, W, H in host)
    d2h = sum(p.numel() + s.numel() * 2 + z.numel() + 3 * 8 for p, s, z in res.values())
    steps = max(1, min(args.steps, args.e2e_steps))

    st = {name: torch.empty(3, dtype=torch.float64).pin_memory() for name, _, _ in LAYERS}

    def step():
        for name, Wh, Hh in host:
            p, s, z = res[name]

            def fetch(o, p=p, s=s, z=z, name=name):
                p.copy_(o["packed"], non_blocking=True)
                s.copy_(o["scales"], non_blocking=True)
                z.copy_(o["zero_points"], non_blocking=True)
                st[name].copy_(o["stats"], non_blocking=True)
            pool.submit(Wh, Hh, rot_size=ROT, block_size=BLOCK, damping=DAMP, then=fetch)

    with pool:
        step()
    torch.cuda.synchronize(dev)
    if world > 1:
        torch.distributed.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    pool.fork()
    for _ in range(steps):
        step()
    pool.join()
    e1.record()
    torch.cuda.synchronize(dev)
    pool.check()
    val = PARAMS_PER_SET * steps * world / (max_over_ranks(e0.elapsed_time(e1), dev) * 1e-3) / 1e6
    return {"value": round(val, 3), "unit": "Mparams/s", "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
            "steps": steps, "api": "int_crush_converter_b200.LayerStreams.submit -> quantize_gptq_layer (C ABI ic_gptq_layer)"}


def run_hbm_kernels(reps: int = 5) -> None:
    """HBM-bound kernels of the path at the BASELINE configs' shapes, each timed
    alone with CUDA events and reported against the measured copy bandwidth.
    Algorithmic bytes (the minimum a kernel must move):
      rtn_fused (config 1: fp16 W [4096,4096] x 8 layers, INT4 sym rot256):
          2 B read + 0.5 B packed written per weight (+ 2 B scale per row)
      rotate_weights (fp16 -> fp32 rot256, [4096,16384]): 2 B read + 4 B written per weight
      rotate_hessian (fp32 H [16384,16384] -> rotated TF32 hi/lo pair, rot256):
          4 B read + 8 B written per element"""
    from int_crush_converter_b200 import _native as nat
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    nat.require_device(dev)
    lib = nat.load()
    st = nat.stream_ptr(dev)
    try:
        peak = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))["hbm_gbs"]
        basis = "of measured"
    except (OSError, ValueError, KeyError):
        peak, basis = 6650.0, "of fallback"
    g = torch.Generator(device=dev).manual_seed(11)

    def timed(fn, nbytes):
        fn()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            fn()
        e1.record()
        torch.cuda.synchronize(dev)
        ms = e0.elapsed_time(e1) / reps
        gbs = nbytes / (ms * 1e-3) / 1e9
        return round(ms, 4), round(gbs, 1), round(gbs / peak, 4)

    out = []
    # config 1: RTN INT4 sym rot256 over 8 fp16 layers (256 MB of input, larger than L2)
    Ws = [(torch.randn(4096, 4096, generator=g, device=dev) * 0.02).half() for _ in range(8)]
    packed = torch.empty(4096, 2048, dtype=torch.uint8, device=dev)
    sc = torch.empty(4096, dtype=torch.float16, device=dev)
    sq = torch.empty(4096, dtype=torch.float64, device=dev)
    mx = torch.empty(4096, dtype=torch.float32, device=dev)

    def rtn():
        for W in Ws:
            nat.check(lib.ic_rtn_fused(W.data_ptr(), nat.IC_F16, 4096, 4096, 4096, 256, 4, 0, None, 0, None,
                                       packed.data_ptr(), sc.data_ptr(), None, sq.data_ptr(), mx.data_ptr(), st))
    ms, gbs, frac = timed(rtn, 8 * (4096 * 4096 * 2.5 + 4096 * 2))
    out.append(dict(kernel="rtn_regs_kernel (ic_rtn_fused)", workload="config 1: 8 x fp16 [4096,4096] INT4 sym rot256",
                    ms_per_call=ms, achieved_gbs=gbs, frac=frac))
    del Ws
    W = (torch.randn(4096, 16384, generator=g, device=dev) * 0.02).half()
    Wr = torch.empty(4096, 16384, device=dev)

    def rot():
        nat.check(lib.ic_rotate_weights(W.data_ptr(), nat.IC_F16, 4096, 16384, 16384, 256, Wr.data_ptr(), 16384, st))
    ms, gbs, frac = timed(rot, 4096 * 16384 * 6)
    out.append(dict(kernel="rotate_regs_kernel (ic_rotate_weights)", workload="fp16 [4096,16384] -> fp32, rot256",
                    ms_per_call=ms, achieved_gbs=gbs, frac=frac))
    del W, Wr
    n = 16384
    H = torch.randn(n, n, generator=g, device=dev)
    hh = torch.empty(n, n, device=dev)
    hl = torch.empty(n, n, device=dev)

    def roth():
        nat.check(lib.ic_rotate_hessian(H.data_ptr(), 1, n, n, 256, hh.data_ptr(), hl.data_ptr(), n, st))
    ms, gbs, frac = timed(roth, n * n * 12)
    out.append(dict(kernel="rotate_regs_kernel + hess_cols256_kernel (ic_rotate_hessian)",
                    workload="fp32 H [16384,16384] -> hi/lo pair, rot256", ms_per_call=ms, achieved_gbs=gbs,
                    frac=frac))
    for o in out:
        o.update(unit="GB/s", peak_gbs=peak, peak_basis=basis, bound="hbm")
        print(json.dumps(o), flush=True)


def run_configs() -> None:
    """The BASELINE configs other than the headline one, each through the public
    API on device-resident synthetic inputs of the config's shapes (seeded),
    timed with CUDA events after a warm-up; one JSON line per config."""
    import int_crush_converter_b200 as B
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    g = torch.Generator(device=dev).manual_seed(21)

    def timed(fn, reps):
        fn()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            fn()
        e1.record()
        torch.cuda.synchronize(dev)
        return e0.elapsed_time(e1) / reps

    def weights(m, n, std, outlier_frac=0.0, outlier_mult=1.0):
        W = torch.randn(m, n, generator=g, device=dev) * std
        if outlier_frac:
            k = max(1, int(n * outlier_frac))
            cols = torch.randperm(n, generator=g, device=dev)[:k]
            W[:, cols] *= outlier_mult
        return W.half()

    lines = []
    # config 1: RTN INT4 sym rot256, 8 x [4096,4096]
    W1 = [weights(4096, 4096, 0.02, 0.001, 20.0) for _ in range(8)]
    ms = timed(lambda: [B.rtn_quantize_fused(W, 256, int_bits=4, want_codes=False) for W in W1], 3)
    lines.append(dict(config=1, workload="RTN INT4 sym rot256, 8 fp16 layers [4096,4096]", params=8 * 4096 * 4096, ms=ms))
    del W1
    # config 2: RTN INT8 sym rot64 with the clipping-ratio search, 16 x [3072,3072] + 16 x [12288,3072]
    t = torch.distributions.StudentT(torch.tensor(3.0, device=dev))

    def w2(m, n):
        W = torch.randn(m, n, generator=g, device=dev) * 0.02
        mask = torch.rand(m, n, generator=g, device=dev) < 0.01
        W = W + mask * (0.02 * t.sample((m, n)))
        return W.half()
    W2 = [w2(3072, 3072) for _ in range(16)] + [w2(12288, 3072) for _ in range(16)]
    ratios = [0.8, 0.85, 0.9, 0.95, 1.0]
    ms = timed(lambda: [B.rtn_quantize_fused(W, 64, int_bits=8, clipping_ratios=ratios, want_codes=True,
                                             want_packed=False) for W in W2], 2)
    lines.append(dict(config=2, workload="RTN INT8 sym rot64, clipping ratios {0.8..1.0}, 16 x [3072,3072] + "
                      "16 x [12288,3072] fp16 (N(0,0.02^2) + Student-t(3) tails on 1%)",
                      params=16 * 3072 * 3072 + 16 * 12288 * 3072, ms=ms))
    del W2
    # config 4: LDLQ INT4 rot256, 2 iterations, 8 greedy passes, weight-only Hessian; one [8192,8192] layer
    W4 = weights(8192, 8192, 0.015, 0.0005, 30.0)

    def ldlq():
        Wr = B.rotate_weights(W4, 256)
        return B.ldlq_quantize_layer(Wr, None, block_size=128, int_bits=4, iterations=2, greedy_passes=8)
    import warnings
    with warnings.catch_warnings():
        warnings.simplefilter("ignore")
        ms = timed(ldlq, 1)
    lines.append(dict(config=4, workload="LDLQ INT4 rot256, 2 iterations, 8 greedy passes, weight-only Hessian, "
                      "one fp16 layer [8192,8192] (N(0,0.015^2), 0.05% columns x30)", params=8192 * 8192, ms=ms))
    for d in lines:
        d.update(metric="Mparams quantized/s", value=round(d["params"] / (d["ms"] * 1e-3) / 1e6, 2),
                 ms=round(d["ms"], 3), data="synthetic, device-resident")
        print(json.dumps(d), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=24)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--sets", type=int, default=8, help="distinct resident sets per GPU (cycled)")
    ap.add_argument("--e2e-steps", type=int, default=12)
    ap.add_argument("--ref-budget", type=float, default=150.0,
                    help="reference arm: stop the timed sets after this many seconds (at least one set)")
    ap.add_argument("--streams", type=int, default=4, help="CUDA streams the layers are issued on")
    ap.add_argument("--gemm-only", type=int, default=0,
                    help="time only the dominant 3xTF32 GEMM at n^3 (small profiling case)")
    ap.add_argument("--hbm-kernels", action="store_true",
                    help="time the HBM-bound kernels (RTN, rotations) alone and exit")
    ap.add_argument("--one-step", action="store_true",
                    help="quantize one set once and exit (for an ncu launch list of exactly one step)")
    ap.add_argument("--configs", action="store_true", help="time BASELINE configs 1, 2 and 4 and exit")
    args = ap.parse_args()
    if args.configs:
        run_configs()
        return
    if args.one_step:
        import int_crush_converter_b200 as B
        dev = torch.device("cuda", 0)
        torch.cuda.set_device(dev)
        s = make_set(0, dev)
        torch.cuda.synchronize(dev)
        with B.LayerStreams(args.streams, dev) as pool:
            for _, W, H in s:
                pool.submit(W, H, rot_size=ROT, block_size=BLOCK, damping=DAMP)
        torch.cuda.synchronize(dev)
        print(json.dumps({"one_step": "ok", "layers": len(s)}))
        return
    if args.hbm_kernels:
        run_hbm_kernels()
        return
    if args.gemm_only:
        dev = torch.device("cuda", 0)
        tf, ms = dominant_gemm_tflops(dev, n=args.gemm_only, reps=2)
        print(json.dumps({"gemm_n": args.gemm_only, "tflops": round(tf, 2), "ms": round(ms, 3)}))
        return
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    if world > 1:
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", 0)))
        torch.distributed.init_process_group("nccl")
    try:
        run_device(args, rank, world)
    finally:
        if world > 1:
            torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
