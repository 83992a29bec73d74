"""Benchmark: GPTQ-INT4 rot-256 Mparams quantized/s (BASELINE.json metric) on a
fixed model at 1/2/4/8 B200 (config 5's workload; strong scaling).

The workload is the synthetic 9B-parameter DiT of config 5: 40 linear sets (8
double-stream blocks x {img, txt} + 24 single-stream blocks) of qkv
[12288,4096], proj [4096,4096], mlp_up [16384,4096] and mlp_down [4096,16384],
8.05e9 parameters, GPTQ INT4 rot256, block 128, damping 0.01, SmoothQuant
alpha 0.5 (which with rotation is SmoothRot on the FFN down layers: factors
from the per-channel activation amax, W * s and H / (s_i s_j) fused into the
rotations, the Hessian in the pipeline's own rotate-smooth-rotate order) and
PermuQuant tau 0.  One step quantizes the whole model: every layer through the
whole per-layer path (rotate W and H, row scales / zero-points, damping,
tensor-core inverse, GPTQ column loop with the tensor-core lazy update, INT4
packing, verify statistics), the layers handed out by a work queue across the
ranks (longest first), and every layer's packed codes, scales, zero-points and
statistics gathered to rank 0 over NVLink.  Inputs are seeded synthetic
tensors resident in HBM (a pool of distinct sets per rank, each ~1.7 GB, far
larger than L2, cycled over the model's 40 sets).

PermuQuant at INT4 uses per-row groups (pipeline.py:604): a column permutation
leaves every row's absmax, scale and codes unchanged, so its acceptance test
(relative improvement > tau = 0, permuquant.py:143-149) is false in exact
arithmetic and no permutation is applied; the reference decides it on the
summation-order noise of two fp32 sums.

Modes:
  python bench.py [--gpus N --steps K --warmup W]      B200 path (one process per GPU)
  python bench.py --impl reference ...                 the reference's own CPU code (baseline/_ref)
  python bench.py --hbm-kernels | --configs | --gemm-only N | --one-step
"""

from __future__ import annotations

import argparse
import ctypes
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
SMOOTH_ALPHA = 0.5
MODEL_SETS = 40  # 8 double-stream blocks x (img, txt) + 24 single-stream blocks
METRIC = "GPTQ-INT4 rot256 Mparams quantized/s"
CONFIG = {"workload": "config 5: synthetic 9B DiT, 40 linear sets of qkv[12288,4096] proj[4096,4096] "
                      "mlp_up[16384,4096] mlp_down[4096,16384] (8.05e9 params); GPTQ INT4 rot256, block 128, "
                      "damping 0.01; SmoothQuant alpha 0.5 -> SmoothRot on the 40 mlp_down layers; PermuQuant tau 0 "
                      "(INT4 per-row groups: never accepted in exact arithmetic, no permutation); one step = the "
                      "whole model, layers from a work queue over the ranks, outputs gathered to rank 0; "
                      "fp16 W ~ N(0,0.02^2), H = X^T X/8192 with X rows N(0, diag(s^2)), s ~ LogNormal(0,1)",
          "rot_size": ROT, "block_size": BLOCK, "damping": DAMP, "int_bits": 4, "smooth_alpha": SMOOTH_ALPHA,
          "l2": "inputs larger than L2 (each set ~1.7 GB, a pool of sets cycled over the model)"}


def make_set(seed: int, dev: torch.device):
    """One synthetic linear set on the device: (name, fp16 W ~ N(0, 0.02^2), H = X^T X / 8192,
    per-channel activation amax max_t |X[t, j]|) per layer."""
    g = torch.Generator(device=dev).manual_seed(seed)
    out = []
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    for li, (name, m, n) in enumerate(LAYERS):
        W = (torch.randn(m, n, generator=g, device=dev) * 0.02).half()
        s = torch.exp(torch.randn(n, generator=g, device=dev))  # LogNormal(0, 1) channel scales
        H = torch.zeros(n, n, device=dev)
        amax = torch.zeros(n, device=dev)
        for c0 in range(0, N_SAMPLES, 2048):  # X in chunks to bound the temporary
            X = torch.randn(min(2048, N_SAMPLES - c0), n, generator=g, device=dev) * s
            H.addmm_(X.T, X)
            amax = torch.maximum(amax, X.abs().amax(dim=0))
            del X
        H.div_(N_SAMPLES)
        H = 0.5 * (H + H.T)
        out.append((name, W, H, amax))
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
    """The unmodified reference package installed under baseline/_ref (pip --target);
    None when it is not installed."""
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


def reference_cpu_subprocess(steps: int, warmup: int, budget: float, sample: str = "set") -> dict | None:
    """Run the reference's CPU arm in a child process that sees no GPU; its JSON line or None."""
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    for k in ("RANK", "LOCAL_RANK", "WORLD_SIZE", "LOCAL_WORLD_SIZE"):
        env.pop(k, None)
    cmd = [sys.executable, os.path.abspath(__file__), "--impl", "reference-cpu", "--steps", str(steps),
           "--warmup", str(warmup), "--ref-budget", str(budget), "--ref-sample", sample]
    p = subprocess.run(cmd, env=env, stdout=subprocess.PIPE, text=True)
    lines = [ln for ln in p.stdout.splitlines() if ln.startswith("{")]
    if p.returncode != 0 or not lines:
        return None
    return json.loads(lines[-1])


def cpu_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def run_reference(args, rank: int, world: int) -> None:
    """The reference arm: its own CPU implementation timed in a child process
    that sees no GPU (the reference picks its Triton GPU loop whenever CUDA is
    visible, gptq.py:61-62, and has no switch for it), plus, as context, one set
    through its stock path on this box (Triton GPTQ loop on the GPU, rotations
    and inverse on the CPU).  Rank 0 only."""
    if rank != 0:
        return
    line = reference_cpu_subprocess(args.steps, args.warmup, args.ref_budget)
    if line is None:
        print(json.dumps({"impl": "reference", "unavailable": "the reference's CPU run failed"}), flush=True)
        return
    if "unavailable" not in line:
        line["n_gpus"] = world
        ref = _reference_converter()
        if ref is not None and torch.cuda.is_available():
            tot = 0.0
            for i, (name, m, n) in enumerate(LAYERS):
                tot += reference_layer_seconds(ref, *cpu_layer_inputs(name, m, n, 77 + i))
            line["stock_path_one_set"] = {
                "value": round(PARAMS_PER_SET / tot / 1e6, 4), "unit": "Mparams/s", "seconds": round(tot, 3),
                "note": "the reference's default code path on this box: Triton GPTQ loop on the GPU "
                        "(gptq.py:27-88), rotations and the Hessian inverse on the CPU"}
    print(json.dumps(line), flush=True)


def run_reference_cpu(args) -> None:
    """The reference's own CPU implementation on the B200 arm's config: one step =
    one DiT linear set (qkv, proj, mlp_up, mlp_down) through its per-layer calls,
    all host threads.  A set takes tens of seconds of CPU, so the timed steps stop
    at --ref-budget seconds (after at least one whole set); `steps` reports the
    sets actually timed.  Warm-up steps run the proj layer only.  Run with no GPU
    visible."""
    if torch.cuda.is_available():
        raise RuntimeError("the reference's CPU arm must run with no GPU visible (CUDA_VISIBLE_DEVICES=)")
    ref = _reference_converter()
    if ref is None:
        print(json.dumps({"impl": "reference", "unavailable": "reference not installed under baseline/_ref "
                                                               "(pip install --target baseline/_ref)"}), flush=True)
        return
    torch.set_num_threads(cpu_cores())
    inputs = {name: cpu_layer_inputs(name, m, n, 77 + i) for i, (name, m, n) in enumerate(LAYERS)
              if args.ref_sample == "set" or name == "proj"}
    for _ in range(args.warmup):
        reference_layer_seconds(ref, *inputs["proj"])
    layers = LAYERS if args.ref_sample == "set" else [LAYERS[1]]
    per_step_params = sum(m * n for _, m, n in layers)
    per_layer: dict[str, list[float]] = {name: [] for name, _, _ in layers}
    total, sets = 0.0, 0
    t_start = time.perf_counter()
    while sets < args.steps:
        for name, _, _ in layers:
            per_layer[name].append(reference_layer_seconds(ref, *inputs[name]))
        sets += 1
        if time.perf_counter() - t_start > args.ref_budget:
            break
    total = sum(sum(v) for v in per_layer.values())
    val = per_step_params * sets / total / 1e6
    what = "whole set(s) of 4 layers" if args.ref_sample == "set" else "proj layer(s) [4096,4096]"
    sample = (f"{sets} {what} through the reference's own converter.rotation.rotate_weights -> "
              f"rotate_hessian -> gptq.gptq_quantize_layer -> packing.pack_int4 on CPU tensors "
              f"(baseline/_ref, no GPU visible), torch threads {torch.get_num_threads()}")
    line = {
        "impl": "reference", "metric": METRIC, "value": round(val, 4), "unit": "Mparams/s", "n_gpus": 0,
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
    """The dominant kernel (3xTF32 tcgen05 GEMM) at the largest product a step
    runs: H^-1 = U U^T of the mlp_down inverse, U upper triangular [16384,16384],
    lower output tiles only (ic_gemm_tn_tri, tri = 3), exactly as the inverse
    issues it; timed with CUDA events on the launching stream.  Algorithmic flop
    n^3 / 3 (the triangular product).  Returns (TFLOP/s, ms per launch)."""
    from int_crush_converter_b200 import _native as nat
    lib = nat.load()
    g = torch.Generator(device=dev).manual_seed(7)
    hi = torch.randn(n, n, generator=g, device=dev).triu_()
    lo = (torch.randn(n, n, generator=g, device=dev) * 1e-4).triu_()
    out_hi = torch.empty_like(hi)
    out_lo = torch.empty_like(hi)
    st = nat.stream_ptr(dev)

    def go():
        nat.check(lib.ic_gemm_tn_tri(n, n, n, 1.0, hi.data_ptr(), lo.data_ptr(), n, hi.data_ptr(), lo.data_ptr(), n,
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
    return n ** 3 / 3.0 / (ms * 1e-3) / 1e12, ms


def cublas_tf32_tflops(dev: torch.device, n: int = 16384, reps: int = 3) -> float | None:
    """Context for the roofline: the TF32 rate cuBLAS itself reaches on this GPU
    (a square fp32 product with TF32 tensor cores allowed), CUDA events."""
    prev = torch.backends.cuda.matmul.allow_tf32
    try:
        torch.backends.cuda.matmul.allow_tf32 = True
        g = torch.Generator(device=dev).manual_seed(3)
        a = torch.randn(n, n, generator=g, device=dev)
        b = torch.randn(n, n, generator=g, device=dev)
        c = a @ b
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            torch.matmul(a, b, out=c)
        e1.record()
        torch.cuda.synchronize(dev)
        ms = e0.elapsed_time(e1) / reps
        del a, b, c
        return round(2.0 * n ** 3 / (ms * 1e-3) / 1e12, 1)
    except RuntimeError:
        return None
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


def model_layers(n_sets: int) -> list[tuple[int, str, int, int]]:
    """(set, layer name, out, in) of every linear layer of the model."""
    return [(si, name, m, n) for si in range(n_sets) for name, m, n in LAYERS]


def layer_order(layers, how: str) -> list[int]:
    from int_crush_converter_b200.sharding import layer_cost, longest_first
    if how == "natural":
        return list(range(len(layers)))
    return longest_first([layer_cost(m, n) for _, _, m, n in layers])


def output_specs(layers):
    def specs(i):
        m, n = layers[i][2], layers[i][3]
        return {"packed": ((m, n // 2), torch.uint8), "scales": ((m, 1), torch.float16),
                "zero_points": ((m, 1), torch.int8), "stats": ((3,), torch.float64)}
    return specs


def smoothrot_hook(amax: torch.Tensor):
    """SmoothRot pre-pass of an FFN down layer (pipeline.py:362-415): factors from
    the activation amax and the unrotated weight, on the device."""
    from int_crush_converter_b200.smoothquant import compute_smoothing_factors

    def before(Wd):
        a = amax if amax.is_cuda else amax.to(Wd.device, non_blocking=True)
        return {"smoothing": compute_smoothing_factors(a, Wd, alpha=SMOOTH_ALPHA), "smoothing_order": "pipeline"}
    return before


def run_model_steps(args, tag, steps, layers, order, fetch, pool, world, dev, on_gathered=None):
    """`steps` whole-model steps: work queue -> quantize -> gather to rank 0."""
    from int_crush_converter_b200.sharding import WorkQueue, gather_results, quantize_from_queue
    specs = output_specs(layers)
    for k in range(steps):
        res = quantize_from_queue(WorkQueue(order, f"{tag}{k}"), fetch, pool, depth=args.depth)
        pool.join()
        if world > 1:
            res = gather_results(res, len(layers), specs, dst=0, device=dev)
        if on_gathered is not None:
            on_gathered(res)


def run_device(args, rank: int, world: int) -> None:
    import int_crush_converter_b200 as B
    from int_crush_converter_b200 import _native as nat

    local = int(os.environ.get("LOCAL_RANK", 0))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    nat.require_device(dev)
    layers = model_layers(args.model_sets)
    order = layer_order(layers, args.order)
    n_params = sum(m * n for _, _, m, n in layers)
    n_flop = args.model_sets * FLOP_PER_SET
    n_pool = max(1, min(args.sets, args.model_sets))
    sets = [{name: (W, H, a) for name, W, H, a in make_set(1000 * rank + i, dev)} for i in range(n_pool)]
    pool = B.LayerStreams(args.streams, dev)

    def fetch(i):
        si, name, _, _ = layers[i]
        W, H, amax = sets[si % n_pool][name]
        kw = dict(rot_size=ROT, block_size=BLOCK, damping=DAMP)
        if name == "mlp_down":
            kw["before"] = smoothrot_hook(amax)
        return W, H, kw

    pool.fork()
    run_model_steps(args, "w", args.warmup, layers, order, fetch, pool, world, dev)
    pool.check()
    torch.cuda.synchronize(dev)
    if world > 1:
        torch.distributed.barrier()
    lib = nat.load()
    cvd = os.environ.get("CUDA_VISIBLE_DEVICES", "")
    phys = int(cvd.split(",")[local]) if cvd and cvd.split(",")[local].strip().isdigit() else local
    done_layers = [0]

    def count(res):
        done_layers[0] += len(res)
    with ClockSampler(phys) as clk:
        l0 = lib.ic_launch_count()
        g0 = lib.ic_inverse_graph_count()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize(dev)
        e0.record()
        pool.fork()
        run_model_steps(args, "t", args.steps, layers, order, fetch, pool, world, dev, on_gathered=count)
        e1.record()
        torch.cuda.synchronize(dev)
        launches = lib.ic_launch_count() - l0
        graphs = lib.ic_inverse_graph_count() - g0
    pool.check()
    if rank == 0 and done_layers[0] != args.steps * len(layers):
        raise RuntimeError(f"rank 0 holds {done_layers[0]} layer results, expected {args.steps * len(layers)}")
    if world > 1:
        torch.distributed.barrier()
    ms_max = max_over_ranks(e0.elapsed_time(e1), dev)
    value = n_params * args.steps / (ms_max * 1e-3) / 1e6
    launches = int(max_over_ranks(float(launches), dev)) if world > 1 else int(launches)
    passes3 = None
    if args.passes3_steps > 0:
        # the same model pass with the trailing update in 3xTF32 (update_passes=3)
        def fetch3(i):
            W, H, kw = fetch(i)
            return W, H, dict(kw, update_passes=3)
        pool.fork()
        run_model_steps(args, "p3w", 1, layers, order, fetch3, pool, world, dev)
        pool.check()
        torch.cuda.synchronize(dev)
        if world > 1:
            torch.distributed.barrier()
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record()
        pool.fork()
        run_model_steps(args, "p3t", args.passes3_steps, layers, order, fetch3, pool, world, dev)
        f1.record()
        torch.cuda.synchronize(dev)
        pool.check()
        ms3 = max_over_ranks(f0.elapsed_time(f1), dev)
        passes3 = {"value": round(n_params * args.passes3_steps / (ms3 * 1e-3) / 1e6, 3), "unit": "Mparams/s",
                   "steps": args.passes3_steps, "ms_per_step": round(ms3 / args.passes3_steps, 3),
                   "note": "GPTQ trailing update in 3xTF32 (update_passes=3) instead of one TF32 pass with fp32 "
                           "accumulation; everything else as the headline"}
    del sets
    torch.cuda.empty_cache()

    e2e = run_e2e(args, dev, pool, rank, world, layers, order)
    if rank != 0:
        return
    achieved, gemm_ms = dominant_gemm_tflops(dev)
    cublas_tf32 = cublas_tf32_tflops(dev)
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except (OSError, ValueError):
        pass
    bf16 = peaks.get("bf16_tflops", 1590.0)
    peak = bf16 / 2.0 / 3.0  # TF32 runs at half the bf16 rate; 3xTF32 issues three products
    bf16_s = peaks.get("bf16_tflops_sustained", 1400.0)
    peak_s = bf16_s / 2.0 / 3.0
    cpu = reference_cpu_subprocess(1, 0, 0.0, "proj")
    dropin = run_dropin(dev) if args.dropin else None
    other = None
    if args.other_configs:
        torch.cuda.empty_cache()
        cpu_cfg = {c["config"]: c for c in reference_configs_subprocess()}
        other = measure_configs(dev, _peaks().get("hbm_gbs"))
        for d in other:
            d["cpu_baseline"] = cpu_cfg.get(d["config"])
    ms_step = ms_max / args.steps
    line = {
        "metric": METRIC, "value": round(value, 3), "unit": "Mparams/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_step, 3), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None,
        "dtype": "f32 (3xTF32 inverse; TF32 products with fp32 accumulation for the GPTQ trailing update)",
        "data": "synthetic",
        "config": dict(CONFIG, parallelism=f"{world} GPU(s): layers from a work queue (longest first), outputs "
                                           f"gathered to rank 0 over NCCL", streams=args.streams,
                       model_sets=args.model_sets, params=n_params, order=args.order),
        "e2e": e2e,
        "dropin_e2e": dropin,
        "trailing_update_3xtf32": passes3,
        "other_configs": other,
        "gpu_launches": launches,
        "inverse_graphs_instantiated_in_timed_region": int(graphs),
        "roofline": {"bound": "tensor", "achieved": round(achieved, 2), "peak": round(peak, 2), "unit": "TFLOP/s",
                     "frac": round(achieved / peak, 4), "traffic": TRAFFIC_BYTES,
                     "kernel": "gemm_pair_kernel (3xTF32, tcgen05 cta_group::2 CTA pairs, K-slabs of 4096), "
                               "triangular U*U^T of the mlp_down inverse "
                               f"(16384^3/3 flop), {gemm_ms:.2f} ms/launch",
                     "context": {"cublas_tf32_tflops": cublas_tf32,
                                 "tf32_work_over_cublas_tf32": (round(3 * achieved / cublas_tf32, 3)
                                                                if cublas_tf32 else None),
                                 "note": "cuBLAS's own fp32 GEMM on TF32 tensor cores (torch.matmul, "
                                         "allow_tf32) at 16384^3 on this GPU, timed the same way; the kernel "
                                         "does three TF32 products per output term"},
                     "peak_basis": ("measured bf16 burst / 2 (TF32 rate) / 3 (3xTF32 products), of measured"
                                    if "bf16_tflops" in peaks else "fallback 1.59 PF bf16 / 2 / 3, of fallback")},
        "step_roofline": {"bound": "tensor", "flop_per_step": n_flop,
                          "target_ms": round(n_flop / (world * peak_s * 1e12) * 1e3, 3),
                          "ms_per_step": round(ms_step, 3),
                          "frac": round(n_flop / (world * peak_s * 1e12) * 1e3 / ms_step, 4),
                          "note": "whole step's algorithmic flop over N x the sustained 3xTF32 peak "
                                  "(bf16_tflops_sustained / 2 / 3), of measured"},
        "cpu_baseline": (cpu["cpu_baseline"] if cpu else {"value": None, "unavailable": "reference not installed"}),
        "clocks": clk.summary(),
    }
    print(json.dumps(line), flush=True)


# DRAM bytes (read + write) of the 16384^3 3xTF32 product timed by dominant_gemm_tflops, from
# the ncu captures summarised in profiles/ (null until captured for the triangular product)
TRAFFIC_BYTES = None


def run_dropin(dev: torch.device, reps: int = 2) -> dict:
    """The same metric through the reference pipeline's own per-layer call
    shape with this package installed in its place (pipeline_hook): per layer
    rotate_weights(W) -> rotate_hessian(H) -> gptq_quantize_layer(W_rot, H_rot)
    -> pack_int4(q), every call on host tensors as the pipeline passes them (W
    upcast to fp32 on the host, pipeline.py:524), each call copying in and
    out.  One config-3 set per rep, rank 0 only."""
    import int_crush_converter_b200 as B
    host = [(name, W.float().cpu(), H.cpu()) for name, W, H, _ in make_set(77, dev)]
    torch.cuda.empty_cache()

    def one_set():
        for _, W, H in host:
            Wr = B.rotate_weights(W, ROT)
            Hr = B.rotate_hessian(H, ROT)
            r = B.gptq_quantize_layer(Wr, Hr, block_size=BLOCK, damping=DAMP, int_bits=4)
            B.pack_int4(r.quantized_W)
    one_set()
    torch.cuda.synchronize(dev)
    t0 = time.perf_counter()
    for _ in range(reps):
        one_set()
    torch.cuda.synchronize(dev)
    dt = (time.perf_counter() - t0) / reps
    return {"value": round(PARAMS_PER_SET / dt / 1e6, 3), "unit": "Mparams/s", "seconds_per_set": round(dt, 3),
            "sets": reps, "api": "reference call shape: rotate_weights -> rotate_hessian -> gptq_quantize_layer "
                                 "-> pack_int4 on CPU tensors (pipeline.py:547-559, 702-789, 1010-1013), "
                                 "one layer at a time, host wall clock"}


def run_e2e(args, dev: torch.device, pool, rank: int, world: int, layers, order) -> dict:
    """The same metric through the public API with HOST buffers: every step copies
    each layer's fp16 weight, fp32 Hessian and activation amax from pinned host
    memory (LayerStreams' copy streams), quantizes, gathers the outputs to rank 0
    and copies every layer's packed codes, scales, zero-points and statistics to
    pinned host memory on rank 0; all inside the timed region."""
    n_host = max(1, min(args.host_sets, args.model_sets))
    host = []
    for i in range(n_host):
        hs = {}
        for name, W, H, a in make_set(5000 + 100 * rank + i, dev):
            hs[name] = (W.cpu().pin_memory(), H.cpu().pin_memory(), a.cpu().pin_memory())
        host.append(hs)
    torch.cuda.empty_cache()
    specs = output_specs(layers)
    outs = {}
    if rank == 0:
        for i in range(len(layers)):
            outs[i] = {k: torch.empty(shape, dtype=dt).pin_memory() for k, (shape, dt) in specs(i).items()}
    h2d = sum(m * n * 2 + n * n * 4 + n * 4 for _, _, m, n in layers)
    d2h = sum(sum(t.numel() * t.element_size() for t in o.values()) for o in outs.values())
    steps = max(1, min(args.steps, args.e2e_steps))

    def fetch(i):
        si, name, _, _ = layers[i]
        W, H, amax = host[si % n_host][name]
        kw = dict(rot_size=ROT, block_size=BLOCK, damping=DAMP)
        if name == "mlp_down":
            kw["before"] = smoothrot_hook(amax)
        if world == 1:
            def then(o, i=i):
                for k, t in outs[i].items():
                    t.copy_(o[k], non_blocking=True)
            kw["then"] = then
        return W, H, kw

    def to_host(res):
        if world > 1 and rank == 0:
            for i, o in res.items():
                for k, t in outs[i].items():
                    t.copy_(o[k], non_blocking=True)

    pool.fork()
    run_model_steps(args, "ew", 1, layers, order, fetch, pool, world, dev, on_gathered=to_host)
    pool.check()
    torch.cuda.synchronize(dev)
    if world > 1:
        torch.distributed.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    pool.fork()
    run_model_steps(args, "et", steps, layers, order, fetch, pool, world, dev, on_gathered=to_host)
    pool.join()
    e1.record()
    torch.cuda.synchronize(dev)
    pool.check()
    n_params = sum(m * n for _, _, m, n in layers)
    val = n_params * steps / (max_over_ranks(e0.elapsed_time(e1), dev) * 1e-3) / 1e6
    return {"value": round(val, 3), "unit": "Mparams/s", "h2d_bytes_per_step": int(h2d),
            "d2h_bytes_per_step": int(d2h), "steps": steps, "host_sets": n_host,
            "api": "int_crush_converter_b200.sharding.WorkQueue + LayerStreams.submit -> quantize_gptq_layer "
                   "(C ABI ic_gptq_layer) with pinned host inputs; gather_results to rank 0; D2H of every "
                   "layer's outputs on rank 0"}


def run_hbm_kernels(reps: int = 5) -> None:
    """HBM-bound kernels of the path at the BASELINE configs' shapes, each timed
    alone with CUDA events and reported against the measured copy bandwidth.
    Algorithmic bytes (the minimum a kernel must move):
      rtn_fused (config 1: fp16 W [4096,4096] x 8 layers, INT4 sym rot256):
          2 B read + 0.5 B packed written per weight (+ 2 B scale per row)
      rtn_fused (config 2: fp16 W, 16 x [3072,3072] + 16 x [12288,3072], INT8 sym rot64, 5 ratios):
          2 B read + 1 B codes written per weight (+ 2 B scale per row)
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
    out.append(dict(kernel="rtn_pair_kernel<half,256> (ic_rtn_fused)", workload="config 1: 8 x fp16 [4096,4096] INT4 sym rot256",
                    ms_per_call=ms, achieved_gbs=gbs, frac=frac))
    del Ws
    # config 2: RTN INT8 sym rot64 with the 5-ratio clip search, 16 x [3072,3072] + 16 x [12288,3072]
    ratios = (ctypes.c_float * 5)(0.8, 0.85, 0.9, 0.95, 1.0)
    W2 = [(torch.randn(m, 3072, generator=g, device=dev) * 0.02).half() for m in [3072] * 16 + [12288] * 16]
    c2 = torch.empty(12288, 3072, dtype=torch.int8, device=dev)
    sc2 = torch.empty(12288, dtype=torch.float16, device=dev)
    sq2 = torch.empty(12288, dtype=torch.float64, device=dev)
    mx2 = torch.empty(12288, dtype=torch.float32, device=dev)
    p2 = sum(W.shape[0] * 3072 for W in W2)

    def rtn8():
        for W in W2:
            m = W.shape[0]
            nat.check(lib.ic_rtn_fused(W.data_ptr(), nat.IC_F16, m, 3072, 3072, 64, 8, 0, ratios, 5, c2.data_ptr(),
                                       None, sc2.data_ptr(), None, sq2.data_ptr(), mx2.data_ptr(), st))
    ms, gbs, frac = timed(rtn8, p2 * 3 + sum(W.shape[0] for W in W2) * 2)
    out.append(dict(kernel="rtn_pair_kernel<half,64> (ic_rtn_fused)",
                    workload="config 2: 16 x [3072,3072] + 16 x [12288,3072] fp16, INT8 sym rot64, 5 clipping ratios",
                    ms_per_call=ms, achieved_gbs=gbs, frac=frac))
    del W2, c2
    W = (torch.randn(4096, 16384, generator=g, device=dev) * 0.02).half()
    Wr = torch.empty(4096, 16384, device=dev)

    def rot():
        nat.check(lib.ic_rotate_weights(W.data_ptr(), nat.IC_F16, 4096, 16384, 16384, 256, Wr.data_ptr(), 16384, st))
    ms, gbs, frac = timed(rot, 4096 * 16384 * 6)
    out.append(dict(kernel="rotate_pair256_kernel (ic_rotate_weights)", workload="fp16 [4096,16384] -> fp32, rot256",
                    ms_per_call=ms, achieved_gbs=gbs, frac=frac))
    del W, Wr
    n = 16384
    H = torch.randn(n, n, generator=g, device=dev)
    hh = torch.empty(n, n, device=dev)
    hl = torch.empty(n, n, device=dev)

    def roth():
        nat.check(lib.ic_rotate_hessian(H.data_ptr(), 1, n, n, 256, hh.data_ptr(), hl.data_ptr(), n, st))
    ms, gbs, frac = timed(roth, n * n * 12)
    out.append(dict(kernel="rotate_pair256_kernel + hess_cols256_kernel (ic_rotate_hessian)",
                    workload="fp32 H [16384,16384] -> hi/lo pair, rot256", ms_per_call=ms, achieved_gbs=gbs,
                    frac=frac))
    for o in out:
        o.update(unit="GB/s", peak_gbs=peak, peak_basis=basis, bound="hbm")
        print(json.dumps(o), flush=True)


def measure_configs(dev: torch.device, peak_gbs: float | None = None, e2e: bool = True) -> list[dict]:
    """The BASELINE configs other than the headline one, each through the public
    API on synthetic inputs of the config's shapes (seeded), timed with CUDA
    events after a warm-up: device-resident `value`; for the RTN configs the
    HBM roofline (algorithmic bytes: fp16 in, codes out, fp16 scales) and an
    `e2e` with the fp16 weights copied from pinned host memory and the codes
    and scales copied back inside the timed region."""
    import int_crush_converter_b200 as B
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

    def rtn_e2e(Ws, rot, bits, ratios, reps=2):
        host = [W.cpu().pin_memory() for W in Ws]
        outs = []
        for W in Ws:
            m, n = W.shape
            outs.append((torch.empty(m, n // 2 if bits == 4 else n, dtype=torch.uint8 if bits == 4 else torch.int8)
                         .pin_memory(), torch.empty(m, 1, dtype=torch.float16).pin_memory()))

        def go():
            for Wh, (c, sc) in zip(host, outs):
                o = B.rtn_quantize_fused(Wh.to(dev, non_blocking=True), rot, int_bits=bits, clipping_ratios=ratios,
                                         want_codes=bits == 8, want_packed=bits == 4)
                c.copy_(o["packed"] if bits == 4 else o["codes"], non_blocking=True)
                sc.copy_(o["scales"], non_blocking=True)
        ms = timed(go, reps)
        h2d = sum(W.numel() * 2 for W in Ws)
        d2h = sum(c.numel() + sc.numel() * 2 for c, sc in outs)
        return ms, h2d, d2h

    lines = []
    # config 1: RTN INT4 sym rot256, 8 x [4096,4096]
    W1 = [weights(4096, 4096, 0.02, 0.001, 20.0) for _ in range(8)]
    p1 = 8 * 4096 * 4096
    ms = timed(lambda: [B.rtn_quantize_fused(W, 256, int_bits=4, want_codes=False) for W in W1], 5)
    d = dict(config=1, workload="RTN INT4 sym rot256, 8 fp16 layers [4096,4096] (0.1% columns x20)", params=p1,
             ms=ms, algorithmic_bytes=p1 * 2.5 + 8 * 4096 * 2)
    if e2e:
        ems, h2d, d2h = rtn_e2e(W1, 256, 4, None)
        d["e2e"] = {"value": round(p1 / (ems * 1e-3) / 1e6, 2), "unit": "Mparams/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h}
    lines.append(d)
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
    p2 = 16 * 3072 * 3072 + 16 * 12288 * 3072
    ms = timed(lambda: [B.rtn_quantize_fused(W, 64, int_bits=8, clipping_ratios=ratios, want_codes=True,
                                             want_packed=False) for W in W2], 3)
    d = dict(config=2, workload="RTN INT8 sym rot64, clipping ratios {0.8..1.0}, 16 x [3072,3072] + "
                                "16 x [12288,3072] fp16 (N(0,0.02^2) + Student-t(3) tails on 1%)",
             params=p2, ms=ms, algorithmic_bytes=p2 * 3 + (16 * 3072 + 16 * 12288) * 2)
    if e2e:
        ems, h2d, d2h = rtn_e2e(W2, 64, 8, ratios)
        d["e2e"] = {"value": round(p2 / (ems * 1e-3) / 1e6, 2), "unit": "Mparams/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h}
    lines.append(d)
    del W2
    # config 4: LDLQ INT4 rot256, 2 iterations, 8 greedy passes, weight-only Hessian; one [8192,8192] layer
    W4 = weights(8192, 8192, 0.015, 0.0005, 30.0)

    def ldlq():
        Wr = B.rotate_weights(W4.float(), 256)
        return B.ldlq_quantize_layer(Wr, None, block_size=128, int_bits=4, iterations=2, greedy_passes=8)
    import warnings
    with warnings.catch_warnings():
        warnings.simplefilter("ignore")
        ms = timed(ldlq, 1)
        os.environ["IC_GREEDY_GEMM_PASSES"] = "1"
        try:
            ms1 = timed(ldlq, 1)
        finally:
            del os.environ["IC_GREEDY_GEMM_PASSES"]
    w4 = ("LDLQ INT4 rot256, 2 iterations, 8 greedy passes, weight-only Hessian, "
          "one fp16 layer [8192,8192] (N(0,0.015^2), 0.05% columns x30)")
    lines.append(dict(config=4, workload=w4, params=8192 * 8192, ms=ms))
    lines.append(dict(config=4, workload=w4 + "; opt-in one-pass TF32 greedy cross terms (IC_GREEDY_GEMM_PASSES=1)",
                      params=8192 * 8192, ms=ms1))
    for d in lines:
        d.update(metric="Mparams quantized/s", value=round(d["params"] / (d["ms"] * 1e-3) / 1e6, 2),
                 ms=round(d["ms"], 3), data="synthetic, device-resident")
        if "algorithmic_bytes" in d and peak_gbs:
            gbs = d["algorithmic_bytes"] / (d["ms"] * 1e-3) / 1e9
            d["roofline"] = {"bound": "hbm", "achieved": round(gbs, 1), "peak": peak_gbs, "unit": "GB/s",
                             "frac": round(gbs / peak_gbs, 4), "traffic": None,
                             "kernel": "rtn_pair_kernel (ic_rtn_fused), all layers of the config"}
    return lines


def reference_cpu_configs() -> list[dict]:
    """The reference's own CPU code on bounded samples of configs 1, 2 and 4
    (run with no GPU visible): one layer of each RTN config, and LDLQ with the
    config's settings on a [1024, 1024] layer (the full [8192, 8192] greedy
    search takes hours on the CPU)."""
    import numpy as np
    ref = _reference_converter()
    if ref is None:
        return []
    import importlib
    scales = importlib.import_module("converter.scales")
    ldlq = importlib.import_module("converter.ldlq")
    torch.set_num_threads(cpu_cores())
    g = torch.Generator().manual_seed(3)
    out = []

    def run(fn, reps=2):
        fn()
        t0 = time.perf_counter()
        for _ in range(reps):
            fn()
        return (time.perf_counter() - t0) / reps

    W = (torch.randn(4096, 4096, generator=g) * 0.02).half().float()

    def c1():
        Wr = ref["rotation"].rotate_weights(W, 256)
        s = scales.calculate_scales(Wr, Wr.shape[1])
        ref["packing"].pack_int4(scales.quantize_weights(Wr, s, Wr.shape[1]))
    sec = run(c1)
    out.append(dict(config=1, value=round(4096 * 4096 / sec / 1e6, 3), unit="Mparams/s", cores=torch.get_num_threads(),
                    kind="reference", sample="one [4096,4096] layer: rotate_weights -> calculate_scales -> "
                                             "quantize_weights -> pack_int4"))
    W = (torch.randn(3072, 3072, generator=g) * 0.02).half().float()
    ratios = [0.8, 0.85, 0.9, 0.95, 1.0]

    def c2():
        Wr = ref["rotation"].rotate_weights(W, 64)
        s = scales.calculate_scales_int8(Wr, clipping_ratios=ratios)
        scales.quantize_weights_int8(Wr, s)
    sec = run(c2)
    out.append(dict(config=2, value=round(3072 * 3072 / sec / 1e6, 3), unit="Mparams/s", cores=torch.get_num_threads(),
                    kind="reference", sample="one [3072,3072] layer: rotate_weights(64) -> calculate_scales_int8 "
                                             "(5 ratios) -> quantize_weights_int8"))
    W = (torch.randn(1024, 1024, generator=g) * 0.015).half().float()
    import warnings

    def c4():
        Wr = ref["rotation"].rotate_weights(W, 256)
        with warnings.catch_warnings():
            warnings.simplefilter("ignore")
            ldlq.ldlq_quantize_layer(Wr, None, block_size=128, int_bits=4, iterations=2, greedy_passes=8)
    sec = run(c4, 1)
    out.append(dict(config=4, value=round(1024 * 1024 / sec / 1e6, 3), unit="Mparams/s", cores=torch.get_num_threads(),
                    kind="reference", sample="one [1024,1024] layer (the config's [8192,8192] takes hours): "
                                             "LDLQ INT4 rot256, 2 iterations, 8 greedy passes"))
    del np
    return out


def run_configs(with_reference: bool = True) -> None:
    """Configs 1, 2 and 4 (one JSON line each), with the reference's CPU samples
    unless ``with_reference`` is off (device-only runs, e.g. under a profiler)."""
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    peak = _peaks().get("hbm_gbs")
    cpu = {c["config"]: c for c in reference_configs_subprocess()} if with_reference else {}
    for d in measure_configs(dev, peak):
        d["cpu_baseline"] = cpu.get(d["config"])
        print(json.dumps(d), flush=True)


def _peaks() -> dict:
    try:
        return json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except (OSError, ValueError):
        return {}


def reference_configs_subprocess() -> list[dict]:
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    for k in ("RANK", "LOCAL_RANK", "WORLD_SIZE", "LOCAL_WORLD_SIZE"):
        env.pop(k, None)
    p = subprocess.run([sys.executable, os.path.abspath(__file__), "--impl", "reference-cpu-configs"], env=env,
                       stdout=subprocess.PIPE, text=True)
    lines = [ln for ln in p.stdout.splitlines() if ln.startswith("[")]
    return json.loads(lines[-1]) if p.returncode == 0 and lines else []


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=8)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference", "reference-cpu", "reference-cpu-configs"])
    ap.add_argument("--sets", type=int, default=8, help="distinct resident input sets per GPU (cycled)")
    ap.add_argument("--host-sets", type=int, default=2, help="distinct pinned host input sets per GPU (e2e)")
    ap.add_argument("--model-sets", type=int, default=MODEL_SETS, help="linear sets in the model (config 5: 40)")
    ap.add_argument("--order", default="lpt", choices=["lpt", "natural"], help="work-queue order of the layers")
    ap.add_argument("--depth", type=int, default=6, help="layers a rank keeps unfinished on its GPU")
    ap.add_argument("--passes3-steps", type=int, default=2,
                    help="also time this many model passes with the 3xTF32 trailing update")
    ap.add_argument("--dropin", type=int, default=1, help="also time the reference call shape (drop-in API)")
    ap.add_argument("--other-configs", type=int, default=1,
                    help="also measure configs 1, 2 and 4 (rank 0) with the reference's CPU samples")
    ap.add_argument("--e2e-steps", type=int, default=3)
    ap.add_argument("--ref-sample", default="set", choices=["set", "proj"],
                    help="reference CPU arm: time whole sets or the proj layer only")
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
    ap.add_argument("--no-ref", action="store_true",
                    help="with --configs: skip the reference's CPU samples (device work only)")
    ap.add_argument("--profile-side", action="store_true",
                    help="run small cases of the side-path kernels twice and exit (kernel captures)")
    ap.add_argument("--profile-layer", default="",
                    help="M,N: quantize one synthetic GPTQ layer [M,N] twice (one warm-up) and exit -- a small "
                         "case for kernel captures")
    args = ap.parse_args()
    if args.configs:
        run_configs(with_reference=not args.no_ref)
        return
    if args.profile_side:
        # small cases of the side-path kernels, for kernel captures: PiSO (4096 x
        # 4096, INT4 asymmetric), greedy search (1024 x 1024, one pass), SmoothQuant
        # factors, PermuQuant order and errors (4096 x 16384), SVD split (4096 x 4096, rank 32)
        import warnings
        import int_crush_converter_b200 as B
        dev = torch.device("cuda", 0)
        torch.cuda.set_device(dev)
        g = torch.Generator(device=dev).manual_seed(9)
        W = torch.randn(4096, 4096, generator=g, device=dev) * 0.02
        hd = torch.rand(4096, generator=g, device=dev) + 0.1
        Wg = torch.randn(1024, 1024, generator=g, device=dev) * 0.02
        Wd = torch.randn(4096, 16384, generator=g, device=dev).half() * 0.02
        amax = torch.rand(16384, generator=g, device=dev) * 5
        for _ in range(2):
            B.compute_piso_scales_int4_asymmetric(W, hd)
            with warnings.catch_warnings():
                warnings.simplefilter("ignore")
                B.ldlq_quantize_layer(Wg, None, block_size=128, int_bits=4, iterations=1, greedy_passes=1)
            B.compute_smoothing_factors(amax, Wd)
            B.find_permutation_with_acceptance(Wd, None, 0.5, 128, 0.0, 4)
            B.decompose_weight(W, rank=32)
        torch.cuda.synchronize(dev)
        print(json.dumps({"profile_side": "ok"}))
        return
    if args.profile_layer:
        import int_crush_converter_b200 as B
        m, n = (int(x) for x in args.profile_layer.split(","))
        dev = torch.device("cuda", 0)
        torch.cuda.set_device(dev)
        g = torch.Generator(device=dev).manual_seed(5)
        W = (torch.randn(m, n, generator=g, device=dev) * 0.02).half()
        X = torch.randn(N_SAMPLES, n, generator=g, device=dev) * torch.exp(torch.randn(n, generator=g, device=dev))
        H = X.T @ X / N_SAMPLES
        del X
        for _ in range(2):
            B.quantize_gptq_layer(W, H, rot_size=ROT, block_size=BLOCK, damping=DAMP)
        torch.cuda.synchronize(dev)
        print(json.dumps({"profile_layer": [m, n], "ok": True}))
        return
    if args.one_step:
        import int_crush_converter_b200 as B
        dev = torch.device("cuda", 0)
        torch.cuda.set_device(dev)
        s = make_set(0, dev)
        torch.cuda.synchronize(dev)
        with B.LayerStreams(args.streams, dev) as pool:
            for _, W, H, _ in s:
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
    if args.impl == "reference-cpu":
        run_reference_cpu(args)
        return
    if args.impl == "reference-cpu-configs":
        print(json.dumps(reference_cpu_configs()), flush=True)
        return
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
