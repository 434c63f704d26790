#!/usr/bin/env python3
"""Benchmark of the B200 dense-layer path (the driver's bench contract).

Workload (the metric's multi-GPU config): the f32
dense layer Y = relu(X @ W + b) with X[65536, 4096], W[4096, 4096], b[4096];
rows of X/Y are split evenly across the N ranks (strong scaling), W and b
are replicated, no collective on the data path. One step = one pass of the
hot path over the rank's rows: tf32 hi/lo split of W and of the X rows, then
the fused tcgen05 GEMM + bias + ReLU kernel.

  value     TFLOP/s over all ranks (2*M*N*K per step), device-resident
            inputs, CUDA events on the launching stream, max over ranks.
  e2e       the same metric through the reference-facing plugin ABI
            (b200_memref_dense_relu_f32, the flattened-memref signature of
            ml-edsl's JIT'd functions) with pinned host buffers: every step
            copies X-rows, W and b to the device and Y back inside the call.
  roofline  the GEMM kernel alone (launched on pre-split operands) against
            the 3xTF32-effective tensor peak = measured bf16 burst / 6.
  e2e_pageable  the same call with plain (pageable) NumPy arrays, the path the
            reference's own callers take.
  check     the timed output itself: 256 sampled rows per rank (first, last,
            shard edges, random) against float64 NumPy, with the path's f32
            tolerance 1e-4*sqrt(K)*max|X|*max|W|.
  cpu_baseline  (rank 0, N=1) the CPU oracle, a restatement of the reference's
            CPU pipeline, on a bounded row sample of the same inputs; its
            output is compared with the GPU's rows (gpu_vs_oracle).
  headline_8192 (N=1) the 8192^3 dense layer with bias, device-resident.
  configs   (N=1) the other BASELINE.json configurations (256^3, 1024^3 dense,
            ragged 1000x999x1001, 4096^3, the 2-layer MLP, i32 2048^3), each
            call timed alone after an L2 flush, sampled rows checked.

Inputs are the seeded arrays of mlir_edsl.workloads (np.random.default_rng,
the generator the parity tests use); each rank draws only its own rows.

`--impl reference` times the reference's CPU pipeline restatement (oracle/)
on all host cores on bounded row samples of the same workload; under
torchrun only rank 0 runs it.

Run: python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
"""
import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "ml-edsl_b200"))
sys.path.insert(0, ROOT)

M_TOTAL, N_DIM, K_DIM = 65536, 4096, 4096
METRIC = "TFLOP/s, f32 matmul+bias+ReLU at 8192^3 & M=65536 (1/2/4/8 B200), % roofline"
UNIT = "TFLOP/s"
FALLBACK_BF16_TFLOPS = 1590.0


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-headline", action="store_true")
    ap.add_argument("--no-gather", action="store_true",
                    help="N>1: skip the all-gathered (single-device result) measurement")
    ap.add_argument("--gather-slabs", type=int, default=4)
    ap.add_argument("--gather-reserve-sms", type=int, default=8,
                    help="SMs the GEMM leaves free for NCCL while gathering")
    ap.add_argument("--configs", action="store_true",
                    help="time the standalone HBM-bound ops (bias+relu, reductions), one JSON "
                         "line each")
    ap.add_argument("--rows", type=int, default=0,
                    help="rows per GPU override (small cases for profiling); 0 = 65536/N")
    return ap.parse_args()


def dist_env():
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("LOCAL_RANK", 0)),
            int(os.environ.get("WORLD_SIZE", 1)))


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return float(p["bf16_tflops"]), "measured"
    except Exception:
        return FALLBACK_BF16_TFLOPS, "fallback"


def host_cores():
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


# ----------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi sampling of SM clocks / throttle reasons during a region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,utilization.gpu,"
              "clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.tmp = None

    def start(self):
        try:
            self.tmp = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=self.tmp, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.tmp.flush()
        with open(self.tmp.name) as f:
            rows = [r.split(",") for r in f.read().strip().splitlines() if r.strip()]
        os.unlink(self.tmp.name)
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        sm, mx, reasons, loaded = [], None, set(), 0
        for r in rows:
            r = [x.strip() for x in r]
            if len(r) < 10:
                continue
            try:
                clk, cmax, util = float(r[1]), float(r[2]), float(r[4])
            except ValueError:
                continue
            mx = cmax
            if util < 20:
                continue
            loaded += 1
            sm.append(clk)
            for name, val in zip(names, r[6:10]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples_under_load": loaded}


# ----------------------------------------------------------------- seeded inputs
WORKLOAD = "dense_65536"  # mlir_edsl.workloads: np.random.default_rng(3), U[-0.5, 0.5]


def workload_rows(r0, r1):
    from mlir_edsl import workloads
    return workloads.config_rows(WORKLOAD, "X", r0, r1)


def workload_weights():
    from mlir_edsl import workloads
    return workloads.config_array(WORKLOAD, "W"), workloads.config_array(WORKLOAD, "b")


def f32_bound(K, X, W):
    """The path's f32 tolerance: 1e-4 * sqrt(K) * max|X| * max|W|."""
    import numpy as np
    return 1e-4 * K ** 0.5 * float(np.max(np.abs(X))) * float(np.max(np.abs(W)))


def sample_rows(M, n=256, shards=8, seed=0):
    """First and last row, both sides of every `shards`-way edge, random rest."""
    import numpy as np
    edges = {0, M - 1}
    for k in range(1, shards):
        if 0 < k * (M // shards) < M:
            edges.update((k * (M // shards) - 1, k * (M // shards)))
    edges = sorted(e for e in edges if 0 <= e < M)
    rest = np.setdiff1d(np.arange(M), edges)
    extra = np.random.default_rng(seed).choice(rest, max(0, min(n - len(edges), rest.size)),
                                               replace=False)
    return np.sort(np.concatenate([np.array(edges, dtype=np.int64), extra]))


def check_rows(Xh, Wh, bh, Yrows, rows, act=1):
    """max |Y - act(X @ W + b)| over the sampled rows, against float64 NumPy."""
    import numpy as np
    ref = Xh[rows].astype(np.float64) @ Wh.astype(np.float64)
    if bh is not None:
        ref += bh
    if act == 1:
        ref = np.maximum(ref, 0.0)
    return float(np.max(np.abs(Yrows.astype(np.float64) - ref))) if len(rows) else 0.0


# ----------------------------------------------------------------- CPU oracle timing
def time_oracle_rows(X, W, b, threads, act=1):
    """Times the CPU restatement of the reference pipeline on the rows of X;
    returns (seconds, flops, Y)."""
    import oracle
    t0 = time.perf_counter()
    Y = oracle.dense_f32(X, W, b, act=act, threads=threads)
    dt = time.perf_counter() - t0
    return dt, 2.0 * X.shape[0] * N_DIM * K_DIM, Y


def calibrate_rows(target_s, threads, X, W, b, cap=None):
    """Row count (at most `cap`, default X's rows; a multiple of 64) whose
    oracle run takes about target_s seconds, timed on X's first 64 rows."""
    probe = 64
    dt, _, _ = time_oracle_rows(X[:probe], W, b, threads)
    rows = int(probe * target_s / max(dt, 1e-3))
    return max(64, min(cap or X.shape[0], rows // 64 * 64))


def run_reference(args):
    rank, _, world = dist_env()
    if rank != 0:
        return 0
    import oracle
    oracle.build()
    cores = host_cores()
    per_step = max(1.0, min(8.0, 150.0 / max(1, args.steps + args.warmup)))
    W, b = workload_weights()
    X = workload_rows(0, 64)
    rows = calibrate_rows(per_step, cores, X, W, b, cap=M_TOTAL)
    X = workload_rows(0, rows)
    for _ in range(args.warmup):
        time_oracle_rows(X, W, b, cores)
    times = []
    for _ in range(args.steps):
        dt, flops, _ = time_oracle_rows(X, W, b, cores)
        times.append(dt)
    total = sum(times)
    value = 2.0 * rows * N_DIM * K_DIM * args.steps / total / 1e12
    sample = (f"X[{rows},{K_DIM}] rows of the {M_TOTAL}-row workload @ W[{K_DIM},{N_DIM}] + b, "
              f"relu; restatement of the reference CPU pipeline (64x64 tiles, k-ascending "
              f"f32 fma), {cores} threads")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": total / args.steps * 1e3, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (np.random.default_rng(3), uniform[-0.5,0.5])",
        "config": {"workload": "dense_relu X[65536,4096] @ W[4096,4096] + b (row sample)",
                   "M_total": M_TOTAL, "N": N_DIM, "K": K_DIM, "rows_per_step": rows,
                   "parallelism": "host threads"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    emit_line(line)
    return 0


# ----------------------------------------------------------------- B200 arm
class L2Flush:
    """Writes a buffer larger than the 126 MB L2 between timed iterations."""

    def __init__(self, torch, dev, nbytes=256 << 20):
        self.buf = torch.empty(nbytes // 4, dtype=torch.float32, device=dev)

    def __call__(self):
        self.buf.fill_(1.0)


def time_calls(torch, stream, fn, iters, warmup, flush):
    """Median device time (ms) of fn() over `iters` calls, each bracketed by
    CUDA events on `stream`, with the L2 flushed before every call."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(iters)]
    for e0, e1 in evs:
        flush()
        e0.record(stream)
        fn()
        e1.record(stream)
    torch.cuda.synchronize()
    return statistics.median(e0.elapsed_time(e1) for e0, e1 in evs)


def small_configs(torch, L, _native, dev, stream, peak, args):
    """Device time of the other BASELINE.json configurations at N=1 (the
    reference's own benchmark sizes), each call timed alone after an L2
    flush, with sampled rows checked against float64 NumPy."""
    import numpy as np
    from mlir_edsl import workloads
    sp = ctypes.c_void_p(stream.cuda_stream)
    P = lambda t: ctypes.c_void_p(t.data_ptr()) if t is not None else None
    flush = L2Flush(torch, dev)
    iters = max(20, args.steps)
    out = []

    def dense(X, W, b, Y, act):
        M, K = X.shape
        N = W.shape[1]
        _native.check(L.b200_dense_f32(P(X), K, P(W), N, P(b), P(Y), N, M, N, K, act, 0.0, sp))

    for name, act in [("matmul_256", 0), ("dense_1024", 1), ("dense_ragged", 1),
                      ("matmul_4096", 0)]:
        g = workloads.config_inputs(name)
        Xh, Wh = (g["X"], g["W"]) if "X" in g else (g["A"], g["B"])
        bh = g.get("b")
        X, W = torch.from_numpy(Xh).to(dev), torch.from_numpy(Wh).to(dev)
        b = torch.from_numpy(bh).to(dev) if bh is not None else None
        M, K = Xh.shape
        N = Wh.shape[1]
        Y = torch.empty((M, N), device=dev)
        ms = time_calls(torch, stream, lambda: dense(X, W, b, Y, act), iters, 3, flush)
        _native.check(L.b200_stream_sync(sp))
        rows = sample_rows(M, 64)
        err = check_rows(Xh, Wh, bh, Y.cpu().numpy()[rows], rows, act)
        bound = f32_bound(K, Xh, Wh)
        fl = 2.0 * M * N * K
        out.append({"config": name, "ms": ms, "TFLOP/s": fl / ms / 1e9,
                    "frac_of_3xtf32_peak": fl / ms / 1e9 / peak,
                    "launches": _native.dense_launches(M, N, K),
                    "max_abs_err_vs_f64": err, "bound": bound, "ok": err <= bound})
        del X, W, b, Y
    # 2-layer MLP relu(relu(X@W1+b1)@W2+b2); the hidden activation stays in HBM
    g = workloads.config_inputs("mlp_2layer")
    t = {k: torch.from_numpy(v).to(dev) for k, v in g.items()}
    H = torch.empty((512, 11008), device=dev)
    Y = torch.empty((512, 4096), device=dev)

    def mlp():
        dense(t["X"], t["W1"], t["b1"], H, 1)
        dense(H, t["W2"], t["b2"], Y, 1)

    ms = time_calls(torch, stream, mlp, iters, 3, flush)
    _native.check(L.b200_stream_sync(sp))
    rows = sample_rows(512, 32)
    h64 = np.maximum(g["X"][rows].astype(np.float64) @ g["W1"] + g["b1"], 0)
    y64 = np.maximum(h64 @ g["W2"] + g["b2"], 0)
    err = float(np.max(np.abs(Y.cpu().numpy()[rows] - y64)))
    # bound of the second layer over its own (exact) input
    bound = 1e-4 * 11008 ** 0.5 * float(np.max(h64)) * float(np.max(np.abs(g["W2"])))
    fl = 2.0 * 512 * 4096 * 11008 * 2
    out.append({"config": "mlp_2layer", "ms": ms, "TFLOP/s": fl / ms / 1e9,
                "frac_of_3xtf32_peak": fl / ms / 1e9 / peak, "max_abs_err_vs_f64": err,
                "bound": bound, "ok": err <= bound})
    del t, H, Y
    # the same MLP end to end through @ml_function with host (NumPy) arrays:
    # every call copies X, W1, W2 in and Y out, unless W1 and W2 are
    # registered (b200_weights_register keeps their device copies and splits)
    from mlir_edsl import Tensor, f32, ml_function, register_weights, release_weights, relu

    @ml_function(target="b200")
    def mlp_fn(X: Tensor[f32, 512, 4096], W1: Tensor[f32, 4096, 11008], b1: Tensor[f32, 11008],
               W2: Tensor[f32, 11008, 4096], b2: Tensor[f32, 4096]) -> Tensor[f32, 512, 4096]:
        return relu(relu(X @ W1 + b1) @ W2 + b2)

    margs = (g["X"], g["W1"], g["b1"], g["W2"], g["b2"])

    def host_ms(k=5):
        mlp_fn(*margs)
        t0 = time.perf_counter()
        for _ in range(k):
            mlp_fn(*margs)
        return (time.perf_counter() - t0) / k * 1e3

    ms_plain = host_ms()
    register_weights(g["W1"])
    register_weights(g["W2"])
    try:
        ms_reg = host_ms()
    finally:
        release_weights(g["W1"])
        release_weights(g["W2"])
    out.append({"config": "mlp_2layer_frontend_e2e", "ms_per_call": ms_plain,
                "ms_per_call_registered_weights": ms_reg,
                "TFLOP/s": fl / ms_plain / 1e9, "TFLOP/s_registered_weights": fl / ms_reg / 1e9,
                "api": "@ml_function(target='b200') on NumPy arrays, host wall clock; "
                       "registered: mlir_edsl.register_weights(W1), (W2)"})
    # i32 2048^3 (byte-sliced int8 tensor-core path), bit-exact on sampled rows
    g = workloads.config_inputs("matmul_i32_2048")
    A, B = torch.from_numpy(g["A"]).to(dev), torch.from_numpy(g["B"]).to(dev)
    C = torch.empty_like(A)
    ms = time_calls(torch, stream, lambda: _native.check(L.b200_matmul_i32(
        P(A), 2048, P(B), 2048, None, P(C), 2048, 2048, 2048, 2048, sp)), iters, 3, flush)
    _native.check(L.b200_stream_sync(sp))
    rows = sample_rows(2048, 64)
    exact = (g["A"][rows].astype(np.int64) @ g["B"].astype(np.int64)).astype(np.int32)
    bf16, _ = peaks()
    i32_peak = 2.0 * bf16 / 10.0  # int8 rate = 2 x bf16; one i32 product = 10 u8 products
    out.append({"config": "matmul_i32_2048", "ms": ms, "Tint-op/s": 2.0 * 2048 ** 3 / ms / 1e9,
                "frac_of_tensor_peak": 2.0 * 2048 ** 3 / ms / 1e9 / i32_peak,
                "bit_exact": bool(np.array_equal(C.cpu().numpy()[rows], exact))})
    del A, B, C, flush
    torch.cuda.empty_cache()
    return out


def run_b200(args):
    import numpy as np
    import torch
    from mlir_edsl import _native

    rank, local_rank, world = dist_env()
    if world != args.gpus and world > 1:
        print(f"WORLD_SIZE={world} but --gpus {args.gpus}", file=sys.stderr)
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=dev)

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    from mlir_edsl.sharding import max_over_ranks as _max, row_shards

    def max_over_ranks(x):
        return _max(x, dist, dev)

    L = _native.lib()
    r0, rows = row_shards(M_TOTAL, world)[rank]
    if args.rows > 0:
        r0, rows = rank * args.rows, args.rows
    M, N, K = rows, N_DIM, K_DIM
    # this rank's rows of the seeded workload (bit-identical to the slice of
    # the whole X the parity tests check), W and b replicated
    Xh = workload_rows(r0, r0 + rows)
    Wh, bh = workload_weights()
    X = torch.from_numpy(Xh).to(dev)
    W = torch.from_numpy(Wh).to(dev)
    b = torch.from_numpy(bh).to(dev)
    Y = torch.empty((M, N), device=dev)
    stream = torch.cuda.current_stream()
    sp = ctypes.c_void_p(stream.cuda_stream)
    P = lambda t: ctypes.c_void_p(t.data_ptr())
    cpu_rows = 0
    if world == 1 and not args.no_cpu_baseline:
        import oracle
        oracle.build()
        cpu_rows = calibrate_rows(10.0, host_cores(), Xh, Wh, bh)

    def step():
        _native.check(L.b200_dense_f32(P(X), K, P(W), N, P(b), P(Y), N, M, N, K, 1, 0.0, sp))

    # ---- value: full step (split W, split X, GEMM), device-resident.
    # Clocks are sampled from the warm-up through the GEMM-only loop below.
    sampler = ClockSampler(local_rank)
    sampler.start()
    time.sleep(0.5)
    for _ in range(args.warmup):
        step()
    _native.check(L.b200_stream_sync(sp))
    barrier()
    launches0 = _native.launch_count()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        step()
    e1.record(stream)
    barrier()
    launches = _native.launch_count() - launches0
    _native.check(L.b200_stream_sync(sp))
    ms_local = e0.elapsed_time(e1)
    ms_total = max_over_ranks(ms_local)
    flops_step = 2.0 * M * N * K
    flops_job = (2.0 * M_TOTAL * N * K) if args.rows == 0 else world * flops_step
    value = flops_job * args.steps / (ms_total / 1e3) / 1e12
    # ---- result check of the timed output: sampled rows (first, last, shard
    # edges of the whole 65536-row layer, random) against float64 NumPy
    rows_s = sample_rows(M, 256, shards=max(1, 8 // world))
    idx = torch.from_numpy(rows_s).to(dev)
    err = check_rows(Xh, Wh, bh, Y.index_select(0, idx).cpu().numpy(), rows_s)
    bound = f32_bound(K, Xh, Wh)
    check = {"rows_checked_per_rank": int(len(rows_s)), "max_abs_err_vs_f64": max_over_ranks(err),
             "bound": -max_over_ranks(-bound),
             "tolerance": "1e-4*sqrt(K)*max|X|*max|W|"}
    check["ok"] = check["max_abs_err_vs_f64"] <= check["bound"]
    Y_cpu_rows = Y[:cpu_rows].cpu().numpy() if cpu_rows else None

    # ---- roofline: the GEMM kernel alone on pre-split operands
    Kp = _native.split_pitch(K)
    xhi = torch.empty((M, Kp), device=dev)
    xlo = torch.empty_like(xhi)
    whi = torch.empty((N, Kp), device=dev)
    wlo = torch.empty_like(whi)
    _native.check(L.b200_tf32_split_rows(P(X), K, M, K, P(xhi), P(xlo), sp))
    _native.check(L.b200_tf32_split_transpose(P(W), N, K, N, P(whi), P(wlo), sp))

    def gemm():
        _native.check(L.b200_gemm_tf32x3_presplit(P(xhi), P(xlo), P(whi), P(wlo), P(b), P(Y), N,
                                                  M, N, K, 1, 0.0, sp))

    for _ in range(2):
        gemm()
    barrier()
    e0.record(stream)
    for _ in range(args.steps):
        gemm()
    e1.record(stream)
    barrier()
    _native.check(L.b200_stream_sync(sp))
    gemm_ms = max_over_ranks(e0.elapsed_time(e1) / args.steps)
    # keep the GPU busy long enough for several clock samples, then stop
    t_soak = time.perf_counter()
    while time.perf_counter() - t_soak < 1.0:
        gemm()
        torch.cuda.synchronize()
    clocks = sampler.stop()
    bf16, peak_src = peaks()
    peak = bf16 / 6.0
    achieved = flops_step / (gemm_ms / 1e3) / 1e12
    traffic, traffic_src = None, None
    tfile = os.path.join(ROOT, "profiles", "gemm_tf32x3_dense65536_traffic.txt")
    if os.path.exists(tfile):
        for ln in open(tfile):
            if ln.startswith("bytes_per_launch_rows_") and f"rows_{M}:" in ln:
                traffic = float(ln.split(":")[1].split()[0])
                traffic_src = ln.split("#", 1)[1].strip() if "#" in ln else "ncu capture"
    del xhi, xlo, whi, wlo
    roofline = {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                "frac": achieved / peak, "traffic": traffic, "traffic_source": traffic_src,
                "algorithmic_bytes": 4.0 * (M * K + K * N + M * N + N),
                "kernel": "gemm_tf32x3_kernel",
                "peak_source": f"{peak_src} cuBLAS bf16 burst {bf16:.1f} TFLOP/s / 2 (tf32 "
                               f"rate) / 3 (three MMAs per product) = 3xTF32-effective",
                "kernel_ms": gemm_ms, "step_ms": ms_total / args.steps,
                "kernel_share_of_step": gemm_ms / (ms_total / args.steps)}

    # ---- e2e: plugin ABI with host buffers, copies inside every step
    fn = L.b200_memref_dense_relu_f32
    i64 = ctypes.c_int64
    vp = ctypes.c_void_p
    fn.argtypes = [vp, vp, i64, i64, i64, i64, i64] * 2 + [vp, vp, i64, i64, i64] + \
                  [vp, vp, i64, i64, i64, i64, i64]
    fn.restype = None

    def memref_args(xa, wa, ba, ya):
        d2 = lambda p, r, c: [vp(p), vp(p), 0, r, c, c, 1]
        return d2(xa, M, K) + d2(wa, K, N) + [vp(ba), vp(ba), 0, N, 1] + d2(ya, M, N)

    def e2e_time(call_args, steps):
        def e2e_step():
            fn(*call_args)
            _native.check_last()
        for _ in range(max(1, min(args.warmup, 2))):
            e2e_step()
        barrier()
        t0 = time.perf_counter()
        for _ in range(steps):
            e2e_step()
        return max_over_ranks(time.perf_counter() - t0)

    e2e, e2e_pageable = None, None
    if not args.no_e2e:
        Xp = torch.from_numpy(Xh).pin_memory()
        Wp = torch.from_numpy(Wh).pin_memory()
        bp = torch.from_numpy(bh).pin_memory()
        Yp = torch.empty((M, N), pin_memory=True)
        t_e2e = e2e_time(memref_args(Xp.data_ptr(), Wp.data_ptr(), bp.data_ptr(),
                                     Yp.data_ptr()), args.steps)
        e2e_err = max_over_ranks(check_rows(Xh, Wh, bh, Yp.numpy()[rows_s], rows_s))
        # e2e roofline: the same bytes copied alone (H2D and D2H concurrently
        # on two streams, pinned buffers), i.e. the PCIe floor of one step
        dX, dW, db, dY = torch.empty_like(X), torch.empty_like(W), torch.empty_like(b), \
            torch.empty_like(Y)
        s_in, s_out = torch.cuda.Stream(), torch.cuda.Stream()

        def copies():
            with torch.cuda.stream(s_in):
                dX.copy_(Xp, non_blocking=True)
                dW.copy_(Wp, non_blocking=True)
                db.copy_(bp, non_blocking=True)
            with torch.cuda.stream(s_out):
                Yp.copy_(dY, non_blocking=True)
        copies()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(3):
            copies()
        torch.cuda.synchronize()
        copy_floor_ms = (time.perf_counter() - t0) / 3 * 1e3
        del dX, dW, db, dY
        e2e = {"value": flops_job * args.steps / t_e2e / 1e12, "unit": UNIT,
               "copy_floor_ms": copy_floor_ms,
               "frac_of_copy_floor": copy_floor_ms / (t_e2e / args.steps * 1e3),
               "h2d_bytes_per_step": (M * K + K * N + N) * 4, "d2h_bytes_per_step": M * N * 4,
               "ms_per_step": t_e2e / args.steps * 1e3, "max_abs_err_vs_f64": e2e_err,
               "api": "b200_memref_dense_relu_f32 (reference flattened-memref ABI), pinned host "
                      "buffers, host wall clock, max over ranks"}
        del Xp, Wp, bp, Yp
        # the path the reference's callers take: plain (pageable) NumPy arrays
        Yh = np.empty((M, N), np.float32)
        k_pg = max(1, min(args.steps, 5))
        t_pg = e2e_time(memref_args(Xh.ctypes.data, Wh.ctypes.data, bh.ctypes.data,
                                    Yh.ctypes.data), k_pg)
        e2e_pageable = {"value": flops_job * k_pg / t_pg / 1e12, "unit": UNIT,
                        "ms_per_step": t_pg / k_pg * 1e3, "steps": k_pg,
                        "h2d_bytes_per_step": (M * K + K * N + N) * 4,
                        "d2h_bytes_per_step": M * N * 4,
                        "max_abs_err_vs_f64": max_over_ranks(
                            check_rows(Xh, Wh, bh, Yh[rows_s], rows_s)),
                        "api": "b200_memref_dense_relu_f32 with pageable NumPy arrays (staged "
                               "through the runtime's pinned slabs), host wall clock"}
        del Yh

    # ---- single-device result requested: the full Y on every rank
    gathered = None
    if world > 1 and not args.no_gather:
        from mlir_edsl.sharding import dense_rows

        def gtime(slabs, transport="ce"):
            for _ in range(2):
                Yf = dense_rows(X, W, b, 1, 0.0, gather=True, slabs=slabs,
                                reserve_sms=args.gather_reserve_sms, transport=transport)
            barrier()
            e0.record(stream)
            for _ in range(args.steps):
                Yf = dense_rows(X, W, b, 1, 0.0, gather=True, slabs=slabs,
                                reserve_sms=args.gather_reserve_sms, transport=transport)
            e1.record(stream)
            barrier()
            ms = max_over_ranks(e0.elapsed_time(e1) / args.steps)
            step()
            torch.cuda.synchronize()
            # this rank's gathered rows against its sharded result, and a
            # sample of every rank's rows against float64; max over ranks so
            # that every rank reaches the same verdict
            mine = float((Yf.view(world, M, N)[rank] - Y).abs().max())
            other = (rank + 1) % world
            orows = rows_s[:32]
            oerr = check_rows(workload_rows(other * M, (other + 1) * M)[: orows.max() + 1],
                              Wh, bh, Yf.view(world, M, N)[other].index_select(
                                  0, idx[:32]).cpu().numpy(), orows)
            return ms, max_over_ranks(max(mine, oerr))

        try:
            gf_ms, gf_err = gtime(1, "fused")
            g_ms, g_err = gtime(args.gather_slabs)
            gn_ms, gn_err = gtime(args.gather_slabs, "nccl")
            try:
                gm_ms, gm_err = gtime(1, "multimem")
                gm_note = None
            except RuntimeError as ex:  # no NVSwitch multicast: agreed on every rank
                gm_ms, gm_err, gm_note = float("inf"), 0.0, str(ex)[:200]
            if max(g_err, gn_err, gf_err, gm_err) > check["bound"]:
                raise RuntimeError(f"gathered rows differ: {max(g_err, gn_err, gf_err, gm_err)} "
                                   f"> {check['bound']}")
            recv = (world - 1) * M * N * 4
            best = min(gf_ms, g_ms, gn_ms, gm_ms)
            gathered = {
                "value": flops_job / (best / 1e3) / 1e12, "unit": UNIT, "ms_per_step": best,
                "sharded_ms_per_step": ms_total / args.steps,
                "ratio_to_sharded": best / (ms_total / args.steps),
                "recv_bytes_per_rank": recv, "recv_GBps_per_rank": recv / (best / 1e3) / 1e9,
                "multimem_ms_per_step": gm_ms if gm_note is None else None,
                "multimem_transport": gm_note or "the GEMM epilogue (and the cut-tile reduction) "
                                     "stores every final value once to the NVSwitch multicast "
                                     "address of the rows (multimem.st), which writes it into "
                                     "every rank's output buffer",
                "fused_ms_per_step": gf_ms,
                "fused_transport": "the GEMM epilogue (and the cut-tile reduction) stores every "
                                   "final value into each peer's IPC-mapped output buffer as "
                                   "well as its own (st.global over NVLink, no copy pass)",
                "ce_ms_per_step": g_ms, "slabs": args.gather_slabs,
                "ce_transport": "copy engines: each finished slab pushed into every peer's "
                                "CUDA-IPC-mapped output buffer (peer DMA over NVLink/NVSwitch, "
                                "one copy stream per peer), overlapping the next slab's GEMM",
                "nccl_ms_per_step": gn_ms, "reserve_sms": args.gather_reserve_sms,
                "nccl_transport": "NCCL all_gather_into_tensor per slab on a side stream, GEMM "
                                  "grid leaving reserve_sms SMs free",
                "max_abs_err_vs_f64": max(g_err, gn_err, gf_err, gm_err)}
        except RuntimeError as ex:  # raised on every rank alike (agreed collectively)
            gathered = {"unavailable": str(ex)[:200]}
        torch.cuda.empty_cache()

    # ---- CPU baseline (rank 0, N=1): the oracle on the first rows of the same
    # inputs, its result compared with the timed GPU output of those rows
    cpu = None
    if world == 1 and rank == 0 and cpu_rows:
        cores = host_cores()
        dt, fl, Yo = time_oracle_rows(Xh[:cpu_rows], Wh, bh, cores)
        err_o = float(np.max(np.abs(Yo.astype(np.float64) - Y_cpu_rows)))
        cpu = {"value": fl / dt / 1e12, "unit": UNIT, "cores": cores, "kind": "port",
               "sample": f"X[:{cpu_rows}] rows of the workload @ W + b, relu, one run "
                         f"({dt:.1f} s); oracle/ref_linalg.c restatement of the reference CPU "
                         f"pipeline",
               "gpu_vs_oracle": {"rows": cpu_rows, "max_abs_err": err_o, "bound": bound,
                                 "ok": err_o <= bound}}
        # NumPy (BLAS) on the same rows, as the reference's benchmarks time it
        # for context (benchmarks/bench_dense_layer.py); not the baseline
        np.maximum(Xh[:64] @ Wh + bh, 0)
        t0 = time.perf_counter()
        np.maximum(Xh[:cpu_rows] @ Wh + bh, 0)
        dtn = time.perf_counter() - t0
        cpu["numpy_context"] = {"value": 2.0 * cpu_rows * N_DIM * K_DIM / dtn / 1e12,
                                "unit": UNIT, "sample": f"np.maximum(X @ W + b, 0) on the same "
                                                        f"{cpu_rows} rows ({dtn:.2f} s)"}
        del Yo, Y_cpu_rows

    # ---- headline 8192^3 dense layer and the other configurations (N=1 only)
    headline, configs = None, None
    if world == 1 and not args.no_headline:
        del X, Y
        torch.cuda.empty_cache()
        from mlir_edsl import workloads
        g8 = workloads.config_inputs("dense_8192")
        n = 8192
        A, B, bb = (torch.from_numpy(g8[k]).to(dev) for k in ("A", "B", "b"))
        C = torch.empty((n, n), device=dev)

        def hstep():
            _native.check(L.b200_dense_f32(P(A), n, P(B), n, P(bb), P(C), n, n, n, n, 1, 0.0, sp))

        for _ in range(args.warmup):
            hstep()
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(args.steps):
            hstep()
        e1.record(stream)
        torch.cuda.synchronize()
        hms = e0.elapsed_time(e1) / args.steps
        hval = 2.0 * n ** 3 / (hms / 1e3) / 1e12
        hrows = sample_rows(n, 128)
        herr = check_rows(g8["A"], g8["B"], g8["b"],
                          C.index_select(0, torch.from_numpy(hrows).to(dev)).cpu().numpy(), hrows)
        hbound = f32_bound(n, g8["A"], g8["B"])
        headline = {"workload": "dense_relu 8192^3 (seed 2, with bias)", "value": hval,
                    "unit": UNIT, "ms_per_step": hms, "frac_of_3xtf32_peak": hval / peak,
                    "l2": "inputs larger than L2 (A, B 256 MiB each)",
                    "max_abs_err_vs_f64": herr, "bound": hbound, "ok": herr <= hbound}
        del A, B, bb, C, g8
        torch.cuda.empty_cache()
        configs = small_configs(torch, L, _native, dev, stream, peak, args)

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_total / args.steps,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (np.random.default_rng(3), uniform[-0.5,0.5]; each rank draws "
                    "its own rows of the one seeded X)",
            "config": {"workload": "dense_relu X[65536,4096] @ W[4096,4096] + b, rows split "
                                   "across GPUs", "M_total": M_TOTAL, "N": N, "K": K,
                       "rows_per_gpu": M, "parallelism": f"dp{world} (row shards, W/b "
                                                         "replicated, no collective)",
                       "l2": "inputs larger than L2 (X rows >= 128 MiB + W 64 MiB per GPU)",
                       "precision": "3xTF32 tensor cores, f32 accumulation promoted every 256 "
                                    "of K"},
            "check": check,
            "roofline": roofline, "e2e": e2e, "e2e_pageable": e2e_pageable,
            "cpu_baseline": cpu, "clocks": clocks, "gathered": gathered,
            "gpu_launches": launches, "headline_8192": headline, "configs": configs,
        }
        emit_line(line)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    return 0


# ----------------------------------------------------------------- HBM-bound ops
def run_configs(args):
    """Device time of the standalone HBM-bound ops (unfused bias+relu over the
    65536 x 4096 layer output, 1-D reductions and dot over 2^28 f32), one JSON
    line each; the dense configurations are part of the default line."""
    import torch
    from mlir_edsl import _native
    L = _native.lib()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    stream = torch.cuda.current_stream()
    sp = ctypes.c_void_p(stream.cuda_stream)
    P = lambda t: ctypes.c_void_p(t.data_ptr()) if t is not None else None
    g = torch.Generator(device=dev)

    def timed(fn):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        _native.check(L.b200_stream_sync(sp))
        return e0.elapsed_time(e1) / args.steps

    def u(shape, seed):
        g.manual_seed(seed)
        return torch.rand(shape, generator=g, device=dev) * 2 - 1

    def emit(name, ms, nbytes):
        emit_line({"config": name, "ms": ms, "GB/s": nbytes / ms / 1e6})

    Xe, be = u((65536, 4096), 9), u((4096,), 10)
    Ye = torch.empty_like(Xe)
    ms = timed(lambda: _native.check(L.b200_bias_act_f32(P(Xe), 4096, P(be), P(Ye), 4096, 65536,
                                                         4096, 1, 0.0, sp)))
    emit("bias_relu_65536x4096", ms, 2.0 * 65536 * 4096 * 4 + 4096 * 4)
    del Xe, be, Ye
    n = 1 << 28
    xr, yr = u((n,), 11), u((n,), 12)
    out = torch.empty(1, device=dev)
    ms = timed(lambda: _native.check(L.b200_reduce_f32(P(xr), n, 0, 0.0, P(out), sp)))
    emit("tensor_sum_2^28", ms, 4.0 * n)
    ms = timed(lambda: _native.check(L.b200_dot_f32(P(xr), P(yr), n, P(out), sp)))
    emit("dot_2^28", ms, 8.0 * n)
    return 0

_STDOUT_FD = None


def emit_line(line):
    """Writes the one JSON result line to the real stdout (libraries such as
    NCCL print to stdout during the run, which is redirected to stderr)."""
    os.write(_STDOUT_FD if _STDOUT_FD is not None else 1, (json.dumps(line) + "\n").encode())


def main():
    global _STDOUT_FD
    args = parse_args()
    sys.stdout.flush()
    _STDOUT_FD = os.dup(1)
    os.dup2(2, 1)
    if args.configs:
        return run_configs(args)
    if args.impl == "reference":
        return run_reference(args)
    return run_b200(args)


if __name__ == "__main__":
    sys.exit(main())
