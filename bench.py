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
  cpu_baseline  (rank 0, N=1) the CPU oracle, a restatement of the reference's
            CPU pipeline, on a bounded row sample of the same workload.
  headline_8192 (N=1) the 8192^3 dense layer, device-resident.

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
                    help="measure every BASELINE.json config on one GPU, one JSON line each")
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


# ----------------------------------------------------------------- CPU oracle timing
_ORACLE_INPUTS = {}


def _oracle_inputs(rows):
    import numpy as np
    have = _ORACLE_INPUTS.get("X")
    if have is None or have.shape[0] < rows:
        rng = np.random.default_rng(3)
        _ORACLE_INPUTS["W"] = rng.uniform(-0.5, 0.5, (K_DIM, N_DIM)).astype(np.float32)
        _ORACLE_INPUTS["b"] = rng.uniform(-0.5, 0.5, (N_DIM,)).astype(np.float32)
        _ORACLE_INPUTS["X"] = rng.uniform(-0.5, 0.5, (max(rows, 64), K_DIM)).astype(np.float32)
    return _ORACLE_INPUTS["X"][:rows], _ORACLE_INPUTS["W"], _ORACLE_INPUTS["b"]


def time_oracle_rows(rows, threads, act=1):
    """Times the CPU restatement of the reference pipeline on `rows` rows of
    the workload; returns (seconds, flops)."""
    import oracle
    X, W, b = _oracle_inputs(rows)
    t0 = time.perf_counter()
    oracle.dense_f32(X, W, b, act=act, threads=threads)
    dt = time.perf_counter() - t0
    return dt, 2.0 * rows * N_DIM * K_DIM


def calibrate_rows(target_s, threads):
    """Row count whose oracle run takes about target_s seconds (multiple of 64)."""
    probe = 64
    dt, _ = time_oracle_rows(probe, threads)
    rows = int(probe * target_s / max(dt, 1e-3))
    return max(64, min(M_TOTAL, rows // 64 * 64))


def run_reference(args):
    rank, _, world = dist_env()
    if rank != 0:
        return 0
    import oracle
    oracle.build()
    cores = host_cores()
    per_step = max(1.0, min(8.0, 150.0 / max(1, args.steps + args.warmup)))
    rows = calibrate_rows(per_step, cores)
    for _ in range(args.warmup):
        time_oracle_rows(rows, cores)
    times = []
    for _ in range(args.steps):
        dt, flops = time_oracle_rows(rows, cores)
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
    rows = args.rows if args.rows > 0 else row_shards(M_TOTAL, world)[rank][1]
    M, N, K = rows, N_DIM, K_DIM
    g = torch.Generator(device=dev)
    g.manual_seed(3 + 1000 * rank)
    X = torch.rand((M, K), generator=g, device=dev) - 0.5
    W = torch.rand((K, N), generator=g, device=dev) - 0.5
    b = torch.rand((N,), generator=g, device=dev) - 0.5
    Y = torch.empty((M, N), device=dev)
    stream = torch.cuda.current_stream()
    sp = ctypes.c_void_p(stream.cuda_stream)
    P = lambda t: ctypes.c_void_p(t.data_ptr())

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
    traffic = None
    tfile = os.path.join(ROOT, "profiles", "gemm_tf32x3_dense65536_traffic.txt")
    if os.path.exists(tfile):
        for ln in open(tfile):
            if ln.startswith("bytes_per_launch_rows_") and f"rows_{M}:" in ln:
                traffic = float(ln.split(":")[1])
    del xhi, xlo, whi, wlo
    roofline = {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                "frac": achieved / peak, "traffic": traffic,
                "kernel": "gemm_tf32x3_kernel",
                "peak_source": f"{peak_src} cuBLAS bf16 burst {bf16:.1f} TFLOP/s / 2 (tf32 "
                               f"rate) / 3 (three MMAs per product) = 3xTF32-effective",
                "kernel_ms": gemm_ms, "step_ms": ms_total / args.steps,
                "kernel_share_of_step": gemm_ms / (ms_total / args.steps)}

    # ---- e2e: plugin ABI with pinned host buffers, copies inside every step
    e2e = None
    if not args.no_e2e:
        Xh = torch.empty((M, K), pin_memory=True)
        Wh = torch.empty((K, N), pin_memory=True)
        bh = torch.empty((N,), pin_memory=True)
        Yh = torch.empty((M, N), pin_memory=True)
        Xh.copy_(X)
        Wh.copy_(W)
        bh.copy_(b)
        fn = L.b200_memref_dense_relu_f32
        i64 = ctypes.c_int64
        vp = ctypes.c_void_p
        fn.argtypes = [vp, vp, i64, i64, i64, i64, i64] * 2 + [vp, vp, i64, i64, i64] + \
                      [vp, vp, i64, i64, i64, i64, i64]
        fn.restype = None
        d2 = lambda t, r, c: [vp(t.data_ptr()), vp(t.data_ptr()), 0, r, c, c, 1]
        call_args = d2(Xh, M, K) + d2(Wh, K, N) + [vp(bh.data_ptr()), vp(bh.data_ptr()), 0, N, 1] \
            + d2(Yh, M, N)

        def e2e_step():
            fn(*call_args)
            _native.check_last()

        for _ in range(max(1, min(args.warmup, 2))):
            e2e_step()
        barrier()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            e2e_step()
        t_e2e = max_over_ranks(time.perf_counter() - t0)
        # correctness of the e2e result against the device-resident path
        step()
        torch.cuda.synchronize()
        # (split-K or slab boundaries may change the K summation order)
        bound = 1e-4 * K ** 0.5 * float(X.abs().max()) * float(W.abs().max())
        e2e_err = float((Yh - Y.cpu()).abs().max())
        assert e2e_err <= bound, f"e2e result differs from device path: {e2e_err} > {bound}"
        # e2e roofline: the same bytes copied alone (H2D and D2H concurrently
        # on two streams, pinned buffers), i.e. the PCIe floor of one step
        dX, dW, db, dY = torch.empty_like(X), torch.empty_like(W), torch.empty_like(b), \
            torch.empty_like(Y)
        s_in, s_out = torch.cuda.Stream(), torch.cuda.Stream()

        def copies():
            with torch.cuda.stream(s_in):
                dX.copy_(Xh, non_blocking=True)
                dW.copy_(Wh, non_blocking=True)
                db.copy_(bh, non_blocking=True)
            with torch.cuda.stream(s_out):
                Yh.copy_(dY, non_blocking=True)
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
               "ms_per_step": t_e2e / args.steps * 1e3,
               "api": "b200_memref_dense_relu_f32 (reference flattened-memref ABI), pinned host "
                      "buffers, host wall clock, max over ranks"}
        del Xh, Wh, bh, Yh

    # ---- single-device result requested: the full Y on every rank, all-gathered
    # with NCCL over NVLink slab by slab while the next slab's GEMM runs
    # (mlir_edsl.sharding.dense_rows(gather=True)); device time, max over ranks
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
            # this rank's gathered rows against its sharded result; max over
            # ranks so that every rank reaches the same verdict
            err = max_over_ranks(float((Yf.view(world, M, N)[rank] - Y).abs().max()))
            return ms, err

        bound = 1e-4 * K ** 0.5 * float(X.abs().max()) * float(W.abs().max())
        bound = -max_over_ranks(-bound)  # the tightest rank's bound, the same on every rank
        try:
            g_ms, g_err = gtime(args.gather_slabs)
            g1_ms, _ = gtime(1)
            gn_ms, gn_err = gtime(args.gather_slabs, "nccl")
            gf_ms, gf_err = gtime(1, "fused")
            if max(g_err, gn_err, gf_err) > bound:
                raise RuntimeError(f"gathered rows differ from the sharded result: "
                                   f"{max(g_err, gn_err, gf_err)} > {bound}")
            recv = (world - 1) * M * N * 4
            gathered = {
                "value": flops_job / (g_ms / 1e3) / 1e12, "unit": UNIT, "ms_per_step": g_ms,
                "slabs": args.gather_slabs, "reserve_sms": args.gather_reserve_sms,
                "ms_per_step_unpipelined": g1_ms, "sharded_ms_per_step": ms_total / args.steps,
                "recv_bytes_per_rank": recv, "recv_GBps_per_rank": recv / (g_ms / 1e3) / 1e9,
                "transport": "copy engines: each finished slab pushed into every peer's "
                             "CUDA-IPC-mapped output buffer (peer DMA over NVLink/NVSwitch, one "
                             "copy stream per peer), overlapping the next slab's GEMM",
                "fused_ms_per_step": gf_ms,
                "fused_transport": "the GEMM epilogue (and the cut-tile reduction) stores every "
                                   "final value into each peer's IPC-mapped output buffer as "
                                   "well as its own (st.global over NVLink, no copy pass)",
                "nccl_ms_per_step": gn_ms,
                "nccl_transport": "NCCL all_gather_into_tensor per slab on a side stream, GEMM "
                                  "grid leaving reserve_sms SMs free"}
        except RuntimeError as ex:  # raised on every rank alike (agreed collectively)
            gathered = {"unavailable": str(ex)[:200]}
        torch.cuda.empty_cache()

    # ---- headline 8192^3 dense (N=1 only)
    headline = None
    if world == 1 and not args.no_headline:
        del X, Y
        torch.cuda.empty_cache()
        n = 8192
        g.manual_seed(2)
        A = torch.rand((n, n), generator=g, device=dev) * 2 - 1
        B = torch.rand((n, n), generator=g, device=dev) * 2 - 1
        bb = torch.rand((n,), generator=g, device=dev) * 2 - 1
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
        headline = {"workload": "dense_relu 8192^3 (seed 2)", "value": hval, "unit": UNIT,
                    "ms_per_step": hms, "frac_of_3xtf32_peak": hval / peak}
        del A, B, bb, C

    # ---- CPU baseline (rank 0, N=1)
    cpu = None
    if world == 1 and rank == 0 and not args.no_cpu_baseline:
        import oracle
        oracle.build()
        cores = host_cores()
        rows_s = calibrate_rows(10.0, cores)
        dt, fl = time_oracle_rows(rows_s, cores)
        cpu = {"value": fl / dt / 1e12, "unit": UNIT, "cores": cores, "kind": "port",
               "sample": f"X[{rows_s},{K_DIM}] rows of the workload @ W + b, relu, one run "
                         f"({dt:.1f} s); oracle/ref_linalg.c restatement of the reference CPU "
                         f"pipeline"}
        # NumPy (BLAS) on the same rows, as the reference's benchmarks time it
        # for context (benchmarks/bench_dense_layer.py); not the baseline
        Xs, Ws, bs = _oracle_inputs(rows_s)
        np.maximum(Xs[:64] @ Ws + bs, 0)
        t0 = time.perf_counter()
        np.maximum(Xs @ Ws + bs, 0)
        dtn = time.perf_counter() - t0
        cpu["numpy_context"] = {"value": 2.0 * rows_s * N_DIM * K_DIM / dtn / 1e12,
                                "unit": UNIT, "sample": f"np.maximum(X @ W + b, 0) on the same "
                                                        f"{rows_s} rows ({dtn:.2f} s)"}
        del Xs, Ws, bs

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_total / args.steps,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (torch.Generator seed 3+1000*rank, uniform[-0.5,0.5])",
            "config": {"workload": "dense_relu X[65536,4096] @ W[4096,4096] + b, rows split "
                                   "across GPUs", "M_total": M_TOTAL, "N": N, "K": K,
                       "rows_per_gpu": M, "parallelism": f"dp{world} (row shards, W/b "
                                                         "replicated, no collective)",
                       "l2": "inputs larger than L2 (X rows >= 128 MiB + W 64 MiB per GPU)",
                       "precision": "3xTF32 tensor cores, f32 accumulation promoted every 256 "
                                    "of K"},
            "roofline": roofline, "e2e": e2e, "cpu_baseline": cpu, "clocks": clocks,
            "gathered": gathered,
            "gpu_launches": launches, "headline_8192": headline,
        }
        emit_line(line)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    return 0



# ----------------------------------------------------------------- per-config table
def run_configs(args):
    """Device-resident timing of every BASELINE.json configuration on GPU 0
    (parity for each is covered by tests/); one JSON line per config."""
    import torch
    from mlir_edsl import _native
    L = _native.lib()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    stream = torch.cuda.current_stream()
    sp = ctypes.c_void_p(stream.cuda_stream)
    P = lambda t: ctypes.c_void_p(t.data_ptr()) if t is not None else None
    bf16, _ = peaks()
    peak = bf16 / 6.0
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

    def u(shape, seed, lo=-1.0, hi=1.0):
        g.manual_seed(seed)
        return torch.rand(shape, generator=g, device=dev) * (hi - lo) + lo

    def dense(X, W, b, Y, act):
        M, K = X.shape
        N = W.shape[1]
        _native.check(L.b200_dense_f32(P(X), K, P(W), N, P(b), P(Y), N, M, N, K, act, 0.0, sp))

    def emit(name, ms, flops=None, nbytes=None):
        line = {"config": name, "ms": ms}
        if flops:
            line.update({"TFLOP/s": flops / ms / 1e9, "frac_of_3xtf32_peak": flops / ms / 1e9 / peak})
        if nbytes:
            line["GB/s"] = nbytes / ms / 1e6
        emit_line(line)

    for name, (M, N, K), act, with_b, seed, lo in [
            ("matmul_256", (256, 256, 256), 0, False, 0, -1.0),
            ("dense_1024", (1024, 1024, 1024), 1, True, 1, -1.0),
            ("matmul_4096", (4096, 4096, 4096), 0, False, 2, -1.0),
            ("matmul_8192", (8192, 8192, 8192), 0, False, 2, -1.0),
            ("dense_65536", (65536, 4096, 4096), 1, True, 3, -0.5),
            ("dense_ragged", (1000, 999, 1001), 1, True, 4, -1.0)]:
        X, W = u((M, K), seed, lo, -lo), u((K, N), seed + 100, lo, -lo)
        b = u((N,), seed + 200, lo, -lo) if with_b else None
        Y = torch.empty((M, N), device=dev)
        emit(name, timed(lambda: dense(X, W, b, Y, act)), flops=2.0 * M * N * K)
        del X, W, b, Y
    # 2-layer MLP: relu(relu(X@W1+b1)@W2+b2), hidden activation stays in HBM
    X, W1, b1 = u((512, 4096), 4), u((4096, 11008), 5), u((11008,), 6)
    W2, b2 = u((11008, 4096), 7), u((4096,), 8)
    H, Y = torch.empty((512, 11008), device=dev), torch.empty((512, 4096), device=dev)
    emit("mlp_2layer", timed(lambda: (dense(X, W1, b1, H, 1), dense(H, W2, b2, Y, 1))),
         flops=2.0 * 512 * 4096 * 11008 * 2)
    del X, W1, b1, W2, b2, H, Y
    # i32 2048^3 (byte-sliced int8 tensor-core path) and 8192^3 beside it
    g.manual_seed(2)
    A = torch.randint(-8, 9, (2048, 2048), generator=g, device=dev, dtype=torch.int32)
    B = torch.randint(-8, 9, (2048, 2048), generator=g, device=dev, dtype=torch.int32)
    C = torch.empty_like(A)
    ms = timed(lambda: _native.check(L.b200_matmul_i32(P(A), 2048, P(B), 2048, None, P(C), 2048,
                                                      2048, 2048, 2048, sp)))
    line = {"config": "matmul_i32_2048", "ms": ms, "Tint-op/s": 2.0 * 2048 ** 3 / ms / 1e9}
    # Roofline of the tensor-core path: one i32 multiply-add is ten u8 x u8
    # multiply-adds, and the dense int8 rate is twice the bf16 rate (nominal
    # 4.5 vs 2.25 PFLOP/s), so the peak in i32 int-op/s (2 per multiply-add)
    # is 2 x measured bf16 FLOP/s / 10.
    i32_peak = 2.0 * bf16 / 10.0
    line.update({"tensor_peak_Tint-op/s": i32_peak, "frac_of_tensor_peak":
                 line["Tint-op/s"] / i32_peak,
                 "peak_source": "measured cuBLAS bf16 burst x 2 (int8 rate) / 10 (u8 products "
                                "per i32 product)"})
    Ab = torch.randint(-2**31, 2**31 - 1, (8192, 8192), generator=g, device=dev,
                       dtype=torch.int32)
    Bb = torch.randint(-2**31, 2**31 - 1, (8192, 8192), generator=g, device=dev,
                       dtype=torch.int32)
    Cb = torch.empty_like(Ab)
    ms8 = timed(lambda: _native.check(L.b200_matmul_i32(P(Ab), 8192, P(Bb), 8192, None, P(Cb),
                                                       8192, 8192, 8192, 8192, sp)))
    line["i32_8192_full_range_Tint-op/s"] = 2.0 * 8192 ** 3 / ms8 / 1e9
    line["i32_8192_frac_of_tensor_peak"] = line["i32_8192_full_range_Tint-op/s"] / i32_peak
    del Ab, Bb, Cb
    # the CUDA-core alternative's ceiling: measured INT32 multiply-add issue
    # rate (lib/libb200probe.so)
    probe = ctypes.CDLL(os.path.join(ROOT, "ml-edsl_b200", "lib", "libb200probe.so"))
    probe.b200_probe_imad.restype = ctypes.c_float
    probe.b200_probe_imad.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
    pb, pit = 148 * 8, 2000
    pout = torch.empty(pb * 256, dtype=torch.int32, device=dev)
    pms = probe.b200_probe_imad(pb, pit, P(pout))
    if pms > 0:
        peak_ops = 2.0 * pb * 256 * pit * 128 / pms / 1e9  # multiply + add per IMAD
        line.update({"imad_peak_Tint-op/s": peak_ops,
                     "frac_of_imad_peak": line["Tint-op/s"] / peak_ops})
    emit_line(line)
    # unfused elementwise bias+relu over the cfg4 output shape (HBM-bound)
    Xe, be = u((65536, 4096), 9), u((4096,), 10)
    Ye = torch.empty_like(Xe)
    ms = timed(lambda: _native.check(L.b200_bias_act_f32(P(Xe), 4096, P(be), P(Ye), 4096, 65536,
                                                         4096, 1, 0.0, sp)))
    emit("bias_relu_65536x4096", ms, nbytes=2.0 * 65536 * 4096 * 4 + 4096 * 4)
    del Xe, be, Ye
    # 1-D reductions / dot over 2^28 f32 (1 GiB per operand, HBM-bound)
    n = 1 << 28
    xr, yr = u((n,), 11), u((n,), 12)
    out = torch.empty(1, device=dev)
    ms = timed(lambda: _native.check(L.b200_reduce_f32(P(xr), n, 0, 0.0, P(out), sp)))
    emit("tensor_sum_2^28", ms, nbytes=4.0 * n)
    ms = timed(lambda: _native.check(L.b200_dot_f32(P(xr), P(yr), n, P(out), sp)))
    emit("dot_2^28", ms, nbytes=8.0 * n)
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
