#!/usr/bin/env python
"""bench.py — NVFP4 GEMM throughput on B200, one process per GPU.

Headline: TFLOP/s of the block-scaled NVFP4 GEMM on the square workload M = N = K = 8192
(A, B bf16 N(0,1) drawn on the host from seed 2, quantized on the GPU with the reference
recipe), at 1..8 GPUs. N > 1 is column-parallel (weak scaling): every rank owns an 8192-column
shard of a global M x (8192*P) x K product (its own slice of B and B's scale factors, A
replicated), with no data-path collective; `value` is the work of all ranks over the
max-over-ranks device time.

One JSON line on rank 0. Besides the contract keys it carries:
  roofline      the GEMM kernel against B200's dense FP4 peak, 9.0 PFLOP/s (`frac`); the
                fraction of 4 x the measured cuBLAS bf16 rate is a secondary key
  cpu_baseline  the CPU oracle port (dequantize + fp32 matmul) on the same full 8192^3 problem
  e2e           the same metric through my_plugins.gemm_nvfp4 with pinned host buffers,
                host->device copies of the operands and device->host copy of D in the timing
  quantize / dequantize   GB/s of the 8192x8192 activation workload (0.5% x50 outliers)
  prefill       16384 x 57344 x 8192, weight sharded along N over the ranks (strong scaling):
                GEMM alone, GEMM with the all-gather fused into its epilogue, GEMM + NCCL
                all-gather (N > 1), each with its per-rank roofline fraction
  decode        M x 28672 x 8192 for M = 16 and 128, weight sharded along N: us per step
  clocks        SM clock samples (nvidia-smi) from warm-up start to the end of timing

`--impl reference` times the CPU implementation of the reference arithmetic (the oracle port;
the reference ships no CPU code and its GEMM does not build for sm_100a) on rank 0, on the
same operands and config.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

M_SQ = N_SQ = K_SQ = 8192
L2_FLUSH_BYTES = 256 << 20          # > 126 MB L2
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0
NOMINAL_FP4_TFLOPS = 9000.0        # B200 dense FP4 (the 18 PF HGX figure is with 2:4 sparsity)
NVLINK_GBS = 770.0                 # measured peer copy rate per direction per GPU on this pool
QUANT_BYTES = 8192 * 8192 * 2 + 8192 * 4096 + 8192 * 512   # 171,966,464 per pass


_RESULT_OUT = None


def keep_stdout_for_result():
    """Reserve the process's stdout for the one JSON result line: keep a private duplicate of
    file descriptor 1 for it and point descriptor 1 at stderr, so banners that libraries print
    to stdout (NCCL prints its version line at communicator creation when NCCL_DEBUG asks for
    it) end up on stderr."""
    global _RESULT_OUT
    sys.stdout.flush()
    _RESULT_OUT = os.fdopen(os.dup(1), "w")
    os.dup2(2, 1)


def emit(line):
    out = _RESULT_OUT if _RESULT_OUT is not None else sys.stdout
    print(json.dumps(line), file=out, flush=True)


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=500)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-quant", action="store_true")
    ap.add_argument("--no-sharded", action="store_true",
                    help="square workload: skip the prefill and decode measurements")
    ap.add_argument("--size", type=int, default=8192, help="M = N = K (profiling of small cases)")
    ap.add_argument("--workload", choices=["square", "decode", "prefill"], default="square",
                    help="square: 8192^3 (headline); decode: M x 28672 x 8192; "
                         "prefill: 16384 x 57344 x 8192 (N sharded across ranks)")
    ap.add_argument("--tokens", "--m", dest="m", type=int, default=128,
                    help="decode tokens (16, 32, 64, 128); under torchrun use --tokens, whose "
                         "launcher would take --m for an abbreviation of its own options")
    ap.add_argument("--gather", action="store_true",
                    help="prefill/decode: include the chunked NCCL all-gather of D in the timing")
    ap.add_argument("--swiglu", action="store_true",
                    help="prefill: the weight is gate+up (2 x 28672 rows); SwiGLU in the GEMM "
                         "epilogue, output [M, 28672]")
    ap.add_argument("--shard-of", type=int, default=1,
                    help="prefill/decode on one GPU: time rank 0's column shard of a P-way split "
                         "alone (the per-rank workload of a P-GPU run; profiling)")
    ap.add_argument("--fused-gather", action="store_true",
                    help="with --gather: the all-gather fused into the GEMM epilogue (stores into "
                         "every rank's output over NVLink) instead of NCCL")
    return ap.parse_args()


def measured_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, FALLBACK_BF16_TFLOPS, "fallback"


def profiled_traffic(key):
    """DRAM bytes per launch from a committed ncu summary (profiles/traffic.json), else None."""
    try:
        with open(os.path.join(ROOT, "profiles", "traffic.json")) as f:
            return json.load(f).get(key)
    except Exception:
        return None


# ------------------------------------------------------------------------------------------
class ClockSampler:
    """nvidia-smi samples of one GPU while it runs (started before warm-up, stopped after)."""

    FIELDS = ("uuid,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, uuid):
        self.uuid = uuid
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "20"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.out = ""
        if self.proc is not None:
            time.sleep(0.12)
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        rows = []
        for line in (getattr(self, "out", "") or "").splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9 or (self.uuid and f[0] != self.uuid):
                continue
            try:
                rows.append((float(f[1]), float(f[2]), float(f[3]), f[5:9]))
            except ValueError:
                continue
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        max_mhz = max(r[1] for r in rows)
        loaded = [r for r in rows if r[2] > 200.0] or rows  # samples under load (power > 200 W)
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in loaded for i, v in enumerate(r[3]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(r[0] for r in loaded), "sm_max_mhz": max_mhz,
                "reasons": reasons, "samples": len(loaded),
                "power_w_max": max(r[2] for r in rows)}


def gpu_uuid(torch, dev):
    try:
        u = str(torch.cuda.get_device_properties(dev).uuid)
        return u if u.startswith("GPU-") else "GPU-" + u
    except Exception:
        return None


# ------------------------------------------------------------------------------------------
def dist_setup(torch):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return world, rank, local


def barrier(torch, world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    torch.cuda.synchronize()


def max_over_ranks(torch, world, value):
    if world == 1:
        return value
    import torch.distributed as dist
    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def square_inputs_host(size, rank=0):
    """bf16 bit patterns (numpy uint16) of the square workload: A then B from one N(0,1) stream
    seeded with 2; rank r > 0 of a weak-scaled run draws its own B shard from seed (2, r). Both
    arms (and the CPU baseline) use exactly these operands."""
    import numpy as np
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import nvfp4_cases as cases
    rng = np.random.default_rng(2)
    A = cases.activation(rng, size, size)
    B = cases.activation(rng if rank == 0 else np.random.default_rng([2, rank]), size, size)
    return A, B


def make_square_operands(torch, plugins, size, rank):
    """A (replicated) and this rank's B shard uploaded and quantized on the GPU with the
    reference recipe s = 6*448 / amax."""
    import numpy as np
    A_bits, B_bits = square_inputs_host(size, rank)
    A = torch.from_numpy(A_bits.view(np.int16)).cuda().view(torch.bfloat16)
    B = torch.from_numpy(B_bits.view(np.int16)).cuda().view(torch.bfloat16)
    sA = 6 * 448 / A.abs().max().to(dtype=torch.float32)
    sB = 6 * 448 / B.abs().max().to(dtype=torch.float32)
    a, a_sf = plugins.quantize_nvfp4(A, sA)
    b, b_sf = plugins.quantize_nvfp4(B, sB)
    del A, B
    return a, b, a_sf, b_sf, (sA * sB).reshape(())


def square_config(size, world):
    """`config` of the square workload, the same for both arms."""
    return {"workload": f"square_gemm_{size}", "M": size, "N": size * world, "K": size,
            "n_per_rank": size, "parallelism": f"column-parallel N x{world}",
            "l2": "GPU arm: flushed (256 MiB write) before every timed launch",
            "inputs": "bf16 N(0,1), host numpy stream of seed 2 (A, then B; rank r>0 B from "
                      "seed (2, r)), quantized with s = 6*448/amax"}


def time_device(torch, fn, steps, warmup, flush, world):
    """Warm-up, then `steps` launches each timed by CUDA events on the current stream, with an
    L2 flush (untimed) before each. Returns the summed device milliseconds (max over ranks)."""
    stream = torch.cuda.current_stream()
    for _ in range(warmup):
        fn()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(steps)]
    barrier(torch, world)
    for s, e in ev:
        flush.zero_()
        s.record(stream)
        fn()
        e.record(stream)
    torch.cuda.synchronize()
    barrier(torch, world)
    total = sum(s.elapsed_time(e) for s, e in ev)
    return max_over_ranks(torch, world, total)


def time_device_streaming(torch, fn, steps, warmup, world):
    """For kernels whose per-call working set exceeds L2 (no flush needed between calls):
    `steps` back-to-back launches between one pair of CUDA events, so launch gaps do not count
    against a ~30 us kernel. Returns the summed device milliseconds (max over ranks)."""
    stream = torch.cuda.current_stream()
    for _ in range(warmup):
        fn()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(torch, world)
    s.record(stream)
    for _ in range(steps):
        fn()
    e.record(stream)
    torch.cuda.synchronize()
    barrier(torch, world)
    return max_over_ranks(torch, world, s.elapsed_time(e))


def time_graph_streaming(torch, fn, calls, replays, world):
    """`calls` launches of fn(stream) captured once into a CUDA graph, replayed `replays` times
    between one pair of CUDA events after one untimed replay: the device time per launch without
    the host's launch overhead (ms, max over ranks)."""
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        h = torch.cuda.current_stream().cuda_stream
        for _ in range(calls):
            fn(h)
    g.replay()
    stream = torch.cuda.current_stream()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    barrier(torch, world)
    s.record(stream)
    for _ in range(replays):
        g.replay()
    e.record(stream)
    torch.cuda.synchronize()
    barrier(torch, world)
    del g
    return max_over_ranks(torch, world, s.elapsed_time(e)) / (calls * replays)


def cpu_gemm_timer(qa, fa, qb, fb, scale):
    """One step of the reference arithmetic on the host (the oracle port): decode both
    block-scaled operands (oracle, OpenMP), fp32 matmul (torch, all host threads), / scale,
    bf16. `rows` limits the step to the first rows of A (the full problem when None)."""
    import numpy as np
    import torch
    from oracle import oracle as O
    s = torch.tensor(np.float32(scale))

    def step(rows=None):
        r = qa.shape[0] if rows is None else rows
        da = torch.from_numpy(O.decode_scaled(qa[:r], fa[:r]))
        db = torch.from_numpy(O.decode_scaled(qb, fb))
        return ((da @ db.T) / s).to(torch.bfloat16)
    return step


def cpu_baseline_gemm(a, b, a_sf, b_sf, scale, runs=3):
    """The CPU baseline of the GPU arm: the full problem, median of `runs` steps after one
    untimed step."""
    import torch
    from oracle import oracle as O
    step = cpu_gemm_timer(a.cpu().numpy(), a_sf.view(torch.uint8).cpu().numpy(), b.cpu().numpy(),
                          b_sf.view(torch.uint8).cpu().numpy(), scale.item())
    step()
    times = []
    for _ in range(runs):
        t0 = time.perf_counter()
        step()
        times.append(time.perf_counter() - t0)
    t = statistics.median(times)
    M, N, K = a.shape[0], b.shape[0], a.shape[1] * 2
    return {"value": 2.0 * M * N * K / t / 1e12, "unit": "TFLOP/s", "cores": torch.get_num_threads(),
            "kind": "port",
            "sample": f"the full {M}x{N}x{K} problem (same operands as the GPU arm) per run, median "
                      f"of {runs} runs after one untimed: oracle decode (OpenMP, {O.num_threads()} "
                      f"threads) + torch fp32 matmul + / scale + bf16; os.cpu_count()={os.cpu_count()}"}


def run_reference_arm(args):
    """CPU implementation of the reference arithmetic on the same operands and config as the
    GPU arm (rank 0 only; other ranks exit without work)."""
    import torch
    from oracle import oracle as O
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    size = args.size
    A_bits, B_bits = square_inputs_host(size, 0)
    sA, sB = O.global_scale(A_bits), O.global_scale(B_bits)
    qa, fa = O.quantize(A_bits, sA)            # operands quantized once, as on the GPU arm
    qb, fb = O.quantize(B_bits, sB)
    del A_bits, B_bits
    import numpy as np
    step = cpu_gemm_timer(qa, fa, qb, fb, np.float32(sA) * np.float32(sB))

    # Each step is the full problem unless the requested steps would then run for more than
    # ~3 minutes; then each step covers the first `rows` rows of A (a bounded sample of the same
    # workload) so that the whole run still ends within a few minutes.
    t0 = time.perf_counter()
    step()
    t_full = time.perf_counter() - t0
    rows = size
    n_more = max(args.warmup - 1, 0) + args.steps
    if n_more * t_full > 180.0:
        rows = max(128, min(size, int(size * 180.0 / (n_more * t_full)) // 128 * 128))
    for _ in range(max(args.warmup - 1, 0)):
        step(rows)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step(rows)
    dt = (time.perf_counter() - t0) / max(args.steps, 1)
    val = 2.0 * rows * size * size / dt / 1e12
    cores = torch.get_num_threads()
    sample = ((f"the full {size}x{size}x{size} problem per step" if rows == size else
               f"{rows} of {size} rows of A x full B per step (the full problem took "
               f"{t_full:.1f} s; steps bounded to ~3 min)")
              + f": decode of the block-scaled operands (oracle, OpenMP {O.num_threads()} threads) "
                "+ torch fp32 matmul + / scale + bf16, operands identical to the GPU arm's")
    line = {"metric": "nvfp4_gemm_tflops", "value": val, "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "e2m1/ue4m3->f32",
            "data": "synthetic", "impl": "reference",
            "config": square_config(size, world),
            "cpu_baseline": {"value": val, "unit": "TFLOP/s", "cores": cores, "kind": "port",
                             "sample": sample},
            "e2e": {"value": val, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    emit(line)
    return 0


def run_ours(args):
    import torch
    from my_nvfp4_gemm_b200 import capi, load_my_plugins
    plugins = load_my_plugins()
    world, rank, local = dist_setup(torch)
    dev = torch.cuda.current_device()
    size = args.size
    M = N = K = size
    flops = 2.0 * M * N * K
    hbm_gbs, bf16_tf, peak_src = measured_peaks()
    fp4_peak_bf16 = 4.0 * bf16_tf

    a, b, a_sf, b_sf, scale = make_square_operands(torch, plugins, size, rank)
    d = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device="cuda")
    stream_h = torch.cuda.current_stream().cuda_stream
    ptrs = (a.data_ptr(), b.data_ptr(), a_sf.data_ptr(), b_sf.data_ptr(), scale.data_ptr(), d.data_ptr())

    def gemm_once():
        st = capi.gemm(*ptrs, M, N, K, stream_h)
        if st:
            raise capi.NvFp4Error(st, "nvfp4_gemm")

    sampler = ClockSampler(gpu_uuid(torch, dev))
    with sampler:
        gemm_ms_total = time_device(torch, gemm_once, args.steps, args.warmup, flush, world)
    clocks = sampler.summary()
    ms = gemm_ms_total / args.steps
    value = world * flops / (ms * 1e-3) / 1e12
    achieved = flops / (ms * 1e-3) / 1e12
    traffic = profiled_traffic(f"gemm_square_{size}")

    line = {
        "metric": "nvfp4_gemm_tflops", "value": value, "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "e2m1/ue4m3->f32",
        "data": "synthetic",
        "config": square_config(size, world),
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": NOMINAL_FP4_TFLOPS,
                     "unit": "TFLOP/s", "frac": achieved / NOMINAL_FP4_TFLOPS, "traffic": traffic,
                     "peak_source": "B200 dense FP4 tensor peak, 9.0 PFLOP/s (nominal; "
                                    "MEASURED_PEAKS.json holds no FP4 figure)",
                     "peak_4x_measured_bf16": fp4_peak_bf16,
                     "frac_of_4x_measured_bf16": achieved / fp4_peak_bf16,
                     "peak_4x_measured_bf16_source": f"4 x {peak_src} cuBLAS bf16 burst "
                                                     f"({bf16_tf:.1f} TF/s)",
                     "kernel": "nvfp4::gemm::gemm_kernel (tcgen05 mxf4nvf4)"},
        "gpu_launches": args.steps,
        "clocks": clocks,
    }

    # ---- the sharded workloads at this N (prefill and decode, weight sharded along N); measured
    # right after the headline, before the host-copy and quantize sections
    if not args.no_sharded and size == 8192:
        summary, n_launch = sharded_summary(torch, plugins, capi, world, rank, args.steps,
                                            args.warmup, flush, stream_h, hbm_gbs)
        line.update(summary)
        line["gpu_launches"] += n_launch

    # ---- quantize / dequantize (8192x8192 activation with 0.5% x50 outliers, seed 1)
    if not args.no_quant and size == 8192:
        g = torch.Generator(device="cuda").manual_seed(1)
        X = torch.randn(8192, 8192, device="cuda", generator=g)
        idx = torch.randperm(X.numel(), device="cuda", generator=g)[: int(0.005 * X.numel())]
        X.view(-1)[idx] *= 50.0
        X = X.to(torch.bfloat16)
        sX = (6 * 448 / X.abs().max().to(torch.float32)).reshape(())
        # Four sets of buffers used in rotation (1.3 GB together): no call finds its input in L2
        # from the call before it, as one set re-read back to back partly would.
        n_sets = 4
        Xs = [X] + [X.clone() for _ in range(n_sets - 1)]
        qs = [torch.empty(8192, 4096, dtype=torch.uint8, device="cuda") for _ in range(n_sets)]
        qsfs = [torch.empty(8192, 512, dtype=torch.uint8, device="cuda") for _ in range(n_sets)]
        ys = [torch.empty_like(X) for _ in range(n_sets)]
        for i in range(n_sets):
            capi.check(capi.quantize(Xs[i].data_ptr(), sX.data_ptr(), X.numel(), qs[i].data_ptr(),
                                     qsfs[i].data_ptr(), stream_h), "nvfp4_quantize")
        turn = [0]

        def next_set():
            turn[0] = (turn[0] + 1) % n_sets
            return Xs[turn[0]], qs[turn[0]], qsfs[turn[0]], ys[turn[0]]

        def quant_once():
            x, q, qsf, _ = next_set()
            capi.check(capi.quantize(x.data_ptr(), sX.data_ptr(), x.numel(), q.data_ptr(),
                                     qsf.data_ptr(), stream_h), "nvfp4_quantize")

        def dequant_once():
            _, q, qsf, y = next_set()
            capi.check(capi.dequantize(q.data_ptr(), sX.data_ptr(), qsf.data_ptr(), q.numel(),
                                       y.data_ptr(), stream_h), "nvfp4_dequantize")

        ws_bytes = capi.quantize_auto_scale_workspace_bytes(X.numel())
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
        s_out = torch.empty((), dtype=torch.float32, device="cuda")

        def quant_auto_once():
            x, q, qsf, _ = next_set()
            capi.check(capi.quantize_auto_scale(x.data_ptr(), x.numel(), q.data_ptr(),
                                                qsf.data_ptr(), s_out.data_ptr(), ws.data_ptr(),
                                                ws_bytes, stream_h), "nvfp4_quantize_auto_scale")

        def torch_recipe_then_quant():
            x, q, qsf, _ = next_set()
            s_t = 6 * 448 / x.abs().max().to(torch.float32)
            capi.check(capi.quantize(x.data_ptr(), s_t.data_ptr(), x.numel(), q.data_ptr(),
                                     qsf.data_ptr(), stream_h), "nvfp4_quantize")

        for name, fn in (("quantize", quant_once), ("dequantize", dequant_once),
                         ("quantize_auto_scale", quant_auto_once),
                         ("torch_amax_recipe_then_quantize", torch_recipe_then_quant)):
            t = time_device_streaming(torch, fn, args.steps, args.warmup, world) / args.steps
            gbs = QUANT_BYTES / (t * 1e-3) / 1e9
            line[name] = {"value": world * gbs, "unit": "GB/s", "ms_per_call": t,
                          "workload": "8192x8192 bf16, 0.5% x50 outliers, seed 1",
                          "timing": "back-to-back launches over 4 buffer sets in rotation "
                                    "(164 MB touched per call, 1.3 GB in all)",
                          "roofline": {"bound": "hbm", "achieved": gbs, "peak": hbm_gbs,
                                       "unit": "GB/s", "frac": gbs / hbm_gbs,
                                       "traffic": profiled_traffic(f"{name}_8192"),
                                       "peak_source": f"{peak_src} copy bandwidth"}}
            line[name]["note"] = {
                "quantize_auto_scale": "device amax pass (forward) + finalize + quantize (reverse, "
                                       "L2 reuse); GB/s counts the one-pass algorithmic bytes",
                "torch_amax_recipe_then_quantize": "torch abs().max(), 2688*reciprocal, then the "
                                                   "quantize kernel with the device scale (no .item())",
            }.get(name, "")
            line["gpu_launches"] += args.steps * (3 if name == "quantize_auto_scale" else 1)
        del X, Xs, ys, qs, qsfs

    # ---- NVFP4 output straight from the GEMM epilogue vs GEMM, then quantize of bf16 D
    if not args.no_quant:
        gemm_once()
        s_d = (6 * 448 / d.abs().max().to(torch.float32)).reshape(())
        qd = torch.empty(M, N // 2, dtype=torch.uint8, device="cuda")
        qd_sf = torch.empty(M, N // 16, dtype=torch.uint8, device="cuda")

        def gemm_quantized_once():
            capi.check(capi.gemm_quantized(a.data_ptr(), b.data_ptr(), a_sf.data_ptr(),
                                           b_sf.data_ptr(), scale.data_ptr(), s_d.data_ptr(),
                                           qd.data_ptr(), qd_sf.data_ptr(), M, N, K, stream_h),
                       "nvfp4_gemm_quantized")

        def gemm_then_quantize():
            gemm_once()
            capi.check(capi.quantize(d.data_ptr(), s_d.data_ptr(), d.numel(), qd.data_ptr(),
                                     qd_sf.data_ptr(), stream_h), "nvfp4_quantize")

        n_q = max(3, min(args.steps, 100))
        t_fused = time_device(torch, gemm_quantized_once, n_q, args.warmup, flush, world) / n_q
        t_split = time_device(torch, gemm_then_quantize, n_q, args.warmup, flush, world) / n_q
        line["gemm_quantized_output"] = {
            "value": world * flops / (t_fused * 1e-3) / 1e12, "unit": "TFLOP/s",
            "ms_per_call": t_fused, "gemm_then_quantize_ms": t_split, "steps": n_q,
            "api": "nvfp4_gemm_quantized: NVFP4 D (bytes of quantize(bf16 D, s_out)) from the "
                   "epilogue; compared with nvfp4_gemm + nvfp4_quantize of the bf16 D"}
        line["gpu_launches"] += n_q * 3
        del qd, qd_sf

    # ---- end to end through the torch module with pinned host buffers
    if not args.no_e2e:
        # Every step uploads its operands from pinned host memory, calls the public API and
        # downloads D. Consecutive steps run on two streams with their own device and host
        # buffers, so one step's D download overlaps the next step's upload and GEMM (PCIe is
        # full duplex); the timed region spans all steps' copies and GEMMs.
        ha = a.cpu().pin_memory()
        hb = b.cpu().pin_memory()
        hasf = a_sf.cpu().pin_memory()
        hbsf = b_sf.cpu().pin_memory()
        scale_h = scale.cpu()
        streams = [torch.cuda.Stream() for _ in range(2)]
        bufs = [dict(a=torch.empty_like(a), b=torch.empty_like(b), asf=torch.empty_like(a_sf),
                     bsf=torch.empty_like(b_sf),
                     hd=torch.empty(M, N, dtype=torch.bfloat16).pin_memory()) for _ in range(2)]

        def e2e_step(i):
            st_, bf = streams[i % 2], bufs[i % 2]
            with torch.cuda.stream(st_):
                bf["a"].copy_(ha, non_blocking=True)
                bf["b"].copy_(hb, non_blocking=True)
                bf["asf"].copy_(hasf, non_blocking=True)
                bf["bsf"].copy_(hbsf, non_blocking=True)
                out = plugins.gemm_nvfp4(bf["a"], bf["b"], bf["asf"], bf["bsf"], scale_h)
                bf["hd"].copy_(out, non_blocking=True)
                out.record_stream(st_)

        e2e_steps = max(4, min(args.steps, 20))
        main = torch.cuda.current_stream()
        for i in range(2):
            e2e_step(i)
        torch.cuda.synchronize()
        if world > 1:
            import torch.distributed as dist
            dist.barrier()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record(main)
        for st_ in streams:
            st_.wait_event(ev0)
        for i in range(e2e_steps):
            e2e_step(i)
        for st_ in streams:
            main.wait_stream(st_)
        ev1.record(main)
        torch.cuda.synchronize()
        t = ev0.elapsed_time(ev1) / e2e_steps
        if world > 1:
            tt = torch.tensor([t], device="cuda")
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            t = float(tt.item())
        h2d = sum(t_.numel() * t_.element_size() for t_ in (ha, hb, hasf, hbsf))
        line["e2e"] = {"value": world * flops / (t * 1e-3) / 1e12, "unit": "TFLOP/s",
                       "ms_per_step": t, "steps": e2e_steps, "h2d_bytes_per_step": h2d,
                       "d2h_bytes_per_step": M * N * 2,
                       "api": "my_plugins.gemm_nvfp4, pinned host operands in, bf16 D out; "
                              "consecutive steps on two streams (copies overlap across steps)"}
        line["gpu_launches"] += e2e_steps

    # ---- CPU baseline (rank 0, N = 1 only)
    if world == 1 and rank == 0 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline_gemm(a, b, a_sf, b_sf, scale)

    st = capi.device_status(stream_h)
    if st != 0:
        line["device_status"] = capi.STATUS_NAMES.get(st, st)
    if rank == 0:
        emit(line)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()
    return 0


def sharded_inputs(torch, plugins, workload, m, world, rank, swiglu=False, keep_bf16=False):
    """Operands of the sharded workloads, drawn on the GPU.

    prefill: A 16384 x 8192 bf16 N(0,1) with 0.5% of the elements x50 (seed 4), weight
             57344 x 8192 N(0, 0.02^2) (seed 1004);
    decode:  A m x 8192 N(0,1) (seed 3), weight 28672 x 8192 N(0, 0.02^2) (seed 1003).
    The weight's global scale is taken over the whole weight; this rank quantizes its column
    shard (rows [n0, n1) of the weight). With swiglu the weight is gate+up (rows [gate; up]),
    interleaved in groups of 128 rows before sharding into whole 256-row groups."""
    from my_nvfp4_gemm_b200 import sharded
    K = 8192
    if workload == "decode":
        M, N, seed, frac, name = m, 28672, 3, 0.0, f"decode_m{m}_n28672_k8192"
    else:
        M, N, seed, frac, name = 16384, 57344, 4, 0.005, "prefill_16384x57344x8192"
    n0, n1 = sharded.shard_range(N, world, rank, align=256 if swiglu else 128)
    g = torch.Generator(device="cuda").manual_seed(seed)
    X = torch.randn(M, K, device="cuda", generator=g)
    if frac:
        idx = torch.randperm(X.numel(), device="cuda", generator=g)[: int(frac * X.numel())]
        X.view(-1)[idx] *= 50.0
    X = X.to(torch.bfloat16)
    sX = (6 * 448 / X.abs().max().to(torch.float32)).reshape(())
    x, x_sf = plugins.quantize_nvfp4(X, sX)
    gw = torch.Generator(device="cuda").manual_seed(seed + 1000)
    W = (torch.randn(N, K, device="cuda", generator=gw) * 0.02).to(torch.bfloat16)
    sW = (6 * 448 / W.abs().max().to(torch.float32)).reshape(())
    if swiglu:
        from my_nvfp4_gemm_b200.swiglu import interleave_gate_up
        half = N // 2
        wq, wq_sf = plugins.quantize_nvfp4(W, sW)          # rows [gate; up]
        wi = interleave_gate_up(wq[:half], wq[half:])
        wi_sf = interleave_gate_up(wq_sf[:half].view(torch.uint8), wq_sf[half:].view(torch.uint8))
        w, w_sf = wi[n0:n1].contiguous(), wi_sf[n0:n1].contiguous().view(torch.float8_e4m3fn)
        del wq, wq_sf, wi, wi_sf
    else:
        w, w_sf = plugins.quantize_nvfp4(W[n0:n1].contiguous(), sW)
    out = dict(x=x, x_sf=x_sf, w=w, w_sf=w_sf, scale=(sX * sW).reshape(()), sX=sX, sW=sW,
               M=M, N=N, K=K, n0=n0, n1=n1, n_loc=n1 - n0, name=name)
    if keep_bf16:
        out.update(X=X, W=W)
    else:
        del X, W
        torch.cuda.empty_cache()
    return out


def sharded_step(torch, capi, sharded, inp, mode, stream_h):
    """One step of a sharded workload on this rank. mode: "gemm" (this rank's shard of D),
    "fused" (GEMM with the all-gather fused into the epilogue), "nccl" (GEMM per chunk of rows,
    each chunk's NCCL all-gather overlapping the next chunk), "swiglu" (gate+up GEMM with
    SwiGLU in the epilogue), "rotate" (decode: consecutive calls read copies of the weight in
    rotation, together > 3 x L2, as the layers of a decode step stream different weights)."""
    x, x_sf, w, w_sf, scale = inp["x"], inp["x_sf"], inp["w"], inp["w_sf"], inp["scale"]
    M, K, n_loc = inp["M"], inp["K"], inp["n_loc"]
    if mode == "fused" or mode == "nccl":
        def step():
            sharded.gemm_column_parallel(x, w, x_sf, w_sf, scale, gather=True, chunks=4,
                                         fused=(mode == "fused"))
        return step
    if mode == "swiglu":
        out = torch.empty(M, n_loc // 2, dtype=torch.bfloat16, device="cuda")

        def step():
            capi.check(capi.gemm_swiglu(x.data_ptr(), w.data_ptr(), x_sf.data_ptr(), w_sf.data_ptr(),
                                        scale.data_ptr(), out.data_ptr(), M, n_loc, K, stream_h),
                       "nvfp4_gemm_swiglu")
        return step
    d = torch.empty(M, n_loc, dtype=torch.bfloat16, device="cuda")
    weights = [(w, w_sf)]
    if mode == "rotate":
        per_copy = w.numel() + w_sf.numel()
        n_copies = max(2, -(-3 * (126 << 20) // per_copy))
        weights += [(w.clone(), w_sf.clone()) for _ in range(n_copies - 1)]
        inp["n_copies"] = n_copies
    turn = [0]

    def step(stream=None):
        wc, wc_sf = weights[turn[0]]
        turn[0] = (turn[0] + 1) % len(weights)
        capi.check(capi.gemm(x.data_ptr(), wc.data_ptr(), x_sf.data_ptr(), wc_sf.data_ptr(),
                             scale.data_ptr(), d.data_ptr(), M, n_loc, K,
                             stream_h if stream is None else stream), "nvfp4_gemm")
    return step


def time_sharded(torch, step, mode, steps, warmup, flush, world):
    """ms per step, max over ranks: decode rotation back to back, the rest L2-flushed."""
    if mode == "rotate":
        return time_device_streaming(torch, step, steps, warmup, world) / steps
    return time_device(torch, step, steps, warmup, flush, world) / steps


def sharded_roofline(inp, ms, world, hbm_gbs, gather=False):
    """Per-rank roofline of a sharded step: FP4 tensor peak (prefill), HBM (decode), and with a
    gather the slower of the tensor bound and this rank's output bytes over NVLink."""
    M, K, n_loc = inp["M"], inp["K"], inp["n_loc"]
    flops_rank = 2.0 * M * n_loc * K
    bytes_rank = n_loc * K * (0.5 + 1 / 16) + M * K * (0.5 + 1 / 16) + 2.0 * M * n_loc
    tf = flops_rank / (ms * 1e-3) / 1e12
    gbs = bytes_rank / (ms * 1e-3) / 1e9
    r = {"achieved_tflops_per_rank": tf, "frac_fp4_peak_per_rank": tf / NOMINAL_FP4_TFLOPS,
         "achieved_gbs_per_rank": gbs, "frac_hbm_per_rank": gbs / hbm_gbs,
         "algorithmic_bytes_per_rank": bytes_rank}
    if gather:
        nvlink_bytes = 2.0 * M * n_loc * (world - 1)
        bound_ms = max(flops_rank / (NOMINAL_FP4_TFLOPS * 1e12), nvlink_bytes / (NVLINK_GBS * 1e9)) * 1e3
        r.update(nvlink_bytes_out_per_rank=nvlink_bytes, bound_ms=bound_ms, frac_of_bound=bound_ms / ms)
    return r


def sharded_summary(torch, plugins, capi, world, rank, steps, warmup, flush, stream_h, hbm_gbs):
    """The `prefill` and `decode` keys of the square line: the sharded workloads at this N.
    Decode runs first, after a short pause: right after seconds of power-capped GEMM (the
    headline, and on one GPU the 15-PFLOP prefill steps) the clocks recover over a few tens of
    milliseconds, and the ~10 ms decode rotation measured in that window ran ~20 % slow."""
    import time
    from my_nvfp4_gemm_b200 import sharded
    out, launches = {}, 0
    torch.cuda.synchronize()
    time.sleep(0.25)
    dec = {"workload": "decode_m{16,128}_n28672_k8192", "scaling": "strong",
           "l2": "weight copies (> 3 x L2 together) in rotation, calls back to back"}
    # decode calls take ~8-30 us: a fixed 300 back-to-back calls after 30 untimed ones (~10 ms)
    n_d, w_d = 300, 30
    for m in (16, 128):
        inp = sharded_inputs(torch, plugins, "decode", m, world, rank)
        step = sharded_step(torch, capi, sharded, inp, "rotate", stream_h)
        ms = time_sharded(torch, step, "rotate", n_d, w_d, flush, world)
        # the same rotation captured into a CUDA graph (as a serving loop would run a decode step)
        ms_g = time_graph_streaming(torch, step, 100, 5, world)
        dec[f"m{m}"] = {"us_per_step": ms * 1e3, "n_per_rank": inp["n_loc"], "steps": n_d,
                        "warmup": w_d, "roofline": sharded_roofline(inp, ms, world, hbm_gbs),
                        "graph_us_per_step": ms_g * 1e3,
                        "graph": "100 calls captured once, 5 replays timed after 1"}
        launches += n_d + w_d + 100 * 6
        del inp
        torch.cuda.empty_cache()
    out["decode"] = dec
    inp = sharded_inputs(torch, plugins, "prefill", 0, world, rank)
    n_p = max(3, min(steps, 20))
    pre = {"workload": inp["name"], "n_per_rank": inp["n_loc"], "steps": n_p,
           "scaling": "strong", "l2": "flushed (256 MiB write) before every timed step"}
    modes = ["gemm"] + (["fused", "nccl"] if world > 1 else [])
    for mode in modes:
        ms = time_sharded(torch, sharded_step(torch, capi, sharded, inp, mode, stream_h), mode,
                          n_p, warmup, flush, world)
        key = {"gemm": "gemm_only", "fused": "fused_all_gather", "nccl": "nccl_all_gather"}[mode]
        pre[key] = {"ms_per_step": ms,
                    "value": 2.0 * inp["M"] * inp["N"] * inp["K"] / (ms * 1e-3) / 1e12,
                    "unit": "TFLOP/s",
                    "roofline": sharded_roofline(inp, ms, world, hbm_gbs, gather=mode != "gemm")}
        launches += (n_p + warmup) * (4 if mode == "nccl" else 1)
    if world > 1:
        sharded.release_peer_outputs()
    out["prefill"] = pre
    del inp
    torch.cuda.empty_cache()
    return out, launches


def run_sharded_workload(args):
    """decode / prefill: a fixed global problem (strong scaling) whose weight is sharded
    column-parallel across the ranks; A is replicated. Optionally times the chunked NCCL
    all-gather of D (or the all-gather fused into the GEMM's epilogue) with the GEMM."""
    import torch
    from my_nvfp4_gemm_b200 import capi, load_my_plugins, sharded
    plugins = load_my_plugins()
    world, rank, local = dist_setup(torch)
    swiglu = bool(args.swiglu and args.workload == "prefill")
    if swiglu and args.gather:
        raise SystemExit("--swiglu and --gather are separate measurements")
    shard_of = args.shard_of
    if shard_of > 1 and (world > 1 or args.gather):
        raise SystemExit("--shard-of times one rank's shard alone on one GPU (no gather)")
    inp = sharded_inputs(torch, plugins, args.workload, args.m, max(world, shard_of), rank,
                         swiglu=swiglu)
    M, N, K, n_loc = inp["M"], inp["N"], inp["K"], inp["n_loc"]
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device="cuda")
    stream_h = torch.cuda.current_stream().cuda_stream
    fused = bool(args.gather and args.fused_gather and world > 1)
    if swiglu:
        mode = "swiglu"
    elif args.gather and world > 1:
        mode = "fused" if fused else "nccl"
    elif args.workload == "decode":
        mode = "rotate"
    else:
        mode = "gemm"
    step = sharded_step(torch, capi, sharded, inp, mode, stream_h)

    hbm_gbs, bf16_tf, peak_src = measured_peaks()
    sampler = ClockSampler(gpu_uuid(torch, torch.cuda.current_device()))
    with sampler:
        ms = time_sharded(torch, step, mode, args.steps, args.warmup, flush, world)
    flops = 2.0 * M * (n_loc if shard_of > 1 else N) * K
    rl = sharded_roofline(inp, ms, world, hbm_gbs, gather=mode in ("fused", "nccl"))
    decode = M <= 128
    line = {
        "metric": "nvfp4_gemm_tflops", "value": flops / (ms * 1e-3) / 1e12, "unit": "TFLOP/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "e2m1/ue4m3->f32", "data": "synthetic",
        "config": {"workload": inp["name"] + (f"_shard0of{shard_of}" if shard_of > 1 else ""), "M": M, "N": N, "K": K, "n_per_rank": n_loc,
                   "parallelism": (f"rank 0's shard of column-parallel N x{shard_of}, alone on one "
                                   "GPU" if shard_of > 1 else f"column-parallel N x{world}"),
                   "all_gather_in_timing": mode in ("fused", "nccl"),
                   "epilogue": ("SwiGLU (gate+up interleaved in 128-row groups), output "
                                f"[M, {N // 2}]" if swiglu else "bf16 D"),
                   "all_gather": ("fused into the GEMM epilogue (NVLink stores)" if mode == "fused"
                                  else "NCCL all_gather_into_tensor, 4 chunks" if mode == "nccl"
                                  else None),
                   "l2": (f"{inp.get('n_copies')} copies of the weight shard in rotation, calls "
                          "back to back: every call reads its weight from HBM" if mode == "rotate"
                          else "flushed (256 MiB write) before every timed step")},
        "roofline": dict({"bound": "hbm" if decode else "tensor",
                          "achieved": rl["achieved_gbs_per_rank"] if decode else rl["achieved_tflops_per_rank"],
                          "peak": hbm_gbs if decode else NOMINAL_FP4_TFLOPS,
                          "unit": "GB/s" if decode else "TFLOP/s",
                          "frac": rl["frac_hbm_per_rank"] if decode else rl["frac_fp4_peak_per_rank"],
                          "traffic": (profiled_traffic(f"gemm_decode_m{M}" + (
                                          f"_shard0of{shard_of}" if shard_of > 1 else ""))
                                      if args.workload == "decode" and world == 1 else None),
                          "peak_source": f"{peak_src} HBM {hbm_gbs} GB/s; FP4 dense 9.0 PFLOP/s "
                                         "(nominal)"}, **rl),
        "gpu_launches": args.steps * (4 if mode == "nccl" else 1),
        "clocks": sampler.summary(),
    }
    if mode == "rotate":
        # the same rotation captured into a CUDA graph: the per-call device time without the
        # host's launch overhead
        line["graph_us_per_step"] = time_graph_streaming(torch, step, 100, 5, world) * 1e3
        line["gpu_launches"] += 100 * 6
    if swiglu and world == 1:
        # the unfused equivalent: bf16 D of the gate+up GEMM, then torch silu(g) * u
        import torch.nn.functional as F
        x, x_sf, w, w_sf, scale = inp["x"], inp["x_sf"], inp["w"], inp["w_sf"], inp["scale"]
        d_full = torch.empty(M, n_loc, dtype=torch.bfloat16, device="cuda")
        half = n_loc // 2

        def unfused():
            capi.check(capi.gemm(x.data_ptr(), w.data_ptr(), x_sf.data_ptr(), w_sf.data_ptr(),
                                 scale.data_ptr(), d_full.data_ptr(), M, n_loc, K, stream_h),
                       "nvfp4_gemm")
            (F.silu(d_full[:, :half].float()) * d_full[:, half:].float()).to(torch.bfloat16)

        n_u = max(3, min(args.steps, 10))
        line["gemm_then_torch_silu_mul_ms"] = time_device(torch, unfused, n_u, args.warmup, flush,
                                                          world) / n_u
        del d_full
    if rank == 0:
        emit(line)
    if world > 1:
        import torch.distributed as dist
        sharded.release_peer_outputs()
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main():
    args = parse_args()
    keep_stdout_for_result()
    if args.impl == "reference":
        return run_reference_arm(args)
    if args.workload != "square":
        return run_sharded_workload(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
