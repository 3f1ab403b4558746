"""Benchmark of the FP16 GEMM hot path on B200 (one process per GPU).

Workload (the reference's 1-8 GPU configuration): C = A @ B with M = 65536, N = K = 8192, A and B
iid N(0, 0.02) fp16, A row-sharded over the N GPUs, B replicated; fp32
accumulation, fp16 output.  One step = one pass of the GEMM over this rank's
shard (strong scaling: total work fixed).  The inputs (A shard >= 128 MiB +
B 128 MiB per GPU) exceed the 126 MB L2, so no flush is needed between steps.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

Prints ONE JSON line on rank 0.  `value` is the whole-job TFLOP/s from CUDA
events (max over ranks); `e2e` times the public API with the operands in
pinned host memory (H2D of A shard + B, GEMM, D2H of C inside the timed
region).  At N=1 rank 0 also reports the skinny K=256 shape's HBM bandwidth
(against the copy rate and the read-only / write-only rates), the 8192^3
shapes in both B layouts, torch.mm on the same box, the fused K-means
assignment, and the reference's CPU path timed on a bounded sample.  At N>1
it adds the gathered-output comparison (full C on every rank: GEMM + NCCL
all-gather against the fused peer-store GEMM).  Only the result line goes to
stdout.

`--impl reference` runs the unmodified reference package (installed under
baseline/_ref) through its public `tensorcore_gemm.gemm` on CPU tensors: its
CPU path, `torch.matmul` in fp16 (tensorcore_gemm/gemm.py:219-221), timed on
a bounded row slice of the same workload.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
PKG_DIR = REPO / "ampere-gemm_b200"
REF_DIR = REPO / "baseline" / "_ref"

M_TOTAL, N_DIM, K_DIM = 65536, 8192, 8192
STD = 0.02
SKINNY = (32768, 1024, 256)
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--no-extras", action="store_true", help="skip the N=1 side measurements")
    ap.add_argument("--case", default=None,
                    help="single-GEMM mode for profiling/tuning: MxNxK[:colb] (1 GPU, not the driver line)")
    ap.add_argument("--variant", default="auto",
                    choices=["auto", "cta1", "pair", "skinny", "pair2m", "pair2m_224", "pair2m_192", "torch", "kmeans"],
                    help="kernel for --case (torch = torch.mm comparator; kmeans = fused K-means "
                         "assignment of M points to N centroids, centroids stored N x K)")
    ap.add_argument("--dist", default="uniform", choices=["uniform", "normal"], help="inputs for --case")
    ap.add_argument("--graph", action="store_true", help="--case: time a CUDA-graph replay (device time only)")
    return ap.parse_args()


def load_peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            d = json.loads(p.read_text())
            return d, "measured"
        except Exception:
            pass
    return dict(FALLBACK_PEAKS), "fallback"


def cpu_model() -> str:
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


# ---------------------------------------------------------------------------
# nvidia-smi clock sampling during the timed region
# ---------------------------------------------------------------------------
CLOCK_FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
                "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")


class ClockSampler:
    """nvidia-smi samples every 20 ms; `summary` keeps those taken inside the
    window marked with `mark_start` / `mark_end` (or, for a window shorter than
    the sampling interval, the samples nearest to it)."""

    def __init__(self, gpu_index: int):
        self.gpu_index = gpu_index
        self.proc = None
        self.t0 = self.t1 = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={CLOCK_FIELDS}", "--format=csv,noheader,nounits", "-lms", "20",
                 "-i", str(self.gpu_index)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, FileNotFoundError):
            self.proc = None
        time.sleep(0.3)  # let nvidia-smi start sampling before the timed region
        return self

    def mark_start(self):
        self.t0 = time.time()

    def mark_end(self):
        self.t1 = time.time()
        time.sleep(0.05)

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [l for l in out.splitlines() if l.strip()]
        return False

    def summary(self) -> dict:
        import datetime

        rows = []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in getattr(self, "lines", []):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 10:
                continue
            try:
                ts = datetime.datetime.strptime(parts[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                sm, smax = float(parts[2]), float(parts[3])
            except ValueError:
                continue
            active = {n for n, v in zip(names, parts[6:10]) if v.lower().startswith("active")}
            rows.append((ts, sm, smax, active))
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        if self.t0 is not None and self.t1 is not None:
            inside = [r for r in rows if self.t0 <= r[0] <= self.t1]
            if not inside:  # window shorter than the sampling interval
                inside = sorted(rows, key=lambda r: abs(r[0] - 0.5 * (self.t0 + self.t1)))[:2]
            rows = inside
        reasons = set().union(*(r[3] for r in rows))
        return {"sm_mhz": statistics.median(r[1] for r in rows), "sm_max_mhz": rows[-1][2],
                "reasons": sorted(reasons), "samples": len(rows)}


# ---------------------------------------------------------------------------
# Reference CPU path (bounded samples of the same workload)
# ---------------------------------------------------------------------------
def load_reference_package():
    """The unmodified reference package from baseline/_ref, under its own name."""
    sys.path.insert(0, str(REPO))
    from baseline import reference

    return reference.load_package()


class CpuBaseline:
    """Times the reference's CPU implementation on a row slice of the workload.

    The reference's public gemm() on CPU tensors runs its torch.matmul fp16
    fallback (tensorcore_gemm/gemm.py:219-221).  kind "reference": that call
    made through the unmodified package in baseline/_ref.  kind "port": the
    package is absent, so the same torch.matmul call is made directly.  Both
    use every host thread.  The north star's "fp16 upcast to fp32" variant,
    torch.matmul(A.float(), B.float()), is timed beside it on the same slice.
    """

    def __init__(self, target_s: float = 2.0):
        import torch

        self.torch = torch
        self.cores = os.cpu_count() or 1
        torch.set_num_threads(self.cores)
        self.ref = load_reference_package()
        self.kind = "reference" if self.ref is not None else "port"
        g = torch.Generator().manual_seed(1)
        self.B = (torch.randn((K_DIM, N_DIM), generator=g) * STD).half()
        self.rows = 64
        self.A = self._a(self.rows)
        for _ in range(3):                   # grow the slice until one step takes ~target_s
            t = self.step()
            if t >= 0.6 * target_s or self.rows >= 8192:
                break
            rows = int(self.rows * target_s / max(t, 1e-3))
            self.rows = max(64, min(8192, rows // 64 * 64))
            self.A = self._a(self.rows)

    def _a(self, rows):
        g = self.torch.Generator().manual_seed(0)
        return (self.torch.randn((rows, K_DIM), generator=g) * STD).half()

    def step(self) -> float:
        t0 = time.perf_counter()
        if self.kind == "reference":
            C = self.ref.gemm(self.A, self.B, mode="reg_pingpong_256")
        else:
            C = self.torch.matmul(self.A, self.B)
        assert C.shape[0] == self.rows and C.dtype == self.torch.float16
        return time.perf_counter() - t0

    def step_fp32_upcast(self) -> float:
        t0 = time.perf_counter()
        C = self.torch.matmul(self.A.float(), self.B.float())
        assert C.shape[0] == self.rows
        return time.perf_counter() - t0

    def flops(self) -> float:
        return 2.0 * self.rows * N_DIM * K_DIM

    def sample(self) -> str:
        path = ("reference tensorcore_gemm.gemm on CPU tensors (its torch.matmul fp16 fallback)"
                if self.kind == "reference" else
                "torch.matmul fp16 called directly (the reference's CPU call; baseline/_ref not installed)")
        return (f"{self.rows} x {N_DIM} x {K_DIM} row slice of the {M_TOTAL} x {N_DIM} x {K_DIM} workload; "
                f"{path}; {self.cores} threads; {cpu_model()}")

    def measure(self, reps: int = 3) -> dict:
        t = statistics.median(self.step() for _ in range(reps))
        t32 = statistics.median(self.step_fp32_upcast() for _ in range(max(1, reps - 1)))
        return {"value": round(self.flops() / t / 1e12, 5), "unit": "TFLOP/s", "cores": self.cores,
                "kind": self.kind, "sample": self.sample() + f"; median of {reps}",
                "fp32_upcast_value": round(self.flops() / t32 / 1e12, 5),
                "fp32_upcast_sample": "torch.matmul(A.float(), B.float()) on the same slice and threads"}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0  # the reference is a single-process CPU path: rank 0 alone runs it
    cpu = CpuBaseline(target_s=2.0)
    for _ in range(max(args.warmup, 0)):
        cpu.step()
    times = [cpu.step() for _ in range(args.steps)]
    total = sum(times)
    value = cpu.flops() * args.steps / total / 1e12
    line = {
        "impl": "reference",
        "metric": BASELINE_METRIC, "value": round(value, 5), "unit": "TFLOP/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(total / args.steps * 1e3, 3), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f16 in / f32 accumulate (CPU torch.matmul)",
        "data": "synthetic N(0,0.02) fp16, seeded", "config": workload_config(args.gpus),
        "cpu_baseline": {"value": round(value, 5), "unit": "TFLOP/s", "cores": cpu.cores, "kind": cpu.kind,
                         "sample": cpu.sample(),
                         "fp32_upcast_value": round(cpu.flops() / statistics.median(
                             cpu.step_fp32_upcast() for _ in range(2)) / 1e12, 5)},
        "e2e": {"value": round(value, 5), "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "gpu_launches": 0,
    }
    emit(line)
    return 0


BASELINE_METRIC = "FP16 GEMM TFLOPS/GPU & % dense tensor peak; HBM GB/s at K=256; box TFLOPS 1-8"


def tensor_peak_for_clocks(peaks: dict, src: str, clk: dict) -> dict:
    """Tensor-pipe denominator of the headline kernel.

    The headline GEMM is timed alone, so it is divided by the measured burst
    figure (`bf16_tflops`, cuBLAS at the maximum SM clock), whatever clock the
    timed region ran at: the larger, conservative denominator.  The sustained
    figure (a seconds-long cuBLAS loop under the 1 kW cap, settled to a lower
    median clock) is reported beside it as `frac_of_sustained`, with both
    clocks in `peak_source`, for runs that were power-capped.
    """
    burst = float(peaks["bf16_tflops"])
    sm, smax = clk.get("sm_mhz"), clk.get("sm_max_mhz") or peaks.get("sm_max_mhz")
    note = f"timed region at median {sm:.0f} of {smax:.0f} MHz" if sm and smax else "clocks not sampled"
    settled = (peaks.get("clocks_under_load") or {}).get("sm_mhz_median")
    out = {"peak": burst, "peak_source": f"{src} bf16_tflops (burst; {note}; of {src})"}
    sustained = peaks.get("bf16_tflops_sustained")
    if sustained:
        out["sustained_peak"] = float(sustained)
        out["sustained_source"] = (f"{src} bf16_tflops_sustained (power-capped loop"
                                   + (f" at median {settled:.0f} MHz" if settled else "") + ")")
    return out


def workload_config(n_gpus: int) -> dict:
    return {"workload": f"fp16_gemm_{M_TOTAL}x{N_DIM}x{K_DIM}_A_row_sharded",
            "M": M_TOTAL, "N": N_DIM, "K": K_DIM, "b_layout": "row-major K x N",
            "inputs": "A, B iid N(0, 0.02) fp16", "parallelism": f"A row-sharded over {n_gpus} GPU(s), B replicated",
            "global_batch": M_TOTAL, "l2": "inputs larger than L2 (A shard + B >= 256 MiB per GPU); no flush"}


# ---------------------------------------------------------------------------
# B200 arm
# ---------------------------------------------------------------------------
def _time_graph(torch, fn, iters: int) -> float:
    """Mean ms per call of fn(i), i = 0..iters-1, captured once in a CUDA graph
    and replayed: device time only, no host launch gaps between calls."""
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for i in range(min(iters, 3)):
            fn(i)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for i in range(iters):
            fn(i)
    g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    g.replay()
    e1.record()
    e1.synchronize()
    return e0.elapsed_time(e1) / iters


def _time_launches(torch, fn, iters: int) -> float:
    """Mean ms per call of fn() over `iters` back-to-back calls (CUDA events)."""
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    s.record()
    for i in range(iters):
        fn(i)
    e.record()
    e.synchronize()
    return s.elapsed_time(e) / iters


def read_traffic_per_launch(tag: str):
    """DRAM bytes per full launch recorded from an ncu capture under profiles/."""
    for p in sorted((REPO / "profiles").glob("*.md")):
        for line in p.read_text().splitlines():
            if line.startswith(f"traffic_bytes_per_launch[{tag}]:"):
                try:
                    return int(float(line.split(":", 1)[1].strip().split()[0]))
                except ValueError:
                    return None
    return None


def hbm_direction_peaks(torch, dev) -> dict:
    """Read-only and write-only HBM bandwidth of plain torch kernels (sum and
    fill_ over four rotating 128 MiB buffers, > L2 together, CUDA-graph
    replay): the denominators for traffic that is mostly writes."""
    n = 64 * 1024 * 1024
    src = [torch.randn(n, device=dev).half() for _ in range(4)]
    dst = [torch.empty(n, dtype=torch.float16, device=dev) for _ in range(4)]
    ms_r = _time_graph(torch, lambda i: src[i % 4].sum(dtype=torch.float32), 40)
    ms_w = _time_graph(torch, lambda i: dst[i % 4].fill_(1.0), 40)
    out = {"read_only_GBps": round(2 * n / (ms_r * 1e-3) / 1e9, 1),
           "write_only_GBps": round(2 * n / (ms_w * 1e-3) / 1e9, 1),
           "how": "torch.sum (read) and Tensor.fill_ (write) over 4 rotating 128 MiB fp16 buffers, graph replay"}
    del src, dst
    return out


def side_measurements(torch, tg, dev, peaks) -> dict:
    """N=1 only: skinny K=256 HBM bandwidth (cold L2), 8192^3 both layouts, torch.mm."""
    out = {}
    torch.backends.cuda.matmul.allow_fp16_reduced_precision_reduction = False
    # --- skinny: rotate buffer sets so every launch reads A and writes C from/to HBM
    M, N, K = SKINNY
    set_bytes = 2 * (M * K + K * N + M * N)
    l2 = torch.cuda.get_device_properties(dev).L2_cache_size
    nsets = max(2, -(-2 * l2 // set_bytes))
    g = torch.Generator(device=dev).manual_seed(7)
    sets = [(torch.randn((M, K), generator=g, device=dev, dtype=torch.float16),
             torch.randn((K, N), generator=g, device=dev, dtype=torch.float16),
             torch.empty((M, N), device=dev, dtype=torch.float16)) for _ in range(nsets)]
    bcol = [b.t().contiguous() for _, b, _ in sets]
    row = lambda i: tg.gemm(sets[i % nsets][0], sets[i % nsets][1], out=sets[i % nsets][2])
    col = lambda i: tg.gemm_pretransposed(sets[i % nsets][0], bcol[i % nsets], mode="reg_pingpong_256_colb")
    mm = lambda i: torch.mm(sets[i % nsets][0], sets[i % nsets][1], out=sets[i % nsets][2])
    for f in (row, col, mm):
        for i in range(3 * nsets):
            f(i)
    iters = 40 * nsets
    ms_row = _time_graph(torch, row, iters)
    ms_col = _time_graph(torch, col, iters)
    ms_mm = _time_graph(torch, mm, iters)
    gbs = lambda ms: set_bytes / (ms * 1e-3) / 1e9
    dirs = hbm_direction_peaks(torch, dev)
    read_b, write_b = 2 * (M * K + K * N), 2 * M * N
    bound_us = (read_b / dirs["read_only_GBps"] + write_b / dirs["write_only_GBps"]) / 1e3
    out["skinny_32768x1024x256"] = {
        "cold_l2": f"{nsets} rotating operand sets of {set_bytes / 1e6:.1f} MB (> 2x L2)",
        "timing": "CUDA-graph replay of back-to-back launches (device time, no host gaps)",
        "algorithmic_bytes": set_bytes,
        "rowB_us": round(ms_row * 1e3, 2), "rowB_GBps": round(gbs(ms_row), 1),
        "colb_us": round(ms_col * 1e3, 2), "colb_GBps": round(gbs(ms_col), 1),
        "torch_mm_us": round(ms_mm * 1e3, 2), "torch_mm_GBps": round(gbs(ms_mm), 1),
        "roofline": {"bound": "hbm", "achieved": round(gbs(ms_row), 1), "peak": peaks["hbm_gbs"],
                     "unit": "GB/s", "frac": round(gbs(ms_row) / peaks["hbm_gbs"], 4),
                     "traffic": read_traffic_per_launch("skinny_32768x1024x256")},
        "direction_roofline": {"what": "reads at the read-only rate plus writes at the write-only rate",
                               "read_bytes": read_b, "write_bytes": write_b, **dirs,
                               "bound_us": round(bound_us, 2),
                               "rowB_frac": round(bound_us / (ms_row * 1e3), 4),
                               "colb_frac": round(bound_us / (ms_col * 1e3), 4)},
    }
    del sets, bcol
    out["baseline_configs"] = config_sweep(torch, tg, dev, peaks)
    out["kmeans_assign_262144x1024x256"] = kmeans_measurement(torch, dev, g)
    out["reference_cublas_gemm"] = reference_cublas_measurement(torch, dev)
    return out


# Every single-GPU configuration BASELINE names (configs 1-4): (M, N, K,
# distribution, B layouts timed).  Config 5's one-GPU case is the main line.
BASELINE_SHAPES = [
    (2048, 2048, 2048, "uniform", ("rowB",)),
    (16384, 256, 256, "normal", ("rowB", "colb")),
    (16384, 512, 256, "normal", ("rowB", "colb")),
    (16384, 1024, 256, "normal", ("rowB", "colb")),
    (32768, 256, 256, "normal", ("rowB", "colb")),
    (32768, 512, 256, "normal", ("rowB", "colb")),
    (32768, 1024, 256, "normal", ("rowB", "colb")),
    (4096, 4096, 4096, "uniform", ("rowB", "colb")),
    (8192, 8192, 8192, "uniform", ("rowB", "colb")),
    (4096, 8192, 4096, "uniform", ("rowB",)),
    (8192, 4096, 4096, "uniform", ("rowB",)),
    (4000, 6000, 3000, "uniform", ("rowB",)),
]


def config_sweep(torch, tg, dev, peaks) -> dict:
    """Each BASELINE shape: this library (per B layout) and torch.mm (cuBLAS)
    on the same operands, CUDA-graph replay over rotating operand sets that
    together exceed 2x L2, so every launch reads its operands from HBM."""
    l2 = torch.cuda.get_device_properties(dev).L2_cache_size
    g = torch.Generator(device=dev).manual_seed(11)
    res = {}
    for (M, N, K, dist, layouts) in BASELINE_SHAPES:
        set_bytes = 2 * (M * K + K * N + M * N)
        nsets = max(2, min(16, -(-2 * l2 // set_bytes)))
        mk = ((lambda r, c: (torch.rand((r, c), generator=g, device=dev) * 2 - 1).half()) if dist == "uniform"
              else (lambda r, c: torch.randn((r, c), generator=g, device=dev, dtype=torch.float16)))
        sets = [(mk(M, K), mk(K, N), torch.empty((M, N), device=dev, dtype=torch.float16)) for _ in range(nsets)]
        bcol = [b.t().contiguous() for _, b, _ in sets] if "colb" in layouts else None
        fl = 2.0 * M * N * K
        est_us = max(fl / 1.4e15, set_bytes / 5e12) * 1e6 + 3.0
        iters = nsets * max(1, min(400, int(20000 / est_us)) // nsets)
        fns = {"rowB": lambda i: tg.gemm(sets[i % nsets][0], sets[i % nsets][1], out=sets[i % nsets][2]),
               "torch_mm": lambda i: torch.mm(sets[i % nsets][0], sets[i % nsets][1], out=sets[i % nsets][2])}
        if bcol is not None:
            fns["colb"] = lambda i: tg.gemm(sets[i % nsets][0], bcol[i % nsets].t(), out=sets[i % nsets][2])
        # Short launches are replayed from a CUDA graph (no host gaps), long
        # ones timed back to back; two interleaved rounds, the faster of the
        # two per implementation, so clock drift over the sweep hits every
        # implementation alike.
        graph = est_us < 100.0
        entry = {"operand_sets": nsets, "iters": iters, "dist": dist,
                 "timing": "CUDA-graph replay" if graph else "back-to-back launches",
                 "rounds": "best of 2 rounds in opposite orders, 0.25 s idle before each"}
        best = {}
        names = list(fns)
        for rnd in range(2):
            # The order is reversed in the second round, and every measurement
            # starts after a short idle pause, so that power-cap clock drift over
            # the sweep does not favour whichever implementation runs first.
            for name in (names if rnd == 0 else names[::-1]):
                torch.cuda.synchronize()
                time.sleep(0.25)
                f = fns[name]
                ms = _time_graph(torch, f, iters) if graph else _time_launches(torch, f, iters)
                best[name] = min(best.get(name, ms), ms)
        for name, ms in best.items():
            entry[f"{name}_us"] = round(ms * 1e3, 2)
            entry[f"{name}_TFLOPs"] = round(fl / (ms * 1e-3) / 1e12, 1)
            if K <= 256:
                entry[f"{name}_GBps"] = round(set_bytes / (ms * 1e-3) / 1e9, 1)
        entry["rowB_vs_torch_mm"] = round(entry["torch_mm_us"] / entry["rowB_us"], 4)
        if K <= 256:
            entry["rowB_frac_of_measured_hbm"] = round(entry["rowB_GBps"] / peaks["hbm_gbs"], 4)
        else:
            entry["rowB_frac_of_measured_bf16_burst"] = round(entry["rowB_TFLOPs"] / peaks["bf16_tflops"], 4)
        res[f"{M}x{N}x{K}"] = entry
        del sets, bcol
    torch.cuda.synchronize()
    return res


def reference_cublas_measurement(torch, dev) -> dict:
    """The reference's own cuBLAS mode (tensorcore_gemm/cublas_gemm.py:29-43,
    cublas_gemm.cu:7-62: cublasGemmEx, fp16 I/O, fp32 compute), run from the
    unmodified package in baseline/_ref through its own JIT build
    (cuda_compile.compile_cuda), at 8192^3 and at the main workload's shape,
    timed beside this library's gemm on the same operands (interleaved, so
    both see the same clocks).  It allocates C on every call and launches on
    the legacy default stream, as the reference does; CUDA events on that
    stream, back-to-back calls."""
    sys.path.insert(0, str(REPO))
    from baseline import reference

    try:
        cub = reference.cublas_module()
        if cub is None:
            return {"unavailable": "baseline/_ref not installed"}
        t0 = time.perf_counter()
        cub._get_module()
        build_s = time.perf_counter() - t0
    except Exception as exc:  # noqa: BLE001 - reported in the JSON line
        return {"unavailable": f"reference cublas_gemm build failed: {type(exc).__name__}: {exc}"[:300]}
    out = {"jit_build_s": round(build_s, 1),
           "how": ("reference cublas_gemm.gemm(A, B) from baseline/_ref and this library's gemm on the same "
                   "operands, CUDA events over back-to-back calls; two rounds in opposite orders, 0.25 s "
                   "idle before each measurement, the faster round of each")}
    import tensorcore_gemm as tg

    g = torch.Generator(device=dev).manual_seed(13)
    for (M, N, K, dist, iters) in ((8192, 8192, 8192, "uniform", 20), (M_TOTAL, N_DIM, K_DIM, "normal", 10)):
        mk = ((lambda r, c: (torch.rand((r, c), generator=g, device=dev) * 2 - 1).half()) if dist == "uniform"
              else (lambda r, c: torch.randn((r, c), generator=g, device=dev, dtype=torch.float16) * STD))
        ops = [(mk(M, K), mk(K, N)) for _ in range(2)]
        C = torch.empty((M, N), device=dev, dtype=torch.float16)
        impls = {"reference_cublas": lambda i: cub.gemm(ops[i % 2][0], ops[i % 2][1]),
                 "b200": lambda i: tg.gemm(ops[i % 2][0], ops[i % 2][1], out=C)}
        best = {}
        for rnd in range(2):
            for name in (list(impls) if rnd == 0 else list(impls)[::-1]):
                f = impls[name]
                for i in range(3):
                    f(i)
                torch.cuda.synchronize()
                time.sleep(0.25)
                ms = _time_launches(torch, f, iters)
                best[name] = min(best.get(name, ms), ms)
        tf = {name: 2.0 * M * N * K / (ms * 1e-3) / 1e12 for name, ms in best.items()}
        out[f"{M}x{N}x{K}_TFLOPs"] = round(tf["reference_cublas"], 1)
        out[f"{M}x{N}x{K}_b200_TFLOPs"] = round(tf["b200"], 1)
        out[f"{M}x{N}x{K}_b200_vs_reference_cublas"] = round(tf["b200"] / tf["reference_cublas"], 4)
        del ops, C
        torch.cuda.empty_cache()
    return out


def kmeans_measurement(torch, dev, g) -> dict:
    """Fused K-means assignment (argmin in the skinny GEMM's epilogue) against
    torch.mm + argmin on the same points; two point sets (> L2 together)."""
    from tensorcore_gemm import kmeans

    M, N, K = 262144, 1024, 256
    pts = [torch.randn((M, K), generator=g, device=dev, dtype=torch.float16) for _ in range(2)]
    cent = torch.randn((N, K), generator=g, device=dev, dtype=torch.float16)
    fused = lambda i: kmeans.assign(pts[i % 2], cent)
    cn = cent.float().pow(2).sum(1)
    plain = lambda i: torch.argmin(cn[None, :] - 2 * torch.mm(pts[i % 2], cent.t()).float(), 1)
    agree = bool((fused(0).long() == plain(0)).float().mean().item() > 0.999)
    for f in (fused, plain):
        for i in range(4):
            f(i)
    ms_f = _time_launches(torch, fused, 40)
    ms_p = _time_launches(torch, plain, 10)
    moved = 2 * (M * K + N * K) + 4 * M
    return {"fused_us": round(ms_f * 1e3, 1), "torch_mm_argmin_us": round(ms_p * 1e3, 1),
            "speedup": round(ms_p / ms_f, 2), "fused_GBps": round(moved / (ms_f * 1e-3) / 1e9, 1),
            "algorithmic_bytes": moved, "indices_agree_with_torch": agree,
            "timing": "CUDA events over back-to-back calls through kmeans.assign (norms, argmin GEMM, unpack)"}


def gathered_output_measurement(torch, dist, sharded, A, B, C, dev, world, rank, barrier, max_over_ranks,
                                gemm_ms: float, steps: int = 5) -> dict:
    """Full C on every rank: GEMM then NCCL all-gather, against the fused
    gathered-output GEMM (epilogue peer stores).  Device time, max over ranks."""
    stream = torch.cuda.current_stream(dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def timed(fn):
        fn()
        torch.cuda.synchronize()
        barrier()
        ev0.record(stream)
        for _ in range(steps):
            fn()
        ev1.record(stream)
        ev1.synchronize()
        barrier()
        return max_over_ranks(ev0.elapsed_time(ev1)) / steps

    full_nccl = torch.empty((C.shape[0] * world, C.shape[1]), dtype=C.dtype, device=dev)
    gathered_bytes = 2 * M_TOTAL * N_DIM

    def separate():
        sharded.sharded_gemm(A, B, out=C)
        dist.all_gather_into_tensor(full_nccl, C)

    ms_sep = timed(separate)
    ms_ag = timed(lambda: dist.all_gather_into_tensor(full_nccl, C))
    out = sharded.GatheredOutput(M_TOTAL, N_DIM, device=dev)
    try:
        ms_fused = timed(lambda: out.gemm(A, B))
        same = torch.equal(out.full, full_nccl[:M_TOTAL])
        flag = torch.tensor([0.0 if same else 1.0], device=dev)
        dist.all_reduce(flag)
        match = flag.item() == 0.0
    finally:
        out.close()
    del full_nccl
    link_gbs = gathered_bytes * (world - 1) / world / (ms_ag * 1e-3) / 1e9
    roof_ms = max(gemm_ms, gathered_bytes * (world - 1) / world / (link_gbs * 1e9) * 1e3)
    return {"what": "C (65536 x 8192 fp16) gathered on every rank",
            "gemm_only_ms": round(gemm_ms, 4),
            "gemm_then_nccl_all_gather_ms": round(ms_sep, 4),
            "nccl_all_gather_ms": round(ms_ag, 4),
            "nccl_all_gather_bus_GBps": round(gathered_bytes * (world - 1) / world / (ms_ag * 1e-3) / 1e9, 1),
            "fused_peer_store_ms": round(ms_fused, 4),
            "fused_speedup": round(ms_sep / ms_fused, 3),
            # Target of a fused compute + collective step: the slower of the GEMM
            # and the bytes that must leave each GPU at the link rate measured in
            # this run (the NCCL all-gather's bus bandwidth just above).
            "link_rate_GBps": round(link_gbs, 1),
            "link_rate_source": "nccl_all_gather_bus_GBps of this run",
            "fused_roofline_ms": round(roof_ms, 4),
            "fused_frac_of_roofline": round(roof_ms / ms_fused, 4),
            "nvlink_bytes_out_per_gpu": int(gathered_bytes * (world - 1) // world),
            "bitwise_equal_to_nccl_path": bool(match), "steps": steps}


def run_b200(args) -> int:
    sys.path.insert(0, str(PKG_DIR))
    import torch
    import torch.distributed as dist

    import tensorcore_gemm as tg
    from tensorcore_gemm import _native, sharded
    from tensorcore_gemm.streamed import gemm_streamed

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        print(f"warning: --gpus {args.gpus} but WORLD_SIZE {world}", file=sys.stderr)
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)
    peaks, peaks_src = load_peaks()
    _native.load()

    lo, hi = sharded.row_shard_bounds(M_TOTAL, world, rank)
    m = hi - lo
    gA = torch.Generator(device=dev).manual_seed(1000 + rank)
    gB = torch.Generator(device=dev).manual_seed(1)
    A = torch.randn((m, K_DIM), generator=gA, device=dev, dtype=torch.float16) * STD
    B = torch.randn((K_DIM, N_DIM), generator=gB, device=dev, dtype=torch.float16) * STD
    C = torch.empty((m, N_DIM), device=dev, dtype=torch.float16)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    step = lambda: sharded.sharded_gemm(A, B, out=C)
    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    if _native.last_device_error() != 0:
        raise RuntimeError("device error word set during warm-up")

    stream = torch.cuda.current_stream(dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clocks:
        barrier()
        torch.cuda.synchronize()
        clocks.mark_start()
        ev0.record(stream)
        for _ in range(args.steps):
            step()
        ev1.record(stream)
        ev1.synchronize()
        clocks.mark_end()
    torch.cuda.synchronize()
    barrier()
    ms_local = ev0.elapsed_time(ev1)
    ms_max = max_over_ranks(ms_local)
    dev_err = _native.last_device_error()
    total_flops = 2.0 * M_TOTAL * N_DIM * K_DIM * args.steps
    value = total_flops / (ms_max * 1e-3) / 1e12
    launch_ms = ms_local / args.steps
    achieved = 2.0 * m * N_DIM * K_DIM / (launch_ms * 1e-3) / 1e12

    # ---- end to end through the public API with host buffers
    e2e_steps = max(1, min(args.steps, 5))
    A_h = A.cpu().pin_memory()
    B_h = B.cpu().pin_memory()
    C_h = torch.empty((m, N_DIM), dtype=torch.float16).pin_memory()

    def e2e_step():
        # Public host-operand API: A and B copied in, C copied out, in
        # row chunks pipelined over three streams.
        gemm_streamed(A_h, B_h, out=C_h)

    e2e_step()
    torch.cuda.synchronize()
    barrier()
    ev0.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    ev1.record(stream)
    ev1.synchronize()
    barrier()
    e2e_ms = max_over_ranks(ev0.elapsed_time(ev1))
    e2e_value = 2.0 * M_TOTAL * N_DIM * K_DIM * e2e_steps / (e2e_ms * 1e-3) / 1e12

    gathered = None
    if world > 1 and not args.no_extras:
        # A side measurement: whatever goes wrong here must not cost the main
        # line.  Every rank agrees on success before the result is used.
        try:
            gathered = gathered_output_measurement(torch, dist, sharded, A, B, C, dev, world, rank, barrier,
                                                   max_over_ranks, ms_max / args.steps)
            err = None
        except Exception as exc:  # noqa: BLE001 - reported in the JSON line
            err = f"{type(exc).__name__}: {exc}"[:300]
        bad = torch.tensor([1.0 if err else 0.0], device=dev)
        dist.all_reduce(bad)
        if bad.item() > 0:
            gathered = {"unavailable": err or "failed on another rank"}
        torch.cuda.synchronize()

    extras = None
    cpu = None
    if rank == 0 and world == 1 and not args.no_extras:
        del A_h, B_h, C_h
        extras = side_measurements(torch, tg, dev, peaks)
        cpu = CpuBaseline(target_s=3.0).measure(reps=3)

    if rank == 0:
        clk = clocks.summary()
        rl_peak = tensor_peak_for_clocks(peaks, peaks_src, clk)
        line = {
            "metric": BASELINE_METRIC, "value": round(value, 2), "unit": "TFLOP/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms_max / args.steps, 4), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f16 in / f32 accumulate / f16 out",
            "data": "synthetic N(0,0.02) fp16, seeded on device", "config": workload_config(world),
            "tflops_per_gpu": round(value / world, 2),
            "roofline": {"bound": "tensor", "achieved": round(achieved, 2),
                         **rl_peak, "frac": round(achieved / rl_peak["peak"], 4),
                         **({"frac_of_sustained": round(achieved / rl_peak["sustained_peak"], 4)}
                            if "sustained_peak" in rl_peak else {}),
                         "traffic": read_traffic_per_launch(f"shard_{m}x{N_DIM}x{K_DIM}")},
            "pct_nominal_dense_fp16_peak": round(100 * value / world / 2250.0, 2),
            "e2e": {"value": round(e2e_value, 2), "unit": "TFLOP/s",
                    "h2d_bytes_per_step": int(2 * (m * K_DIM + K_DIM * N_DIM)),
                    "d2h_bytes_per_step": int(2 * m * N_DIM), "steps": e2e_steps,
                    "api": "tensorcore_gemm.streamed.gemm_streamed (pinned host A, B, C; row chunks over 3 streams)"},
            "gpu_launches": args.steps,
            "clocks": {"sm_mhz": clk["sm_mhz"], "sm_max_mhz": clk["sm_max_mhz"], "reasons": clk["reasons"],
                       "samples": clk["samples"]},
            "device_error_word": dev_err,
        }
        if cpu is not None:
            line["cpu_baseline"] = cpu
        if extras is not None:
            line["extras"] = extras
        if gathered is not None:
            line["gathered_output"] = gathered
        emit(line)
    if world > 1:
        dist.destroy_process_group()
    return 0


def run_case(args) -> int:
    """One GEMM shape: W warm-up + K timed launches over rotating operand sets
    (at least 2x L2 in total, so every launch streams from HBM); one JSON line."""
    sys.path.insert(0, str(PKG_DIR))
    import torch

    import tensorcore_gemm as tg
    from tensorcore_gemm import _native

    shape, _, layout = args.case.partition(":")
    M, N, K = (int(x) for x in shape.lower().split("x"))
    colb = layout == "colb"
    dev = torch.device("cuda", 0)
    if args.variant == "kmeans":
        return run_kmeans_case(args, torch, M, N, K, dev)
    if args.variant != "torch":
        _native.set_variant(args.variant)
    torch.backends.cuda.matmul.allow_fp16_reduced_precision_reduction = False
    set_bytes = 2 * (M * K + K * N + M * N)
    l2 = torch.cuda.get_device_properties(dev).L2_cache_size
    nsets = max(1, min(8, -(-2 * l2 // set_bytes)))
    g = torch.Generator(device=dev).manual_seed(5)

    def mk(r, c):
        if args.dist == "uniform":
            return (torch.rand((r, c), generator=g, device=dev) * 2 - 1).half()
        return torch.randn((r, c), generator=g, device=dev, dtype=torch.float16)

    sets = [(mk(M, K), mk(N, K) if colb else mk(K, N), torch.empty((M, N), device=dev, dtype=torch.float16))
            for _ in range(nsets)]

    def f(i):
        A, B, C = sets[i % nsets]
        if args.variant == "torch":
            return torch.mm(A, B.t() if colb else B, out=C)
        if colb:
            return tg.gemm_pretransposed(A, B, mode="reg_pingpong_256_colb")
        return tg.gemm(A, B, out=C)

    for i in range(max(args.warmup, 1)):
        f(i)
    ms = _time_graph(torch, f, args.steps) if args.graph else _time_launches(torch, f, args.steps)
    err = _native.last_device_error()
    emit({"case": args.case, "variant": args.variant, "dist": args.dist, "graph": args.graph,
                      "us": round(ms * 1e3, 2),
                      "TFLOPs": round(2.0 * M * N * K / (ms * 1e-3) / 1e12, 1),
                      "GBps": round(set_bytes / (ms * 1e-3) / 1e9, 1), "operand_sets": nsets,
                      "device_error_word": err})
    return 0 if err == 0 else 1


def run_kmeans_case(args, torch, M, N, K, dev) -> int:
    """`--case MxNxK --variant kmeans`: kmeans.assign of M points (M x K) to N
    centroids (N x K) over rotating point sets (> 2x L2 together)."""
    from tensorcore_gemm import _native, kmeans

    g = torch.Generator(device=dev).manual_seed(5)
    point_bytes = 2 * M * K
    nsets = max(1, min(8, -(-2 * torch.cuda.get_device_properties(dev).L2_cache_size // point_bytes)))
    pts = [torch.randn((M, K), generator=g, device=dev, dtype=torch.float16) for _ in range(nsets)]
    cent = torch.randn((N, K), generator=g, device=dev, dtype=torch.float16)
    f = lambda i: kmeans.assign(pts[i % nsets], cent)
    for i in range(max(args.warmup, 1)):
        f(i)
    ms = _time_launches(torch, f, args.steps)
    err = _native.last_device_error()
    moved = point_bytes + 2 * N * K + 4 * M
    emit({"case": args.case, "variant": "kmeans", "us": round(ms * 1e3, 2),
          "GBps": round(moved / (ms * 1e-3) / 1e9, 1), "point_sets": nsets, "device_error_word": err})
    return 0 if err == 0 else 1


# The result line goes to the process's original stdout; everything else that
# writes to file descriptor 1 (NCCL's version banner, library logs) is sent to
# stderr, so stdout carries exactly one JSON line.
RESULT_OUT = sys.stdout


def emit(line: dict) -> None:
    print(json.dumps(line), file=RESULT_OUT, flush=True)


def _isolate_stdout() -> None:
    global RESULT_OUT
    sys.stdout.flush()
    RESULT_OUT = os.fdopen(os.dup(1), "w")
    os.dup2(2, 1)
    sys.stdout = sys.stderr


def main() -> int:
    _isolate_stdout()
    args = parse_args()
    if args.case:
        return run_case(args)
    if args.impl == "reference":
        return run_reference(args)
    return run_b200(args)


if __name__ == "__main__":
    sys.exit(main())
