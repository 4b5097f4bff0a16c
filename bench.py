"""Benchmark of the sm_100a operator library on the operator family's workloads.

Headline (one JSON line on rank 0): the large sharded Llama-style MLP block
(configuration 5 of the benchmark set) -- bf16 RMSNorm of x[16384, 4096]
feeding the packed GEMM+SwiGLU (M=16384, K=4096, N=14336, W[28672, 4096]) --
as GEMM+SwiGLU
TFLOP/s for the whole job.  One step = the block as the reference defines it:
the bf16 RMSNorm of all rows (each rank needs the whole normalised X for its N
slice) writing the normalised X, then the N-sharded GEMM+SwiGLU with bf16
output.  Every rank normalises all rows: sharding the RMSNorm by rows needs
an NVLink exchange of the normalised rows that measured slower at 2, 4 and 8
GPUs (reported under ``variants``).  Consecutive steps are pipelined over two
normalised-X buffers: step i's RMSNorm runs on a second stream and overlaps
step i-1's GEMM.  All inputs are resident in HBM (X 134 MB and W 235 MB
exceed the 126 MB L2, so no flush between steps is needed).  Scaling is
strong: the total work is fixed and rank r of N owns output columns
[r*N/g, (r+1)*N/g).  Inputs are generated on the
host from one seed, so the GPU step, the CPU baseline and ``--impl
reference`` see the same tensors.

Extra keys: ``e2e`` (the same metric through the public API with the X copy
from pinned host memory -- at N > 1 each rank its own rows -- and the output
shard copied back inside every step, uploads, compute and downloads of
consecutive steps overlapped on three streams; ``serial_value`` without the
overlap), ``roofline`` (the GEMM kernel against the measured bf16 peak: burst
for a timed region under a second),
``cpu_baseline`` (the CPU oracle, rank 0 at N=1) and ``parity`` (the GPU
output of the last timed step against that CPU result, every row the CPU
computed, at the bf16 bar), ``variants`` (the step unpipelined, with the
RMSNorm folded into the GEMM, and at N > 1 with the RMSNorm sharded by rows
and its rows exchanged three ways, the exchanged X checked equal to the
unsharded RMSNorm), ``clocks`` (nvidia-smi sampled during the
timed region), ``gpu_launches`` and ``ops`` (every other configuration of the set:
per-op device time, GB/s or TFLOP/s and the fraction of the measured peak,
timed from CUDA graphs of back-to-back calls -- cold rotates over input sets
three times the L2 size, warm repeats one set -- with the CPU oracle's time
of the same op beside it; the large RMSNorm and the 2^30 reduction are
measured sharded at every N).

``--impl reference`` times the reference's CPU path (the CPU oracle) on a
bounded row sample of the same workload, on rank 0 only.

Launch: python bench.py [--gpus N --steps K --warmup W]; for N > 1 under
torch.distributed.run with one process per GPU (NCCL).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from datetime import timedelta
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "cuda-operator-lab_b200"))
sys.path.insert(0, str(ROOT))

M, K, N = 16384, 4096, 14336
EPS = 1e-6
SEED = 20261201
GEMM_FLOPS = 2 * M * K * 2 * N  # 3,848,290,697,216 per step (whole job)
REDUCTION_N = 1 << 30
METRIC = ("GEMM+SwiGLU TFLOP/s, Llama MLP block (RMSNorm bf16 -> packed GEMM+SwiGLU bf16, "
          "M=16384 K=4096 N=14336)")


def peaks() -> dict:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.is_file():
        data = json.loads(path.read_text())
        return {"hbm_gbs": float(data["hbm_gbs"]), "bf16_tflops": float(data["bf16_tflops"]),
                "bf16_tflops_sustained": float(data.get("bf16_tflops_sustained",
                                                        data["bf16_tflops"])),
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
            "source": "fallback"}


def committed_traffic() -> dict:
    path = ROOT / "profiles" / "traffic.json"
    return json.loads(path.read_text()) if path.is_file() else {}


# ---------------------------------------------------------------- distributed


class Dist:
    def __init__(self) -> None:
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local_rank = int(os.environ.get("LOCAL_RANK", "0"))
        self.enabled = self.world > 1
        self.last_region_ms: list[float] = []
        if self.enabled:
            import torch.distributed as dist

            # NCCL's communicator set-up lines (ranks, devices, transports) on
            # stderr, so a run's log shows the communicator each rank joined
            # (an environment asking for the version line only gets the INIT
            # lines as well)
            if os.environ.get("NCCL_DEBUG", "").upper() in ("", "VERSION"):
                os.environ["NCCL_DEBUG"] = "INFO"
                os.environ.setdefault("NCCL_DEBUG_SUBSYS", "INIT")
            torch.cuda.set_device(self.local_rank)
            dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                                    device_id=torch.device("cuda", self.local_rank))
            self.dist = dist
            # one collective, so the communicator exists (NCCL creates it lazily)
            # and its set-up lines precede the run; then a summary of this rank
            t = torch.ones(1, device="cuda")
            dist.all_reduce(t)
            # one write per line: the ranks share the stream
            sys.stderr.write(f"[bench] rank {self.rank}/{self.world}: NCCL communicator of "
                             f"{int(t.item())} ranks on cuda:{self.local_rank} "
                             f"({torch.cuda.get_device_name(self.local_rank)})\n")
            sys.stderr.flush()
        elif torch.cuda.is_available():
            torch.cuda.set_device(0)

    def barrier(self) -> None:
        if self.enabled:
            self.dist.barrier()
        torch.cuda.synchronize()

    def max(self, value: float) -> float:
        if not self.enabled:
            return value
        t = torch.tensor([value], dtype=torch.float64, device="cuda")
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def values(self, value: float) -> list[float]:
        """`value` of every rank, in rank order (one all-gather)."""
        if not self.enabled:
            return [value]
        t = torch.tensor([value], dtype=torch.float64, device="cuda")
        out = torch.empty(self.world, dtype=torch.float64, device="cuda")
        self.dist.all_gather_into_tensor(out, t)
        return [float(v) for v in out.tolist()]

    def close(self) -> None:
        if self.enabled:
            self.dist.barrier()
            self.dist.destroy_process_group()


# ---------------------------------------------------------------- clocks


class ClockSampler:
    """nvidia-smi samples of SM clock and throttle reasons during a region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpus: list[int], enabled: bool = True) -> None:
        """gpus: nvidia-smi indices of the job's GPUs; one process (rank 0)
        samples them all, the other ranks pass enabled=False."""
        self.gpus = gpus
        self.enabled = enabled
        self.proc = None
        self.file = None

    def __enter__(self):
        if not self.enabled:
            return self
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=self.file, stderr=subprocess.DEVNULL)
            # start timing only once nvidia-smi is producing samples
            deadline = time.time() + 5.0
            while time.time() < deadline and os.path.getsize(self.file.name) == 0:
                time.sleep(0.02)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def __exit__(self, *exc) -> None:
        if self.proc is not None:
            time.sleep(0.1)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        if self.proc is None or self.file is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.file.flush()
        rows = []
        for line in Path(self.file.name).read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                idx = int(parts[0])
            except ValueError:
                continue
            if idx in self.gpus:
                rows.append(parts)
        os.unlink(self.file.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}

        def num(s):
            try:
                return float(s)
            except ValueError:
                return None

        power = [num(r[3]) for r in rows if num(r[3]) is not None]
        loaded = [r for r in rows if num(r[3]) is not None and num(r[3]) > 0.5 * max(power)] or rows
        clocks = [num(r[1]) for r in loaded if num(r[1]) is not None]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in loaded for i in range(4)
                          if r[5 + i].lower().startswith("active")})
        return {"sm_mhz": statistics.median(clocks) if clocks else None,
                "sm_max_mhz": max(num(r[2]) for r in rows if num(r[2]) is not None),
                "reasons": reasons, "samples": len(loaded),
                "power_w_max": max(power) if power else None}


# ---------------------------------------------------------------- inputs


def physical_gpus(world: int) -> list[int]:
    """nvidia-smi indices of the job's GPUs (CUDA_VISIBLE_DEVICES order when
    it lists integers, else 0..world-1)."""
    visible = os.environ.get("CUDA_VISIBLE_DEVICES", "")
    parts = [v.strip() for v in visible.split(",") if v.strip()]
    if parts and all(v.isdigit() for v in parts):
        return [int(v) for v in parts[:world]]
    return list(range(world))


def make_inputs(world: int, rank: int, device: torch.device | str) -> dict:
    """Seeded synthetic inputs of the large MLP workload, generated on the host
    with one CPU generator so that every arm (the GPU step, the CPU baseline
    and ``--impl reference``) sees the same tensors: X ~ N(0,1), the norm
    weight ~ U(0.5,1.5), the packed W[2N, K] ~ N(0, 1/K) (gate rows first).
    Rank r of `world` keeps gate rows and up rows [r*N/g, (r+1)*N/g) of W."""
    g = torch.Generator()
    g.manual_seed(SEED)
    x = torch.randn(M, K, generator=g).to(torch.bfloat16)
    w_norm = (torch.rand(K, generator=g) + 0.5).to(torch.bfloat16)
    n_local = N // world
    lo, hi = rank * n_local, (rank + 1) * n_local
    gate = torch.empty(n_local, K, dtype=torch.bfloat16)
    up = torch.empty(n_local, K, dtype=torch.bfloat16)
    rows_per_chunk = 2048
    for dst in (gate, up):
        for r0 in range(0, N, rows_per_chunk):  # the same stream on every rank
            chunk = torch.randn(rows_per_chunk, K, generator=g) * (K ** -0.5)
            a, b = max(r0, lo), min(r0 + rows_per_chunk, hi)
            if a < b:
                dst[a - lo:b - lo] = chunk[a - r0:b - r0].to(torch.bfloat16)
    packed = torch.cat((gate, up), dim=0).contiguous()
    del gate, up
    return {"x": x.to(device), "w_norm": w_norm.to(device), "packed": packed.to(device),
            "n_local": n_local}


# ---------------------------------------------------------------- our arm


def time_region(d: Dist, fn, steps: int, warmup: int, drain=None, after_start=None) -> float:
    """Max over ranks of the device time (ms) of `steps` calls of fn.  When fn
    also uses other streams, `after_start(start_event)` makes them wait for the
    start event and `drain()` makes the current stream wait for their last
    work, so the timed region covers it."""
    for _ in range(warmup):
        fn()
    if drain is not None:
        drain()
    d.barrier()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record()
    if after_start is not None:
        after_start(start)
    for _ in range(steps):
        fn()
    if drain is not None:
        drain()
    end.record()
    end.synchronize()
    ms = start.elapsed_time(end)
    d.barrier()
    d.last_region_ms = d.values(ms)
    return max(d.last_region_ms)


def event_median_us(fn, reps: int, flush=None) -> float:
    samples = []
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    for _ in range(reps):
        if flush is not None:
            flush()
        start.record()
        fn()
        end.record()
        end.synchronize()
        samples.append(start.elapsed_time(end) * 1000.0)
    return statistics.median(samples)


def graph_us(calls, reps: int = 20) -> float:
    """Device time per call of the closures `calls`, captured once into a CUDA
    graph and replayed back to back (no host launch cost between calls)."""
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for c in calls[:2]:
            c()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for c in calls:
            c()
    graph.replay()
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(reps):
        graph.replay()
    end.record()
    end.synchronize()
    us = start.elapsed_time(end) * 1000.0 / (reps * len(calls))
    del graph
    return us


def rotation(make, nbytes: int, min_calls: int = 64) -> tuple[list, list]:
    """Closures over input sets whose total is 3x the L2 (every call reads
    cold data, and nothing is flushed inside the timed replay), and the same
    number of calls on set 0 (warm L2)."""
    l2 = torch.cuda.get_device_properties(torch.cuda.current_device()).L2_cache_size
    nsets = max(2, -(-3 * l2 // max(nbytes, 1)))
    sets = [make(i) for i in range(nsets)]
    reps = max(min_calls, nsets)
    cold = [sets[i % nsets] for i in range(reps)]
    warm = [sets[0]] * reps
    return cold, warm


def op_table(d: Dist, pk: dict) -> dict:
    """Every other benchmark configuration at N=1 (rank 0), plus the sharded large
    RMSNorm and 2^30 reduction at every N.  Single-GPU configs are timed from
    CUDA graphs of back-to-back calls: cold rotates over input sets 3x the
    L2 size, warm repeats one set."""
    from cuda_operator_lab import bindings as b
    from cuda_operator_lab.benchmarking import L2Flusher

    dev = torch.device("cuda")
    ops: dict = {}
    hbm = pk["hbm_gbs"]
    tc = pk["bf16_tflops"]
    flush = L2Flusher(dev)

    def mem_op(name, make, nbytes):
        cold_calls, warm_calls = rotation(make, nbytes)
        cold = graph_us(cold_calls)
        warm = graph_us(warm_calls)
        ops[name] = {"us_cold": round(cold, 3), "us_warm": round(warm, 3),
                     "gbs_cold": round(nbytes / cold / 1e3, 1),
                     "frac_cold": round(nbytes / cold / 1e3 / hbm, 3), "bytes": nbytes}
        torch.cuda.empty_cache()

    def tc_op(name, make, flops, nbytes):
        cold_calls, _ = rotation(make, nbytes, min_calls=12)
        us = graph_us(cold_calls, reps=5)
        ops[name] = {"us_cold": round(us, 3), "tflops": round(flops / us / 1e6, 1),
                     "frac": round(flops / us / 1e6 / tc, 3), "flops": flops}
        torch.cuda.empty_cache()

    g = torch.Generator(device=dev)
    g.manual_seed(SEED + 1)
    # sharded at every N: RMSNorm bf16 rows [r*M/g, ...) and the 2^30 reduction chunk
    rows = M // d.world
    xs = torch.randn(rows, K, device=dev, generator=g).to(torch.bfloat16)
    ws = (torch.rand(K, device=dev, generator=g) + 0.5).to(torch.bfloat16)
    ys = torch.empty_like(xs)
    nbytes = 2 * rows * K * 2 + K * 2
    us = event_median_us(lambda: b.rmsnorm_bf16_into(xs, ws, ys, EPS), 50, flush)
    us = d.max(us)
    ops["rmsnorm_bf16_16384x4096_rowsharded"] = {
        "us_per_rank": round(us, 3), "gbs_job": round(nbytes * d.world / us / 1e3, 1),
        "frac_per_gpu": round(nbytes / us / 1e3 / hbm, 3)}
    del xs, ys
    chunk = REDUCTION_N // d.world
    xr = torch.rand(chunk, device=dev, generator=g) * 2 - 1
    partial = torch.empty(1, device=dev, dtype=torch.float64)

    def reduce_step():
        b.reduction_partial_f64_into(xr, partial)
        if d.enabled:
            d.dist.all_reduce(partial)
        return partial.to(torch.float32)

    us = d.max(event_median_us(reduce_step, 20))
    ops["reduction_2^30_chunked_allreduce"] = {
        "us": round(us, 3), "gbs_job": round(REDUCTION_N * 4 / us / 1e3, 1),
        "frac_per_gpu": round(chunk * 4 / us / 1e3 / hbm, 3)}
    del xr
    if d.rank != 0 or d.world > 1:
        return ops

    # rank 0 at N=1: the single-GPU configs
    def randn(*shape, scale=1.0):
        return torch.randn(*shape, device=dev, generator=g) * scale

    def rmsnorm_set(i):
        x = randn(128, 8192)
        w = torch.rand(8192, device=dev, generator=g) + 0.5
        y = torch.empty_like(x)
        return lambda: b.rmsnorm_v4_into(x, w, y, EPS)

    mem_op("rmsnorm_fp32_128x8192", rmsnorm_set, 2 * 128 * 8192 * 4 + 8192 * 4)

    def softmax_set(i):
        x = randn(128, 4096, scale=2.0)
        y = torch.empty_like(x)
        return lambda: b.softmax_v5_into(x, y)

    mem_op("softmax_fp32_128x4096", softmax_set, 2 * 128 * 4096 * 4)

    def ln_set(kind):
        def make(i):
            x, r = randn(128, 4096), randn(128, 4096)
            gam = torch.rand(4096, device=dev, generator=g) + 0.5
            bet = randn(4096, scale=0.1)
            y, h = torch.empty_like(x), torch.empty_like(x)
            return {"ln": lambda: b.layernorm_v5_into(x, gam, bet, y),
                    "res": lambda: b.fused_residual_layernorm_v4_into(x, r, gam, bet, y),
                    "res_h": lambda: b.fused_residual_layernorm_h_into(x, r, gam, bet, h, y)}[kind]
        return make

    elems = 128 * 4096
    mem_op("layernorm_fp32_128x4096", ln_set("ln"), 2 * elems * 4 + 2 * 4096 * 4)
    mem_op("residual_layernorm_fp32_128x4096", ln_set("res"), 3 * elems * 4 + 2 * 4096 * 4)
    mem_op("residual_layernorm_h_fp32_128x4096", ln_set("res_h"), 4 * elems * 4 + 2 * 4096 * 4)

    def reduction_set(i):
        xr = torch.rand(16_777_216, device=dev, generator=g) * 2 - 1
        s = torch.empty(1, device=dev)
        return lambda: b.reduction_v5_into(xr, s)

    mem_op("reduction_fp32_16777216", reduction_set, 16_777_216 * 4)

    def bias_gelu_set(i):
        x, bias = randn(1024, 4096), randn(4096, scale=0.1)
        y = torch.empty_like(x)
        return lambda: b.fused_bias_gelu_v2_into(x, bias, y)

    mem_op("bias_gelu_fp32_1024x4096", bias_gelu_set, 2 * 1024 * 4096 * 4 + 4096 * 4)

    def swiglu_set(i):
        x, u = randn(1024, 4096), randn(1024, 4096)
        y = torch.empty_like(x)
        return lambda: b.swiglu_v2_into(x, u, y)

    mem_op("swiglu_fp32_1024x4096", swiglu_set, 3 * 1024 * 4096 * 4)

    def residual_rmsnorm_set(i):
        x, r = randn(M, K).to(torch.bfloat16), randn(M, K).to(torch.bfloat16)
        w = (torch.rand(K, device=dev, generator=g) + 0.5).to(torch.bfloat16)
        h, y = torch.empty_like(x), torch.empty_like(x)
        return lambda: b.fused_residual_rmsnorm_into(x, r, w, h, y, EPS)

    mem_op("residual_rmsnorm_bf16_16384x4096", residual_rmsnorm_set, 4 * M * K * 2 + K * 2)

    fl = 2 * 512 * 4096 * 8192
    xb = randn(512, 4096).to(torch.bfloat16)

    def swiglu_gemm_set(out_kind):
        def make(i):
            wb = randn(8192, 4096, scale=4096 ** -0.5).to(torch.bfloat16)
            if out_kind == "fp32":
                ws32 = torch.empty(512, 8192, device=dev)
                o32 = torch.empty(512, 4096, device=dev)
                return lambda: b.gemm_swiglu_v11_into(xb, wb, ws32, o32)
            ob = torch.empty(512, 4096, device=dev, dtype=torch.bfloat16)
            return lambda: b.gemm_swiglu_bf16_into(xb, wb, ob)
        return make

    tc_op("gemm_swiglu_bf16_512x4096x4096_fp32out_v11", swiglu_gemm_set("fp32"), fl, 8192 * 4096 * 2)
    tc_op("gemm_swiglu_bf16_512x4096x4096_bf16out", swiglu_gemm_set("bf16"), fl, 8192 * 4096 * 2)
    xs_ = randn(128, 64).to(torch.bfloat16)
    wsm = randn(4096, 64, scale=0.125).to(torch.bfloat16)
    os_ = torch.empty(128, 2048, device=dev)
    ws_ = torch.empty(128, 4096, device=dev)
    small = lambda: b.gemm_swiglu_v11_into(xs_, wsm, ws_, os_)  # noqa: E731
    us_graph = graph_us([small] * 64)
    us_single = event_median_us(small, 100)
    # host cost of one call through the public API (Python validation, ctypes,
    # tensor maps, launch): a loop of calls is host-bound when it exceeds the
    # kernel's ~3 us
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(2000):
        small()
    host_us = (time.perf_counter() - t0) / 2000 * 1e6
    torch.cuda.synchronize()
    ops["gemm_swiglu_bf16_128x64x2048_v11"] = {
        "us_back_to_back": round(us_graph, 3), "us_single_call": round(us_single, 3),
        "us_host_per_call": round(host_us, 3),
        "tflops": round(2 * 128 * 64 * 4096 / us_graph / 1e6, 2)}

    def gelu_gemm_set(dtype):
        def make(i):
            bg = randn(4096, scale=0.1)
            if dtype == "bf16":
                wg = randn(4096, 4096, scale=4096 ** -0.5).to(torch.bfloat16)
                og = torch.empty(512, 4096, device=dev, dtype=torch.bfloat16)
                return lambda: b.gemm_bias_gelu_bf16_into(xb, wg, bg, og)
            wf = randn(4096, 4096, scale=4096 ** -0.5)
            of = torch.empty(512, 4096, device=dev)
            return lambda: b.gemm_bias_gelu_v0_into(xf, wf, bg, of)
        return make

    tc_op("gemm_bias_gelu_bf16_512x4096x4096", gelu_gemm_set("bf16"), 2 * 512 * 4096 * 4096,
          4096 * 4096 * 2)
    xf = randn(512, 4096)
    tc_op("gemm_bias_gelu_fp32_512x4096x4096_v0", gelu_gemm_set("fp32"), 2 * 512 * 4096 * 4096,
          4096 * 4096 * 4)

    def down_proj_set(i):
        xd = randn(512, 14336).to(torch.bfloat16)
        wd = randn(4096, 14336, scale=14336 ** -0.5).to(torch.bfloat16)
        hd = randn(512, 4096).to(torch.bfloat16)
        od = torch.empty_like(hd)
        return lambda: b.gemm_residual_bf16_into(xd, wd, hd, od)

    tc_op("gemm_residual_bf16_512x14336x4096", down_proj_set, 2 * 512 * 14336 * 4096,
          4096 * 14336 * 2)

    def swiglu_fp32_set(i):
        wf2 = randn(8192, 4096, scale=4096 ** -0.5)
        ws = torch.empty(512, 8192, device=dev)
        o = torch.empty(512, 4096, device=dev)
        return lambda: b.gemm_swiglu_v3_into(xf, wf2, ws, o)

    tc_op("gemm_swiglu_fp32_512x4096x4096_v3", swiglu_fp32_set, fl, 8192 * 4096 * 4)
    return ops


def run_ours(args, d: Dist) -> dict | None:
    from cuda_operator_lab import bindings as b

    dev = torch.device("cuda", torch.cuda.current_device())
    pk = peaks()
    inp = make_inputs(d.world, d.rank, dev)
    x, w_norm, packed, n_local = inp["x"], inp["w_norm"], inp["packed"], inp["n_local"]
    out = torch.empty(M, n_local, device=dev, dtype=torch.bfloat16)

    # One step = the block as the reference defines it: bf16 RMSNorm of every
    # row of X (each rank needs all rows for its N slice) writing normalised X,
    # then the packed GEMM+SwiGLU of this rank's N slice.  Every rank
    # normalises all rows: the row-sharded form with its NVLink exchange
    # (sharding.RowNormGather) gives the same bytes but measured slower at 2,
    # 4 and 8 GPUs and is timed among the variants.  Steps are pipelined over
    # two normalised-X buffers: step i's RMSNorm runs on a second stream as
    # soon as the GEMM two steps back has read its buffer, so it overlaps the
    # previous GEMM; step i's GEMM waits for it.  Every step's RMSNorm and
    # GEMM run inside the timed region.  The GEMM's stream has the higher
    # priority: when both kernels are ready, the block scheduler places the
    # GEMM's CTAs first.  CUDA events around every GEMM launch of the timed
    # steps (on the launching stream) give the dominant kernel's average
    # duration.
    b.gemm_status(clear=True)
    with ClockSampler(physical_gpus(d.world), enabled=d.rank == 0) as clocks:
        ms, gemm_rank_us = pipelined_block(d, args, x, w_norm, packed, out, None)
    step_ms_ranks = [v / args.steps for v in d.last_region_ms]
    gemm_us_ranks = d.values(gemm_rank_us)
    gemm_us = max(gemm_us_ranks)
    clock_info = clocks.summary() if d.rank == 0 else None
    status = b.gemm_status(clear=True)
    if status != 0:
        raise RuntimeError(f"GEMM bounded wait timed out (status {status})")
    gpu_out = out.cpu() if d.rank == 0 and d.world == 1 and not args.skip_cpu else None

    variants = step_variants(d, args, x, w_norm, packed, out)

    flops_launch = 2 * M * K * 2 * n_local
    achieved = flops_launch / gemm_us / 1e6
    traffic = committed_traffic().get(f"gemm_swiglu_bf16_M{M}_K{K}_N{n_local}")
    # The burst peak applies to a kernel timed in a region well under a
    # second (the sustained one is a seconds-long loop under the power cap).
    timed_s = ms / 1e3
    peak_kind = "burst" if timed_s < 1.0 else "sustained"
    peak = pk["bf16_tflops"] if peak_kind == "burst" else pk["bf16_tflops_sustained"]
    gemm_bytes = (M * K + 2 * n_local * K + M * n_local) * 2  # X, W shard, output (bf16)

    e2e = e2e_pipeline(d, args, x, w_norm, packed, out)

    gather = None
    if d.world > 1 and args.gather:
        rstd = torch.empty(M, device=dev)
        folded = b.fold_rmsnorm_weight(packed, w_norm)
        gather = gather_variant(d, x, rstd, folded, out, args)
        del rstd, folded

    ops = op_table(d, pk) if not args.skip_ops else {}

    cpu = parity = None
    if gpu_out is not None:
        del x, packed  # the CPU leg works on host copies
        torch.cuda.empty_cache()
        host = make_inputs(1, 0, "cpu")
        cpu, parity = cpu_baseline(args.cpu_seconds, host, gpu_out)
        if not args.skip_ops:
            for name, us in cpu_op_times().items():
                if name in ops:
                    ops[name]["cpu_us"] = us

    if d.rank != 0:
        return None
    value = GEMM_FLOPS * args.steps / (ms / 1e3) / 1e12
    return {
        "metric": METRIC,
        "value": round(value, 2),
        "unit": "TFLOP/s",
        "n_gpus": d.world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms / args.steps, 4),
        **({"ms_per_step_ranks": [round(v, 4) for v in step_ms_ranks]} if d.world > 1 else {}),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) X, N(0,1/K) W, U(0.5,1.5) norm weight)",
        "config": {"workload": "llama_mlp_block (BASELINE config 5)", "M": M, "K": K, "N": N,
                   "rmsnorm": ("bf16 RMSNorm of all 16384 rows on every rank, writing the "
                               "normalised X the GEMM reads (the reference's block "
                               "semantics); step i's RMSNorm on a second stream into one of "
                               "two X buffers, overlapping step i-1's GEMM" +
                               ("; the row-sharded form with its NVLink exchange is "
                                "variants.row_sharded_rmsnorm" if d.world > 1 else "")),
                   "gemm": "packed GEMM+SwiGLU bf16 out, N-sharded",
                   "parallelism": f"N-shard x{d.world}" if d.world > 1 else "single GPU",
                   "l2": "inputs larger than L2 (X 134 MB, W 235 MB); no flush"},
        "e2e": e2e,
        "roofline": {"bound": "tensor", "achieved": round(achieved, 1), "peak": peak,
                     "unit": "TFLOP/s", "frac": round(achieved / peak, 3),
                     "traffic": traffic,
                     "traffic_over_algorithmic": (round(traffic / gemm_bytes, 2)
                                                  if traffic else None),
                     "algorithmic_bytes": gemm_bytes,
                     "kernel": "gemm_bf16_tc2_kernel (CTA pair, SwiGLU, bf16 out)",
                     "peak_source": f"{pk['source']} {peak_kind} bf16 (timed region "
                                    f"{timed_s * 1e3:.0f} ms)",
                     "gemm_us_per_launch": round(gemm_us, 2),
                     **({"gemm_us_per_launch_ranks": [round(v, 2) for v in gemm_us_ranks]}
                        if d.world > 1 else {})},
        "cpu_baseline": cpu,
        "parity": parity,
        "variants": {**variants, **({"gathered_output": gather} if gather is not None else {})},
        "clocks": clock_info,
        "gpu_launches": 2 * args.steps,  # per step: RMSNorm + GEMM
        "ops": ops,
    }


def norm_replicated(x, w_norm):
    """Every rank normalises all rows into one of two buffers."""
    from cuda_operator_lab import bindings as b

    xns = [torch.empty_like(x) for _ in range(2)]

    def norm(j):
        b.rmsnorm_bf16_into(x, w_norm, xns[j], EPS)
        return xns[j]
    return norm


def norm_nccl(d: Dist, x, w_norm):
    """Each rank normalises its rows; NCCL all-gathers them into one of two
    full buffers."""
    from cuda_operator_lab import bindings as b

    rows = M // d.world
    lo = d.rank * rows
    parts = [torch.empty(rows, K, device=x.device, dtype=x.dtype) for _ in range(2)]
    xns = [torch.empty_like(x) for _ in range(2)]

    def norm(j):
        b.rmsnorm_bf16_into(x[lo:lo + rows], w_norm, parts[j], EPS)
        d.dist.all_gather_into_tensor(xns[j], parts[j])
        return xns[j]
    return norm


def pipelined_block(d: Dist, args, x, w_norm, packed, out, norm=None) -> tuple[float, float]:
    """Times the pipelined block (see run_ours): returns the max over ranks of
    the timed region (ms) and this rank's mean GEMM launch time (us).
    `norm(slot)` enqueues, on the current (second) stream, the RMSNorm of all
    rows into buffer `slot` and returns that buffer: a row-sharded
    sharding.RowNormGather, or a replicated or NCCL form (default:
    replicated)."""
    from cuda_operator_lab import bindings as b

    main = torch.cuda.Stream(priority=-1)
    main.wait_stream(torch.cuda.current_stream())
    side = torch.cuda.Stream()
    if norm is None:
        norm = norm_replicated(x, w_norm)
    xns = [None, None]
    normed = [torch.cuda.Event() for _ in range(2)]
    consumed = [torch.cuda.Event() for _ in range(2)]
    gemm_events = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                   for _ in range(args.steps)]
    step_index = [0]

    def step():
        j = step_index[0] % 2
        side.wait_event(consumed[j])  # the GEMM two steps back has read xns[j]
        with torch.cuda.stream(side):
            xns[j] = norm(j)
            normed[j].record(side)
        main.wait_event(normed[j])
        i = step_index[0] - args.warmup
        if 0 <= i < args.steps:
            gemm_events[i][0].record(main)
        b.gemm_swiglu_bf16_into(xns[j], packed, out)
        if 0 <= i < args.steps:
            gemm_events[i][1].record(main)
        consumed[j].record(main)
        step_index[0] += 1

    def drain():
        main.wait_stream(side)

    def start(ev):
        side.wait_event(ev)

    with torch.cuda.stream(main):
        ms = time_region(d, step, args.steps, args.warmup, drain=drain, after_start=start)
    torch.cuda.current_stream().wait_stream(main)
    gemm_us = 1000.0 * sum(s_.elapsed_time(e_) for s_, e_ in gemm_events) / args.steps
    return ms, gemm_us


def step_variants(d: Dist, args, x, w_norm, packed, out) -> dict:
    """Other forms of the same step, timed in the same run:

    * ``row_sharded_rmsnorm``, ``nccl_rmsnorm_allgather`` and
      ``copy_engine_rmsnorm_allgather`` (N > 1): the pipelined step with the
      RMSNorm sharded by rows, its rows all-gathered by peer stores from the
      norm kernel, by NCCL or by the copy engines;
    * ``serial``: RMSNorm then GEMM on one stream, one normalised-X buffer
      (no overlap between consecutive steps);
    * ``folded``: the RMSNorm folded into the GEMM (a per-row rstd pass, rstd
      applied to gate and up in the GEMM epilogue, the norm weight folded into
      W once).  Its bf16 rounding falls on W * w instead of on the normalised
      X, so it is not the reference's block bit for bit."""
    from cuda_operator_lab import bindings as b
    from cuda_operator_lab import sharding

    res = {}

    def entry(ms, text):
        return {"value": round(GEMM_FLOPS * args.steps / (ms / 1e3) / 1e12, 2),
                "ms_per_step": round(ms / args.steps, 4), "step": text}

    if d.world > 1:
        ms, _ = pipelined_block(d, args, x, w_norm, packed, out, norm_nccl(d, x, w_norm))
        res["nccl_rmsnorm_allgather"] = entry(
            ms, "pipelined like the headline, each rank normalising its rows, NCCL "
                "all_gather_into_tensor of the normalised rows on the second stream")
        rng = sharding.RowNormGather(M, K)
        try:
            ms, _ = pipelined_block(d, args, x, w_norm, packed, out,
                                    lambda j: rng(x, w_norm, EPS, slot=j))
            rng.check()  # raises if an exchange barrier gave up waiting
            last = rng.outputs[(args.warmup + args.steps - 1) % 2]
            same = torch.equal(last, b.rmsnorm_bf16(x, w_norm, EPS))
            # the norm and its exchange alone, back to back (no GEMM beside them)
            alone_ms = time_region(d, lambda: rng(x, w_norm, EPS), args.steps, args.warmup)
            rng.check()
        finally:
            rng.close()
        res["row_sharded_rmsnorm"] = {
            **entry(ms, "pipelined like the headline, each rank normalising its 16384/N rows "
                        "with rmsnorm_allgather_bf16, whose threads store every row into each "
                        "rank's CUDA IPC buffer over NVLink; two device flag barriers per step"),
            "identical_to_unsharded": d.max(0.0 if same else 1.0) == 0.0,
            "nvlink_bytes_per_rank": (d.world - 1) * (M // d.world) * K * 2,
            "exchange_alone_us_per_call": round(1000.0 * alone_ms / args.steps, 1)}
        rng = sharding.RowNormGather(M, K, exchange="copies")
        try:
            ms, _ = pipelined_block(d, args, x, w_norm, packed, out,
                                    lambda j: rng(x, w_norm, EPS, slot=j))
            rng.check()
        finally:
            rng.close()
        res["copy_engine_rmsnorm_allgather"] = entry(
            ms, "pipelined like the headline, each rank normalising its rows into its own "
                "buffer, one cudaMemcpyAsync per peer (copy engines) between the barriers")
    xn = torch.empty_like(x)

    def serial():
        b.rmsnorm_bf16_into(x, w_norm, xn, EPS)
        b.gemm_swiglu_bf16_into(xn, packed, out)

    ms = time_region(d, serial, args.steps, args.warmup)
    res["serial"] = {"value": round(GEMM_FLOPS * args.steps / (ms / 1e3) / 1e12, 2),
                     "ms_per_step": round(ms / args.steps, 4),
                     "step": "rmsnorm_bf16 + gemm_swiglu_bf16 on one stream"}
    del xn
    folded_w = b.fold_rmsnorm_weight(packed, w_norm)
    rstd = torch.empty(M, device=x.device)

    def folded():
        b.rmsnorm_rstd_bf16_into(x, rstd, EPS)
        b.gemm_swiglu_rowscale_bf16_into(x, rstd, folded_w, out)

    ms = time_region(d, folded, args.steps, args.warmup)
    res["folded"] = {"value": round(GEMM_FLOPS * args.steps / (ms / 1e3) / 1e12, 2),
                     "ms_per_step": round(ms / args.steps, 4),
                     "step": "rmsnorm_rstd_bf16 + gemm_swiglu_rowscale_bf16 (norm weight "
                             "folded into W)"}
    if b.gemm_status(clear=True) != 0:
        raise RuntimeError("GEMM bounded wait timed out in a step variant")
    return res


def e2e_pipeline(d: Dist, args, x, w_norm, packed, out) -> dict:
    """The step through the public API with host buffers: every step copies
    X from pinned host memory and the output shard back.  With N ranks each
    rank uploads only its 1/N of X's rows, normalises them and the norm
    kernel stores them into every rank's normalised-X buffer over NVLink
    (sharding.RowNormGather), so each host byte crosses PCIe once and every
    row is normalised once.  Serving-style pipeline: step i's upload and
    RMSNorm (+ exchange) on a copy stream, the GEMM on this stream and the
    download on a second copy stream overlap steps i-1 and i+1, with two
    device and two pinned host buffers.  The serial form (all of it on one
    stream) is reported beside it."""
    from cuda_operator_lab import bindings as b
    from cuda_operator_lab import sharding

    world = d.world
    if M % world:
        raise SystemExit(f"M={M} must divide evenly between {world} ranks")
    rows = M // world
    x_host = x[d.rank * rows:(d.rank + 1) * rows].cpu().pin_memory()
    out_host = [torch.empty(out.shape, dtype=out.dtype, pin_memory=True) for _ in range(2)]
    x_dev = [torch.empty(rows, K, device=x.device, dtype=x.dtype) for _ in range(2)]
    rng = sharding.RowNormGather(M, K) if world > 1 else None
    xn_dev = rng.outputs if rng is not None else [torch.empty_like(x) for _ in range(2)]
    out_dev = [out, torch.empty_like(out)]
    main = torch.cuda.current_stream()
    up, down = torch.cuda.Stream(), torch.cuda.Stream()
    uploaded = [torch.cuda.Event() for _ in range(2)]
    computed = [torch.cuda.Event() for _ in range(2)]
    downloaded = [torch.cuda.Event() for _ in range(2)]
    index = [0]

    def upload_norm(j):
        """On the current stream: this rank's rows of X in, all rows normalised
        into xn_dev[j]."""
        x_dev[j].copy_(x_host, non_blocking=True)
        if rng is None:
            b.rmsnorm_bf16_into(x_dev[j], w_norm, xn_dev[j], EPS)
        else:
            rng(x_dev[j], w_norm, EPS, slot=j)

    def e2e_step():
        j = index[0] % 2
        index[0] += 1
        with torch.cuda.stream(up):
            up.wait_event(computed[j])  # step i-2's GEMM has read xn_dev[j]
            upload_norm(j)
            uploaded[j].record(up)
        main.wait_event(uploaded[j])
        main.wait_event(downloaded[j])  # step i-2's output has left out_dev[j]
        b.gemm_swiglu_bf16_into(xn_dev[j], packed, out_dev[j])
        computed[j].record(main)
        with torch.cuda.stream(down):
            down.wait_event(computed[j])
            out_host[j].copy_(out_dev[j], non_blocking=True)
            downloaded[j].record(down)

    def drain():
        for ev in downloaded:
            main.wait_event(ev)
        main.wait_stream(up)

    def serial_step():
        upload_norm(0)
        b.gemm_swiglu_bf16_into(xn_dev[0], packed, out)
        out_host[0].copy_(out, non_blocking=True)

    steps = max(6, args.steps // 20)

    def start(ev):
        up.wait_event(ev)
        down.wait_event(ev)

    try:
        e2e_ms = time_region(d, e2e_step, steps, 2, drain=drain, after_start=start)
        last = (index[0] - 1) % 2
        torch.testing.assert_close(out_host[last][:4].float(), out_dev[last][:4].cpu().float())
        # the normalised X assembled from every rank's upload is the RMSNorm of X
        assert torch.equal(xn_dev[last], b.rmsnorm_bf16(x, w_norm, EPS)), \
            "normalised X assembled from the uploads differs"
        serial_ms = time_region(d, serial_step, steps, 2)
        torch.testing.assert_close(out_host[0][:4].float(), out[:4].cpu().float())
        if rng is not None:
            rng.check()
    finally:
        if rng is not None:
            del xn_dev
            rng.close()
    return {"value": round(GEMM_FLOPS * steps / (e2e_ms / 1e3) / 1e12, 2),
            "unit": "TFLOP/s",
            # whole job: each rank copies its rows of X in and its output columns out
            "h2d_bytes_per_step": M * K * 2, "d2h_bytes_per_step": M * N * 2,
            "pipeline": ("upload of this rank's rows of X + their RMSNorm, stored by the "
                         "norm kernel into every rank's X buffer over NVLink / GEMM / "
                         "download on three streams, two buffers")
            if world > 1 else "upload + RMSNorm / GEMM / download on three streams, two buffers",
            "serial_value": round(GEMM_FLOPS * steps / (serial_ms / 1e3) / 1e12, 2)}


def gather_variant(d: Dist, x, rstd, folded, out, args) -> dict:
    """The headline step followed by the all-gather of the [M, N] output to
    every rank, two ways: fused into the GEMM's epilogue (peer stores over
    NVLink per finished tile, then the device flag barrier) and as the GEMM
    followed by an NCCL all-gather.  Checks that both deliver the same blocks."""
    from cuda_operator_lab import bindings as b
    from cuda_operator_lab import sharding

    n_local = N // d.world
    fused_ms = {}
    gathered = {}
    for layout in ("blocks", "columns"):
        pg = sharding.PeerColumnGather(M, N, layout=layout)
        try:
            def fused():
                b.rmsnorm_rstd_bf16_into(x, rstd, EPS)
                pg(x, folded, rstd)

            fused_ms[layout] = time_region(d, fused, args.steps, args.warmup)
            pg.check()  # raises if a peer barrier gave up waiting
            if b.gemm_status(clear=True) != 0:
                raise RuntimeError("GEMM bounded wait timed out (gather step)")
            gathered[layout] = pg.outputs[(pg.calls - 1) % 2].clone()
        finally:
            pg.close()
    parts = torch.empty(d.world, M, n_local, device=x.device, dtype=torch.bfloat16)

    def unfused():
        b.rmsnorm_rstd_bf16_into(x, rstd, EPS)
        b.gemm_swiglu_rowscale_bf16_into(x, rstd, folded, out)
        d.dist.all_gather_into_tensor(parts, out)

    unfused_ms = time_region(d, unfused, args.steps, args.warmup)
    same = torch.equal(gathered["blocks"], parts) and all(
        torch.equal(gathered["columns"][:, r * n_local:(r + 1) * n_local], parts[r])
        for r in range(d.world))
    same = d.max(0.0 if same else 1.0) == 0.0
    del gathered, parts
    link_bytes = (d.world - 1) * M * n_local * 2  # sent by each rank
    link_us = link_bytes / 770e3  # measured peer copy, GB/s per direction
    gemm_us = GEMM_FLOPS / d.world / (peaks()["bf16_tflops_sustained"] * 1e6)
    return {
        "fused_ms_per_step": round(fused_ms["blocks"] / args.steps, 4),
        "fused_value": round(GEMM_FLOPS * args.steps / (fused_ms["blocks"] / 1e3) / 1e12, 2),
        "fused_columns_layout_ms_per_step": round(fused_ms["columns"] / args.steps, 4),
        "nccl_ms_per_step": round(unfused_ms / args.steps, 4),
        "nccl_value": round(GEMM_FLOPS * args.steps / (unfused_ms / 1e3) / 1e12, 2),
        "unit": "TFLOP/s",
        "identical_blocks": same,
        "nvlink_bytes_per_rank": link_bytes,
        "bound_us": round(max(link_us, gemm_us), 1),
        "bound": "nvlink" if link_us > gemm_us else "tensor",
        "step": "rmsnorm_rstd + GEMM with gathering epilogue + peer flag barrier into "
                "[g, M, N/g] (the all_gather_into_tensor layout; [M, N] reported beside), vs "
                "rmsnorm_rstd + GEMM + NCCL all_gather_into_tensor",
    }


# ---------------------------------------------------------------- CPU baseline


class CpuPath:
    """The reference's CPU path (the oracle restating references.py: bf16
    RMSNorm, then the packed GEMM+SwiGLU with fp32 accumulation, bf16 out)
    over a row sample of the workload against the full W, with every host
    thread.  Row samples are spread evenly over X."""

    def __init__(self, inputs: dict) -> None:
        from oracle import reference_math as oracle

        self.oracle = oracle
        torch.set_num_threads(os.cpu_count() or 1)
        self.x, self.w_norm, self.packed = inputs["x"], inputs["w_norm"], inputs["packed"]

    @staticmethod
    def rows_index(rows: int) -> torch.Tensor:
        return torch.linspace(0, M - 1, rows).round().long().unique()

    def run(self, index: torch.Tensor) -> tuple[float, torch.Tensor]:
        t0 = time.perf_counter()
        y = self.oracle.mlp_block_bf16(self.x[index], self.w_norm, self.packed, EPS)
        return time.perf_counter() - t0, y

    def rows_for(self, seconds: float) -> int:
        """Rows whose pass takes about `seconds` (calibrated on 64 rows)."""
        self.run(self.rows_index(16))
        t, _ = self.run(self.rows_index(64))
        return int(max(16, min(M, 64 * seconds / max(t, 1e-6))))


def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def parity_check(gpu_rows: torch.Tensor, cpu_rows: torch.Tensor, rows: int) -> dict:
    """The GPU output rows against the CPU oracle's at the bf16 bar
    (|d| <= 2e-2 + 2e-2 |expected|)."""
    a, e = gpu_rows.float(), cpu_rows.float()
    diff = (a - e).abs()
    bound = 2e-2 + 2e-2 * e.abs()
    return {"rows_checked": rows, "cols_checked": int(a.shape[1]),
            "max_abs_err": round(float(diff.max()), 6),
            "max_err_over_bound": round(float((diff / bound).max()), 4),
            "violations": int((diff > bound).sum()),
            "tolerance": "rtol 2e-2 / atol 2e-2 vs the CPU oracle of the reference block "
                         "(bf16 RMSNorm -> packed GEMM+SwiGLU, fp32 accumulation)",
            "ok": bool((diff <= bound).all())}


def cpu_baseline(seconds: float, inputs: dict, gpu_out: torch.Tensor | None = None
                 ) -> tuple[dict, dict | None]:
    """The CPU path on about `seconds` of work: a row sample when a pass over
    all rows takes longer, else repeated whole passes (median reported).
    When the GPU output is given, the CPU result of the same rows is the
    checker of the GPU step (parity over every row and column computed)."""
    path = CpuPath(inputs)
    rows = path.rows_for(seconds)
    index = path.rows_index(rows)
    times, y = [], None
    while True:
        dt, y = path.run(index)
        times.append(dt)
        if rows < M or sum(times) >= seconds or len(times) >= 20:
            break
    dt = sorted(times)[len(times) // 2]
    n = int(index.numel())
    what = (f"all {M} rows of X against the full W, median of {len(times)} passes "
            f"({sum(times):.1f} s)" if n == M else
            f"{n} of {M} rows of X (evenly spaced) against the full W, one pass ({dt:.2f} s)")
    cpu = {"value": round(2 * n * K * 2 * N / dt / 1e12, 4), "unit": "TFLOP/s",
           "cores": torch.get_num_threads(), "cpu_model": cpu_model(), "kind": "port",
           "sample": what}
    parity = parity_check(gpu_out[index], y, n) if gpu_out is not None else None
    return cpu, parity


def cpu_op_times(budget_s: float = 1.0) -> dict:
    """The CPU oracle (the reference's PyTorch CPU path) on each single-GPU
    configuration of the op table, median microseconds over repeats that fit
    `budget_s` per op, all host threads."""
    from oracle import reference_math as oracle

    torch.set_num_threads(os.cpu_count() or 1)
    g = torch.Generator()
    g.manual_seed(SEED + 2)
    rn = lambda *shape: torch.randn(*shape, generator=g)  # noqa: E731
    ur = lambda *shape: torch.rand(*shape, generator=g) + 0.5  # noqa: E731
    x8, w8 = rn(128, 8192), ur(8192)
    x4, r4, gam, bet = rn(128, 4096), rn(128, 4096), ur(4096), rn(4096) * 0.1
    xr = torch.rand(16_777_216, generator=g) * 2 - 1
    xg, bg, ug = rn(1024, 4096), rn(4096) * 0.1, rn(1024, 4096)
    xb, rb = rn(M, K).to(torch.bfloat16), rn(M, K).to(torch.bfloat16)
    wb = ur(K).to(torch.bfloat16)
    x512 = rn(512, 4096).to(torch.bfloat16)
    w8192 = (rn(8192, 4096) * 4096 ** -0.5).to(torch.bfloat16)
    w4096 = (rn(4096, 4096) * 4096 ** -0.5).to(torch.bfloat16)
    xs, wsm = rn(128, 64).to(torch.bfloat16), (rn(4096, 64) * 0.125).to(torch.bfloat16)
    xd, wd = rn(512, 14336).to(torch.bfloat16), (rn(4096, 14336) * 14336 ** -0.5).to(torch.bfloat16)
    hd = rn(512, 4096).to(torch.bfloat16)
    x512f, w4096f, w8192f = x512.float(), w4096.float(), w8192.float()
    cases = {
        "rmsnorm_fp32_128x8192": lambda: oracle.rmsnorm(x8, w8, EPS),
        "softmax_fp32_128x4096": lambda: oracle.row_softmax(x4),
        "layernorm_fp32_128x4096": lambda: oracle.layernorm(x4, gam, bet),
        "residual_layernorm_fp32_128x4096": lambda: oracle.fused_residual_layernorm(x4, r4, gam, bet),
        "residual_layernorm_h_fp32_128x4096": lambda: oracle.fused_residual_layernorm_h(x4, r4, gam, bet),
        "reduction_fp32_16777216": lambda: oracle.reduction_sum(xr),
        "bias_gelu_fp32_1024x4096": lambda: oracle.fused_bias_gelu(xg, bg),
        "swiglu_fp32_1024x4096": lambda: oracle.swiglu(xg, ug),
        "residual_rmsnorm_bf16_16384x4096": lambda: oracle.fused_residual_rmsnorm(xb, rb, wb, EPS),
        "gemm_swiglu_bf16_512x4096x4096_fp32out_v11":
            lambda: oracle.gemm_swiglu_bf16_fp32_reference(x512, w8192),
        "gemm_swiglu_bf16_512x4096x4096_bf16out": lambda: oracle.gemm_swiglu_bf16_out(x512, w8192),
        "gemm_swiglu_bf16_128x64x2048_v11": lambda: oracle.gemm_swiglu_bf16_fp32_reference(xs, wsm),
        "gemm_bias_gelu_bf16_512x4096x4096": lambda: oracle.gemm_bias_gelu_bf16(x512, w4096, bg),
        "gemm_bias_gelu_fp32_512x4096x4096_v0": lambda: oracle.gemm_bias_gelu(x512f, w4096f, bg),
        "gemm_residual_bf16_512x14336x4096": lambda: oracle.gemm_residual_bf16(xd, wd, hd),
        "gemm_swiglu_fp32_512x4096x4096_v3": lambda: oracle.gemm_swiglu_packed(x512f, w8192f),
    }
    result = {}
    for name, fn in cases.items():
        fn()
        times = []
        while not times or (sum(times) < budget_s and len(times) < 50):
            t0 = time.perf_counter()
            fn()
            times.append(time.perf_counter() - t0)
        result[name] = round(1e6 * statistics.median(times), 1)
    return result


def run_reference(args) -> dict:
    path = CpuPath(make_inputs(1, 0, "cpu"))
    budget = 150.0 / (args.steps + args.warmup)  # whole run within a few minutes
    rows = path.rows_for(min(10.0, budget))
    index = path.rows_index(rows)
    for _ in range(args.warmup):
        path.run(path.rows_index(max(16, rows // 4)))
    times = [path.run(index)[0] for _ in range(args.steps)]
    n = int(index.numel())
    dt = statistics.median(times)
    value = round(2 * n * K * 2 * N / dt / 1e12, 5)
    sample = (f"{n} of {M} rows of X (evenly spaced) against the full W per step, "
              f"median of {len(times)} steps ({dt:.2f} s each)")
    return {
        "impl": "reference",
        "metric": METRIC,
        "value": value,
        "unit": "TFLOP/s",
        "n_gpus": int(os.environ.get("WORLD_SIZE", str(args.gpus))),
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(dt * 1e3, 3),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded)",
        "config": {"workload": "llama_mlp_block (BASELINE config 5)", "M": M, "K": K, "N": N,
                   "sample_rows_per_step": n,
                   "path": "reference CPU math (oracle port of references.py) on host cores"},
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": torch.get_num_threads(),
                         "cpu_model": cpu_model(), "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "gpu_launches": 0,
    }


KERNEL_CASES = ("gemm_swiglu_bf16", "gemm_bias_gelu_bf16", "rmsnorm_bf16", "reduction",
                "rmsnorm_fp32", "softmax_fp32", "layernorm_fp32", "residual_layernorm_fp32",
                "bias_gelu_fp32", "swiglu_fp32",
                "gemm_bias_gelu_fp32", "gemm_swiglu_fp32", "residual_rmsnorm_bf16",
                "gemm_residual_bf16", "gemm_swiglu_rowscale_bf16")


def run_kernel_case(spec: str, reps: int, timed: bool = False) -> None:
    """Launch one op `reps` times at a given size and exit: the command that
    profilers (ncu) wrap.  spec = NAME[:d0,d1,...], e.g. gemm_swiglu_bf16:2048,4096,14336."""
    from cuda_operator_lab import bindings as b

    name, _, dims = spec.partition(":")
    if name not in KERNEL_CASES:
        raise SystemExit(f"unknown kernel case {name}; choose from {KERNEL_CASES}")
    d = [int(v) for v in dims.split(",")] if dims else []
    dev = torch.device("cuda")
    g = torch.Generator(device=dev)
    g.manual_seed(SEED)
    rn = lambda *shape: torch.randn(*shape, device=dev, generator=g)  # noqa: E731
    if name == "gemm_swiglu_bf16":
        m, k, n = d or (2048, K, N)
        x, w = rn(m, k).bfloat16(), (rn(2 * n, k) * k ** -0.5).bfloat16()
        out = torch.empty(m, n, device=dev, dtype=torch.bfloat16)
        fn = lambda: b.gemm_swiglu_bf16_into(x, w, out)  # noqa: E731
    elif name == "gemm_bias_gelu_bf16":
        m, k, n = d or (512, 4096, 4096)
        x, w, bias = rn(m, k).bfloat16(), (rn(n, k) * k ** -0.5).bfloat16(), rn(n) * 0.1
        out = torch.empty(m, n, device=dev, dtype=torch.bfloat16)
        fn = lambda: b.gemm_bias_gelu_bf16_into(x, w, bias, out)  # noqa: E731
    elif name == "gemm_bias_gelu_fp32":
        m, k, n = d or (512, 4096, 4096)
        x, w, bias = rn(m, k), rn(n, k) * k ** -0.5, rn(n) * 0.1
        out = torch.empty(m, n, device=dev)
        fn = lambda: b.gemm_bias_gelu_v0_into(x, w, bias, out)  # noqa: E731
    elif name == "gemm_swiglu_fp32":
        m, k, n = d or (512, 4096, 4096)
        x, w = rn(m, k), rn(2 * n, k) * k ** -0.5
        ws, out = torch.empty(m, 2 * n, device=dev), torch.empty(m, n, device=dev)
        fn = lambda: b.gemm_swiglu_v3_into(x, w, ws, out)  # noqa: E731
    elif name == "residual_rmsnorm_bf16":
        r, c = d or (M, K)
        x, res = rn(r, c).bfloat16(), rn(r, c).bfloat16()
        w = (torch.rand(c, device=dev, generator=g) + 0.5).bfloat16()
        h, y = torch.empty_like(x), torch.empty_like(x)
        fn = lambda: b.fused_residual_rmsnorm_into(x, res, w, h, y, EPS)  # noqa: E731
    elif name == "gemm_swiglu_rowscale_bf16":
        m, k, n = d or (M, K, N)
        x, w = rn(m, k).bfloat16(), (rn(2 * n, k) * k ** -0.5).bfloat16()
        rs = torch.rand(m, device=dev, generator=g) + 0.5
        out = torch.empty(m, n, device=dev, dtype=torch.bfloat16)
        fn = lambda: b.gemm_swiglu_rowscale_bf16_into(x, rs, w, out)  # noqa: E731
    elif name == "gemm_residual_bf16":
        m, k, n = d or (512, 14336, 4096)
        x, w = rn(m, k).bfloat16(), (rn(n, k) * k ** -0.5).bfloat16()
        res, out = rn(m, n).bfloat16(), torch.empty(m, n, device=dev, dtype=torch.bfloat16)
        fn = lambda: b.gemm_residual_bf16_into(x, w, res, out)  # noqa: E731
    elif name == "rmsnorm_bf16":
        r, c = d or (M, K)
        x, w = rn(r, c).bfloat16(), (torch.rand(c, device=dev, generator=g) + 0.5).bfloat16()
        y = torch.empty_like(x)
        fn = lambda: b.rmsnorm_bf16_into(x, w, y, EPS)  # noqa: E731
    elif name == "reduction":
        (n,) = d or (1 << 26,)
        x = torch.rand(n, device=dev, generator=g) * 2 - 1
        out = torch.empty(1, device=dev)
        fn = lambda: b.reduction_v5_into(x, out)  # noqa: E731
    elif name in ("rmsnorm_fp32", "softmax_fp32", "layernorm_fp32", "residual_layernorm_fp32",
                  "bias_gelu_fp32", "swiglu_fp32"):
        r, c = d or (128, 8192 if name == "rmsnorm_fp32" else 4096)
        x, w, bias, y = rn(r, c), torch.rand(c, device=dev, generator=g) + 0.5, rn(c) * 0.1, None
        y = torch.empty_like(x)
        u = rn(r, c)
        fn = {"rmsnorm_fp32": lambda: b.rmsnorm_v4_into(x, w, y, EPS),
              "softmax_fp32": lambda: b.softmax_v5_into(x, y),
              "layernorm_fp32": lambda: b.layernorm_v5_into(x, w, bias, y),
              "residual_layernorm_fp32": lambda: b.fused_residual_layernorm_v4_into(x, u, w, bias,
                                                                                    y),
              "bias_gelu_fp32": lambda: b.fused_bias_gelu_v2_into(x, bias, y),
              "swiglu_fp32": lambda: b.swiglu_v2_into(x, u, y)}[name]
    if not timed:
        for _ in range(reps):
            fn()
        torch.cuda.synchronize()
        return
    from cuda_operator_lab.benchmarking import L2Flusher, measure_batch_us

    warm = measure_batch_us(fn, warmup=3, repeats=max(reps, 10))
    cold = event_median_us(fn, max(reps, 10), L2Flusher(dev))
    print(json.dumps({"kernel_case": spec, "us_warm_back_to_back": round(warm, 3),
                      "us_cold_single": round(cold, 3)}), file=sys.stderr)


def _json_stdout():
    """Keep stdout for the one JSON line: anything else written to fd 1 (NCCL's
    version banner, library prints) is sent to stderr."""
    out = os.fdopen(os.dup(1), "w")
    sys.stdout.flush()
    os.dup2(2, 1)
    return out


def main() -> None:
    json_out = _json_stdout()
    parser = argparse.ArgumentParser(description=__doc__,
                                     formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=300)
    parser.add_argument("--warmup", type=int, default=5)
    parser.add_argument("--impl", choices=("ours", "reference"), default="ours")
    parser.add_argument("--cpu-seconds", type=float, default=15.0)
    parser.add_argument("--skip-ops", action="store_true")
    parser.add_argument("--skip-cpu", action="store_true")
    parser.add_argument("--gather", action="store_true",
                        help="N > 1: also time the step with the output all-gather, fused "
                             "into the GEMM and with NCCL")
    parser.add_argument("--kernel-case", default=None,
                        help="run one op only (for profilers): NAME[:dims], see KERNEL_CASES")
    parser.add_argument("--reps", type=int, default=3)
    parser.add_argument("--time", action="store_true",
                        help="with --kernel-case: print warm and cold CUDA-event times")
    args = parser.parse_args()
    if args.kernel_case:
        run_kernel_case(args.kernel_case, args.reps, args.time)
        return
    if args.warmup < 3:
        parser.error("--warmup must be >= 3")

    if args.impl == "reference":
        if int(os.environ.get("RANK", "0")) != 0:
            return  # rank 0 alone times the CPU path
        print(json.dumps(run_reference(args)), file=json_out, flush=True)
        return

    d = Dist()
    if d.world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={d.world}")
    try:
        result = run_ours(args, d)
    finally:
        d.close()
    if result is not None:
        print(json.dumps(result), file=json_out, flush=True)


if __name__ == "__main__":
    main()
