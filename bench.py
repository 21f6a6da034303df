"""Benchmark of the quantized DiT-block linear path on B200.

Workload: 8 stacked DiT blocks, D=4096, FFN=16384, M=98304 tokens, INT8 weights
with per-channel scales; per block: prologue, QKV GEMM (N=12288), identity
attention (V passthrough) + ConvRot quant, outproj gate-residual, prologue,
FC1 + GELU, ConvRot quant, FC2 gate-residual.  Tokens are sharded contiguously
across the N ranks (weights replicated); one NCCL all-gather assembles the final
BF16 [98304, 4096] output.  A step = one pass of the 8-block stack over all
98304 tokens (total work fixed as N grows: strong scaling).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...

Rank 0 prints one JSON line.  `value` is device-timed tokens/s (inputs resident
in HBM, CUDA events on the compute stream, max over ranks); `e2e` is the same
metric through the public API with the step's input copied from pinned host
memory and the whole [M, D] output read back to host memory inside the timed
region (N>1: every rank writes its rows into one node-shared pinned buffer;
`e2e.output` says which form ran).  The
per-kernel roofline comes from CUDA events around every launch of the timed
region.  `--impl reference` times the CPU restatement of the path (oracle/) on
the host cores: the reference has no CPU implementation of its own.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path[:0] = [str(ROOT), str(ROOT / "comfyui-h3-speedkit_b200")]

METRIC = "INT8 DiT-block TOPS and tokens/s at 1/2/4/8 B200; % INT8/HBM roofline"
D, FFN, BLOCKS, TOKENS = 4096, 16384, 8, 98304
ATTN, SWIGLU = 4096, False          # cfg5: attention width = D, GELU MLP
# --geometry h3: the H3 model's block (hidden 5376, attention 7168, SwiGLU MLP of
# width 14336), the real model's geometry beside config 5's generic one
GEOMETRIES = {"cfg5": (4096, 4096, 16384, False), "h3": (5376, 7168, 14336, True)}
CPU_SAMPLE_TOKENS = 1024
FALLBACK_BF16_SUSTAINED = 1400.0   # TFLOP/s, used only if MEASURED_PEAKS.json is absent
FALLBACK_HBM = 6650.0              # GB/s


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--tokens", type=int, default=TOKENS, help="total tokens (default: config 5's 98304)")
    ap.add_argument("--blocks", type=int, default=BLOCKS)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-single-ops", action="store_true",
                    help="N=1: leave out the BASELINE config 1-4 single-op lines nested in the stack line")
    ap.add_argument("--geometry", choices=tuple(GEOMETRIES), default="cfg5",
                    help="block geometry of the stack: cfg5 (default) or the H3 model's own (SwiGLU)")
    ap.add_argument("--config", type=int, choices=(1, 2, 3, 4, 5), default=5,
                    help="5 (default): the 8-block stack; 1-4: the single-op BASELINE configs on one GPU")
    ap.add_argument("--op", choices=("qkv", "attention", "block"), default=None,
                    help="qkv: the QKV op (projection -> pre-quantised attention operands) at the H3 "
                         "geometry on one GPU, --tokens rows; attention: the INT8 attention on those "
                         "operands (56 heads, one sequence of --attn-tokens tokens); block: one whole H3 "
                         "block with its INT8 attention through runtime.Backend.block (--attn-tokens tokens)")
    ap.add_argument("--attn-tokens", type=int, default=32768,
                    help="sequence length of the --op attention line (default 32768)")
    ap.add_argument("--attn-heads", type=int, default=56,
                    help="head count of the --op attention line (default 56, the H3 geometry)")
    return ap.parse_args()


def measured_peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return data, "measured"
    return {"bf16_tflops": 1590.0, "bf16_tflops_sustained": FALLBACK_BF16_SUSTAINED, "hbm_gbs": FALLBACK_HBM}, "fallback"


def int8_peaks(lib, stream) -> dict:
    """Dense INT8 tensor peak of this GPU, the roofline denominator of the GEMMs.

    burst: the live tcgen05 kind::i8 issue-rate probe (every SM issues back-to-back
    128x256x32 MMAs from shared memory into TMEM; no operand traffic), measured on
    this GPU at the start of the run -- the figure for an op timed alone.
    sustained: burst x (bf16_tflops_sustained / bf16_tflops) of MEASURED_PEAKS.json,
    i.e. scaled by the clock loss the same pool's cuBLAS GEMM shows between a burst
    and a seconds-long loop under the 1 kW power cap -- the figure for a GEMM timed
    inside the long block-stack step.  Without a probe result the burst falls back
    to 2 x bf16_tflops (INT8 dense = 2 x BF16 dense on B200)."""
    import ctypes as ct
    peaks, kind = measured_peaks()
    bf16_burst = float(peaks.get("bf16_tflops", 1590.0))
    bf16_sust = float(peaks.get("bf16_tflops_sustained", FALLBACK_BF16_SUSTAINED))
    tops = ct.c_double(0.0)
    probe = None
    for _ in range(2):   # the first call warms the clocks up; keep the better one
        if lib.h3sk_int8_mma_peak(1 << 16, ct.byref(tops), stream) == 0 and tops.value > 0:
            probe = max(probe or 0.0, tops.value)
    burst = probe if probe else 2.0 * bf16_burst
    src = ("live tcgen05 kind::i8 probe" if probe else f"2 x bf16_tflops of {kind} MEASURED_PEAKS.json")
    return {"burst": burst, "sustained": burst * bf16_sust / bf16_burst, "probe_tops": probe,
            "burst_source": src,
            "sustained_source": f"burst x bf16_tflops_sustained/bf16_tflops ({bf16_sust:.1f}/{bf16_burst:.1f}) "
                                f"of {kind} MEASURED_PEAKS.json"}


class ClockSampler:
    """nvidia-smi clock / throttle-reason sampler running during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self):
        self.proc = None
        self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200"], stdout=self.file, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.file.flush()
        rows = []
        with open(self.file.name) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        os.unlink(self.file.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}

        def num(v):
            try:
                return float(v)
            except ValueError:
                return None
        sm = [num(r[1]) for r in rows if num(r[1]) is not None]
        mx = [num(r[2]) for r in rows if num(r[2]) is not None]
        power = [num(r[3]) for r in rows if num(r[3]) is not None]
        reasons = set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for r in rows:
            for name, v in zip(names, r[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(name)
        loaded = [s for s in sm if s and s > 0.5 * (max(mx) if mx else 0)] or sm
        return {"sm_mhz": statistics.median(loaded) if loaded else None, "sm_max_mhz": max(mx) if mx else None,
                "power_w_max": max(power) if power else None, "samples": len(rows), "reasons": sorted(reasons)}


_CPU_DATA = {}


def _cpu_data(tokens: int):
    """Seeded block-0 weights and `tokens` input rows for the CPU sample (drawn once)."""
    if tokens not in _CPU_DATA:
        import numpy as np
        import torch

        from h3_speedkit import synthetic
        from oracle import chain
        if "block" not in _CPU_DATA:
            _CPU_DATA["block"] = chain.NpBlock.from_torch(synthetic.cfg5_block(0, D, FFN, attn=ATTN, swiglu=SWIGLU))
        x = synthetic.cfg5_tokens(tokens, D).view(torch.int16).numpy().view(np.uint16)
        _CPU_DATA[tokens] = (x, np.zeros((tokens,), np.int32))
    return _CPU_DATA["block"], *_CPU_DATA[tokens]


def cpu_block_sample(tokens: int, threads: int, repeats: int = 1):
    """Time one block of the CPU restatement on `tokens` tokens; returns seconds per block."""
    import torch

    from oracle import chain

    torch.set_num_threads(threads)
    os.environ["H3SK_ORACLE_THREADS"] = str(threads)
    b, x, rows = _cpu_data(tokens)
    chain.block(x[:64], b, rows[:64], threads=threads)   # warm-up (threads, pages)
    times = []
    for _ in range(repeats):
        t0 = time.perf_counter()
        chain.block(x, b, rows, threads=threads)
        times.append(time.perf_counter() - t0)
    return min(times)


def host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def run_reference(args):
    """CPU restatement of the path on the host cores (rank 0 only)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    threads = host_threads()
    for _ in range(args.warmup):
        cpu_block_sample(CPU_SAMPLE_TOKENS // 4, threads)
    t0 = time.perf_counter()
    per_block = []
    for _ in range(args.steps):
        per_block.append(cpu_block_sample(CPU_SAMPLE_TOKENS, threads))
    wall = time.perf_counter() - t0
    sec_block = statistics.median(per_block)
    value = CPU_SAMPLE_TOKENS / (sec_block * args.blocks)
    sample = (f"one block on a {CPU_SAMPLE_TOKENS}-token slice per step (C oracle + torch._int_mm, "
              f"{threads} threads), extrapolated linearly to {args.blocks} blocks")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": sec_block * 1e3 * args.blocks * TOKENS / CPU_SAMPLE_TOKENS,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
        "config": {"workload": workload_name(TOKENS) + " (CPU sample)", "tokens": TOKENS,
                   "blocks": args.blocks, "parallelism": "host threads"},
        "tops": CPU_SAMPLE_TOKENS * block_ops() / sec_block / 1e12,
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "wall_s": wall,
    }
    print(json.dumps(line), flush=True)
    return 0


def fc1_n():
    return 2 * FFN if SWIGLU else FFN


def block_ops():
    """INT8 ops per token per block: QKV + outproj + FC1 + FC2."""
    return 2 * D * 3 * ATTN + 2 * ATTN * D + 2 * D * fc1_n() + 2 * FFN * D


def workload_name(tokens):
    mlp = f"SwiGLU FFN={FFN}" if SWIGLU else f"FFN={FFN} GELU"
    tag = "cfg5" if (D, ATTN, FFN, SWIGLU) == GEOMETRIES["cfg5"] else "H3 geometry"
    return f"{tag}: 8 DiT blocks D={D} attn={ATTN} {mlp} M={tokens}, identity attention, token-sharded"


def run_ours(args):
    import torch
    import torch.distributed as dist

    from h3_speedkit import _lib, synthetic
    from h3_speedkit.stack import ShardedStack, shard_bounds, shared_host_output

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}; launch N>1 with torchrun")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    lib = _lib.load()

    # ---- inputs: weights replicated, tokens sharded -------------------------------
    blocks = [synthetic.cfg5_block(i, D, FFN, device=dev, attn=ATTN, swiglu=SWIGLU) for i in range(args.blocks)]
    start, stop = shard_bounds(args.tokens, world, rank)
    x_full = synthetic.cfg5_tokens(args.tokens, D, device=dev)
    x_src = x_full[start:stop].clone()
    del x_full
    rows = torch.zeros((stop - start,), dtype=torch.int32, device=dev)
    stack = ShardedStack(blocks, rows, args.tokens, D, dev)
    stream = torch.cuda.current_stream(dev)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def step(events=None):
        stack.load(x_src)
        stack.forward(events)

    i8 = int8_peaks(lib, stream.cuda_stream) if rank == 0 else None

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if _lib.pipeline_status(stream.cuda_stream) != 0:
        raise SystemExit("GEMM pipeline reported a timed-out wait during warm-up")

    # ---- device-timed region ------------------------------------------------------
    sampler = ClockSampler() if rank == 0 else None
    events = {}
    if sampler:
        sampler.start()
        time.sleep(0.4)   # first samples before the timed region
    # every rank enters the timed region together (rank 0's sampler start must not
    # show up as waiting time in another rank's first collective)
    barrier()
    torch.cuda.synchronize()
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    t_start.record(stream)
    for _ in range(args.steps):
        step(events)
    t_end.record(stream)
    torch.cuda.synchronize()
    barrier()
    clocks = sampler.stop() if sampler else None
    elapsed = max_over_ranks(t_start.elapsed_time(t_end) / 1e3)
    if _lib.pipeline_status(stream.cuda_stream) != 0:
        raise SystemExit("GEMM pipeline reported a timed-out wait")

    # per-kernel device time (events around every launch inside the timed region)
    per_kernel = {}
    for name, pairs in events.items():
        times = [s.elapsed_time(e) for s, e in pairs]
        per_kernel[name] = {"launches": len(times), "total_ms": sum(times), "avg_ms": sum(times) / len(times)}

    # ---- end-to-end through the public API (pinned host in, host out) -------------
    e2e = None
    if not args.no_e2e:
        host_in = x_src.cpu().pin_memory()
        # N>1: one node-shared pinned output that every rank fills over its own PCIe
        # link; without room for it, rank 0 receives the gathered rows
        host_out = shared_host_output(args.tokens, D) if world > 1 else None
        shared = host_out is not None
        if not shared:
            host_out = torch.empty((args.tokens, D), dtype=torch.bfloat16).pin_memory() if rank == 0 else None
            out_desc = ("rank 0 pinned host buffer after the per-chunk NCCL all-gather" if world > 1
                        else "pinned host buffer")
        else:
            out_desc = "node-shared pinned host buffer [M, D]; every rank copies its own rows (no device gather)"
        stack.forward_host(host_in, host_out, shared_out=shared)   # untimed: builds the chunk plans and streams
        barrier()
        torch.cuda.synchronize()
        e_start = torch.cuda.Event(enable_timing=True)
        e_end = torch.cuda.Event(enable_timing=True)
        e_start.record(stream)
        for _ in range(args.steps):
            # public API: H2D of the input chunks, the block stack and the D2H of
            # the output rows (per rank into the shared buffer, or the per-chunk
            # gather and rank 0's D2H), the copies overlapping the compute
            stack.forward_host(host_in, host_out, shared_out=shared)
        e_end.record(stream)
        torch.cuda.synchronize()
        barrier()
        e_elapsed = max_over_ranks(e_start.elapsed_time(e_end) / 1e3)
        e2e = {"value": args.tokens * args.steps / e_elapsed, "unit": "tokens/s",
               "h2d_bytes_per_step": args.tokens * D * 2, "d2h_bytes_per_step": args.tokens * D * 2,
               "ms_per_step": e_elapsed * 1e3 / args.steps, "output": out_desc}

    # ---- BASELINE single-op configs 1-4 (rank 0, N=1 only) -------------------------
    singles = None
    if rank == 0 and world == 1 and not args.no_single_ops:
        singles = {}
        for c in (1, 2, 3, 4):
            singles[f"cfg{c}"] = single_op(c, lib, i8, warmup=10, iters=50, e2e_iters=5,
                                           cpu_baseline=not args.no_cpu_baseline)
            torch.cuda.empty_cache()

    # ---- CPU baseline (rank 0, N=1 only) ------------------------------------------
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = host_threads()
        sec_block = cpu_block_sample(CPU_SAMPLE_TOKENS, threads, repeats=2)
        cpu = {"value": CPU_SAMPLE_TOKENS / (sec_block * args.blocks), "unit": "tokens/s", "cores": threads,
               "kind": "port",
               "sample": f"one block on a {CPU_SAMPLE_TOKENS}-token slice (C oracle + torch._int_mm), best of 2, "
                         f"extrapolated linearly to {args.blocks} blocks"}

    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return 0

    peaks, peak_kind = measured_peaks()
    int8_peak = i8["sustained"]
    m_local = stop - start
    gemm_ops = {"qkv": 2 * m_local * 3 * ATTN * D, "outproj": 2 * m_local * D * ATTN,
                "fc1": 2 * m_local * fc1_n() * D, "fc2": 2 * m_local * D * FFN}
    gemms = {k: v for k, v in per_kernel.items() if k in gemm_ops}
    dominant = max(gemms, key=lambda k: gemms[k]["total_ms"])
    achieved = gemm_ops[dominant] / (gemms[dominant]["avg_ms"] / 1e3) / 1e12
    # DRAM bytes per launch from the committed ncu capture (per row, scaled by
    # this launch's rows); captured at the cfg5 geometry only
    traffic_rows = {}
    tfile = ROOT / "profiles" / "traffic.json"
    if tfile.exists() and args.geometry == "cfg5":
        traffic_rows = {k: v["bytes_per_row"] for k, v in json.loads(tfile.read_text())["kernels"].items()}
    traffic = traffic_rows[dominant] * m_local if dominant in traffic_rows else None
    step_total = sum(v["total_ms"] for v in per_kernel.values())
    hbm_peak = float(peaks.get("hbm_gbs", FALLBACK_HBM))
    pro = per_kernel.get("prologue")
    prologue_line = None
    if pro:
        pro_bytes = m_local * D * 2 + m_local * D + m_local * 4 + m_local * 4 + 3 * D * 2
        pro_gbs = pro_bytes / (pro["avg_ms"] / 1e3) / 1e9
        prologue_line = {"bound": "hbm", "kernel": "norm_quant_stream (staged tables)", "achieved": pro_gbs,
                         "peak": hbm_peak,
                         "unit": "GB/s", "frac": pro_gbs / hbm_peak, "bytes_per_launch": pro_bytes,
                         "traffic": traffic_rows["prologue"] * m_local if "prologue" in traffic_rows else None}
    value = args.tokens * args.steps / elapsed
    total_ops = args.tokens * block_ops() * args.blocks
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": elapsed * 1e3 / args.steps, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
        "config": {"workload": workload_name(args.tokens),
                   "tokens": args.tokens, "blocks": args.blocks, "d": D, "attn": ATTN, "ffn": FFN,
                   "mlp": "swiglu" if SWIGLU else "gelu",
                   "parallelism": f"tokens/{world} (weights replicated) + 1 all-gather",
                   "l2": "inputs larger than L2 (weights 1.6 GB, activations > 1 GB per step)"},
        "tops": total_ops * args.steps / elapsed / 1e12,
        "roofline": {"bound": "tensor", "kernel": f"int8_gemm_persistent ({dominant})", "achieved": achieved,
                     "peak": int8_peak, "unit": "TOPS", "frac": achieved / int8_peak, "traffic": traffic,
                     "peak_source": "sustained INT8: " + i8["sustained_source"],
                     "int8_mma_probe_tops": i8["probe_tops"], "frac_of_burst": achieved / i8["burst"],
                     "per_gemm": {k: {"tops": round(gemm_ops[k] / (v["avg_ms"] / 1e3) / 1e12, 1),
                                      "frac": round(gemm_ops[k] / (v["avg_ms"] / 1e3) / 1e12 / int8_peak, 4)}
                                  for k, v in gemms.items()},
                     "fc1_epilogue": ("GELU and the FC2-input quantiser's ConvRot256 (h3_int8_gelu_rot); the launch "
                                      "also does that rotation, so its TOPS counts the GEMM's ops over the "
                                      "combined time" if not SWIGLU else "dequant (SwiGLU in the FC2-input quantiser)"),
                     "qkv_epilogue": "dequant, and the V quantiser's ConvRot256 on the V third (h3_int8_rot)"},
        "roofline_prologue": prologue_line,
        "kernels": {k: {"launches": v["launches"], "avg_ms": round(v["avg_ms"], 4),
                        "share": round(v["total_ms"] / step_total, 4)} for k, v in per_kernel.items()},
        "clocks": clocks, "gpu_launches": stack.launches_per_step * args.steps * world,
        "e2e": e2e, "cpu_baseline": cpu, "single_ops": singles,
    }
    print(json.dumps(line), flush=True)
    return 0


# ---- single-op BASELINE configs 1-4 (one GPU) ------------------------------------

def _median_ms(fn, warmup=20, iters=100, rotate=1):
    """Median CUDA-event time of fn(i) over `iters` calls; `rotate` buffer sets
    are cycled so that consecutive calls touch different memory (L2 flushed by
    volume: every config's rotation spans more than twice the 126 MB L2)."""
    import torch
    for i in range(warmup):
        fn(i % rotate)
    torch.cuda.synchronize()
    times = []
    for i in range(iters):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn(i % rotate)
        e.record()
        times.append((s, e))
    torch.cuda.synchronize()
    return statistics.median(a.elapsed_time(b) for a, b in times)


def single_op(cfg: int, lib, i8: dict, *, warmup: int = 20, iters: int = 100, e2e_iters: int = 10,
              cpu_baseline: bool = True) -> dict:
    """One BASELINE single-op config (1-4) on the current GPU: the device-timed
    median with inputs resident in HBM (buffers rotated beyond L2), the same op end
    to end through its Python API with the step's activations copied in from pinned
    host memory and its outputs copied back (weights stay resident, as a model's
    do), the roofline against the burst INT8 peak (an op timed alone) or the
    measured HBM copy bandwidth, and a bounded CPU-restatement baseline."""
    import ctypes as ct
    import numpy as np
    import torch

    from h3_speedkit import synthetic
    from h3_speedkit.ops import gemm
    from h3_speedkit.ops.convrot import quantize_int8_rowwise_convrot64
    dev = torch.device("cuda", torch.cuda.current_device())
    peaks, peak_kind = measured_peaks()
    hbm_peak = float(peaks.get("hbm_gbs", FALLBACK_HBM))
    threads = host_threads()
    torch.set_num_threads(threads)
    st = lambda: torch.cuda.current_stream().cuda_stream
    pin = lambda t: t.contiguous().pin_memory()
    nb = lambda *ts: sum(t.numel() * t.element_size() for t in ts)
    cpu = None
    if cfg == 1:
        inp = synthetic.cfg1()
        x, w, bias = inp["x"].to(dev), inp["w"].to(dev), inp["bias"].to(dev)
        wq, wsc = quantize_int8_rowwise_convrot64(w)          # weights: per output channel, once
        ws = wsc.reshape(-1).contiguous()
        out = torch.empty((x.shape[0], w.shape[0]), dtype=torch.bfloat16, device=dev)

        def run(xd, o):
            q, qs = quantize_int8_rowwise_convrot64(xd)
            gemm.int8_linear(q, wq, qs.reshape(-1), ws, bias=bias, out=o)
        ms = _median_ms(lambda _: run(x, out), warmup=warmup, iters=iters)
        ops = 2.0 * 1024 * 2048 * 2048
        value, unit, bound, peak = ops / (ms / 1e3) / 1e12, "TOPS", "tensor", i8["burst"]
        x_h, out_h = pin(inp["x"]), torch.empty(out.shape, dtype=out.dtype).pin_memory()
        x_d = torch.empty_like(x)

        def e2e(_):
            x_d.copy_(x_h, non_blocking=True)
            run(x_d, out)
            out_h.copy_(out, non_blocking=True)
        io = (nb(x_h), nb(out_h))
        if cpu_baseline:
            from oracle import cpu as ocpu
            xb = inp["x"].view(torch.int16).numpy().view(np.uint16)
            t0 = time.perf_counter()
            qc, sc = ocpu.convrot_quant(xb)
            acc = ocpu.gemm_s32(qc, wq.cpu().numpy())
            ocpu.dequant(acc, sc.reshape(-1), ws.cpu().numpy(), bias.cpu().view(torch.int16).numpy().view(np.uint16))
            cpu_s = time.perf_counter() - t0
            cpu = {"value": ops / cpu_s / 1e12, "unit": "TOPS", "cores": threads, "kind": "port",
                   "sample": "the full config-1 linear (activation quant, int32 GEMM, dequant)"}
        workload = "cfg1: W8A8 linear, X BF16 [1024,2048] quantised per token (ConvRot256), W [2048,2048] per channel"
        per_step = ops
    elif cfg == 2:
        inp = synthetic.cfg2()
        m, k = inp["x"].shape
        sets = 8                                             # 8 x 75.6 MB rotated
        xs = [inp["x"].to(dev) for _ in range(sets)]
        qs_ = [torch.empty((m, k), dtype=torch.int8, device=dev) for _ in range(sets)]
        ss_ = [torch.empty((m, 1), dtype=torch.float32, device=dev) for _ in range(sets)]
        w, sh, sc, rows = (inp[n].to(dev) for n in ("weight", "shift", "scale", "rows"))

        def run(xd, q, qs):
            rc = lib.h3_norm_quant_run_t(xd.data_ptr(), w.data_ptr(), sh.data_ptr(), sc.data_ptr(), rows.data_ptr(),
                                         q.data_ptr(), qs.data_ptr(), None, None, None, m, k, 1, k, k, k,
                                         ct.c_float(1e-6), 1, 0, st())
            if rc:
                raise RuntimeError(f"prologue failed: {rc}")
        ms = _median_ms(lambda i: run(xs[i], qs_[i], ss_[i]), warmup=warmup, iters=iters, rotate=sets)
        nbytes = m * k * 2 + m * k + m * 4 + m * 4 + 3 * k * 2
        value, unit, bound, peak = nbytes / (ms / 1e3) / 1e9, "GB/s", "hbm", hbm_peak
        x_h = pin(inp["x"])
        q_h = torch.empty((m, k), dtype=torch.int8).pin_memory()
        s_h = torch.empty((m, 1), dtype=torch.float32).pin_memory()

        def e2e(_):
            xs[0].copy_(x_h, non_blocking=True)
            run(xs[0], qs_[0], ss_[0])
            q_h.copy_(qs_[0], non_blocking=True)
            s_h.copy_(ss_[0], non_blocking=True)
        io = (nb(x_h), nb(q_h, s_h))
        if cpu_baseline:
            from oracle import cpu as ocpu
            sample = 512
            xb = inp["x"][:sample].view(torch.int16).numpy().view(np.uint16)
            bits = lambda t: t.view(torch.int16).numpy().view(np.uint16)
            t0 = time.perf_counter()
            ocpu.norm_quant(xb, bits(inp["weight"]), bits(inp["shift"]), bits(inp["scale"]),
                            inp["rows"][:sample].numpy(), 1e-6, threads=threads)
            cpu_s = (time.perf_counter() - t0) * m / sample
            cpu = {"value": nbytes / cpu_s / 1e9, "unit": "GB/s", "cores": threads, "kind": "port",
                   "sample": f"{sample} of the 6144 rows, scaled to the full shape"}
        workload = "cfg2: fused prologue, x BF16 [6144,4096], one BF16 table"
        per_step = nbytes
    else:
        inp = synthetic.cfg3() if cfg == 3 else synthetic.cfg4()
        a, w, xs, ws, bias = (inp[n].to(dev) for n in ("a", "w", "xs", "ws", "bias"))
        m, k = a.shape
        n = w.shape[0]
        a_h, xs_h = pin(inp["a"]), pin(inp["xs"])
        if cfg == 3:
            out = torch.empty((m, n), dtype=torch.bfloat16, device=dev)
            op = lambda _: gemm.int8_linear(a, w, xs, ws, bias=bias, gelu=True, out=out)
            out_h = torch.empty((m, n), dtype=torch.bfloat16).pin_memory()

            def e2e(_):
                a.copy_(a_h, non_blocking=True)
                xs.copy_(xs_h, non_blocking=True)
                gemm.int8_linear(a, w, xs, ws, bias=bias, gelu=True, out=out)
                out_h.copy_(out, non_blocking=True)
            io = (nb(a_h, xs_h), nb(out_h))
            workload = "cfg3: FC1 INT8 GEMM + GELU-tanh epilogue, [24576,4096] x [16384,4096]^T"
        else:
            res, gate, rows = inp["residual"].to(dev), inp["gate"].to(dev), inp["rows"].to(dev)
            op = lambda _: gemm.int8_gate_residual(a, w, xs, ws, res, gate, rows, bias=bias, requant=True)
            res_h = pin(inp["residual"])
            back = [torch.empty((m, n), dtype=torch.bfloat16).pin_memory(),
                    torch.empty((m, n), dtype=torch.int8).pin_memory(),
                    torch.empty((m, 1), dtype=torch.float32).pin_memory()]

            def e2e(_):
                a.copy_(a_h, non_blocking=True)
                xs.copy_(xs_h, non_blocking=True)
                res.copy_(res_h, non_blocking=True)
                r, q, s_ = gemm.int8_gate_residual(a, w, xs, ws, res, gate, rows, bias=bias, requant=True)
                for h_t, d_t in zip(back, (r, q, s_)):
                    h_t.copy_(d_t, non_blocking=True)
            io = (nb(a_h, xs_h, res_h), nb(*back))
            workload = ("cfg4: FC2 INT8 GEMM + in-place gate-residual + ConvRot256/INT8 requant, "
                        "[24576,16384] x [4096,16384]^T")
        ms = _median_ms(op, warmup=warmup, iters=iters)
        ops = 2.0 * m * n * k
        value, unit, bound, peak = ops / (ms / 1e3) / 1e12, "TOPS", "tensor", i8["burst"]
        if cpu_baseline:
            sample = 1024
            t0 = time.perf_counter()
            torch._int_mm(inp["a"][:sample], inp["w"].t())
            cpu_s = (time.perf_counter() - t0) * m / sample
            cpu = {"value": ops / cpu_s / 1e12, "unit": "TOPS", "cores": threads, "kind": "port",
                   "sample": f"torch._int_mm on {sample} of the {m} rows (int32 GEMM only), scaled to the full shape"}
        per_step = ops
    e2e_ms = _median_ms(e2e, warmup=2, iters=e2e_iters)
    scale_unit = 1e12 if unit == "TOPS" else 1e9
    return {
        "metric": f"BASELINE config {cfg} ({unit})", "value": value, "unit": unit, "n_gpus": 1, "steps": iters,
        "warmup": warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "int8", "data": "synthetic", "config": {"workload": workload, "timing": f"median of {iters} launches",
                                                       "l2": "buffers rotated beyond L2 or larger than L2"},
        "roofline": {"bound": bound, "achieved": value, "peak": peak, "unit": unit, "frac": value / peak,
                     "traffic": None,
                     "peak_source": ("burst INT8: " + i8["burst_source"] if bound == "tensor"
                                     else f"hbm_gbs of {peak_kind} MEASURED_PEAKS.json")},
        "e2e": {"value": per_step / (e2e_ms / 1e3) / scale_unit, "unit": unit, "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": io[0], "d2h_bytes_per_step": io[1],
                "timing": f"median of {e2e_iters} calls through the op API, copies inside"},
        "cpu_baseline": cpu, "gpu_launches": 2 if cfg in (1, 4) else 1,
    }


def run_config(args):
    """BASELINE configs 1-4 as their own lines (20 warm-up and 100 timed launches,
    median, buffers rotated beyond L2)."""
    if int(os.environ.get("RANK", "0")) != 0:
        return 0
    import torch

    from h3_speedkit import _lib
    torch.cuda.set_device(torch.device("cuda", 0))
    lib = _lib.load()
    i8 = int8_peaks(lib, torch.cuda.current_stream().cuda_stream)
    line = single_op(args.config, lib, i8, cpu_baseline=not args.no_cpu_baseline)
    print(json.dumps(line), flush=True)
    return 0


def run_qkv(args):
    """The QKV op at the H3 geometry (56 heads x 128, hidden 5376, N 21504) on one
    GPU: the five calls of ``QKV.run`` (gather, K-only sample GEMM + its head
    epilogue, anchor detector, QKV GEMM + head epilogue, V scales + V codes: eight
    kernel launches), median over `--steps` calls after `--warmup`, inputs larger
    than L2.  The GEMM alone (same kernel,
    row-major output) is timed beside it for the tensor roofline."""
    if int(os.environ.get("RANK", "0")) != 0:
        return 0
    import ctypes as ct
    import numpy as np
    import torch

    from h3_speedkit import _lib
    from h3_speedkit.ops import gemm
    from h3_speedkit.ops.qkv import QKV
    heads, hidden, m = 56, 5376, args.tokens
    n = 3 * heads * 128
    peaks, peak_kind = measured_peaks()
    hbm_peak = float(peaks.get("hbm_gbs", FALLBACK_HBM))
    threads = host_threads()
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(1234)
    q_cpu = torch.randint(-127, 128, (m, hidden), generator=g, dtype=torch.int8)
    w_cpu = torch.randint(-127, 128, (n, hidden), generator=g, dtype=torch.int8)
    xs_cpu = torch.rand((m, 1), generator=g) * 0.009 + 0.001
    ws_cpu = torch.rand((n, 1), generator=g) * 0.0045 + 0.0005
    ang = torch.rand((m, 48), generator=g) * 6.283
    rope_cpu = torch.stack([ang.cos(), -ang.sin(), ang.sin(), ang.cos()], -1).reshape(1, m, 1, 48, 2, 2)
    rope_cpu = rope_cpu.to(torch.bfloat16)
    qw_cpu = (torch.rand((128,), generator=g) + 0.5).to(torch.bfloat16)
    kw_cpu = (torch.rand((128,), generator=g) + 0.5).to(torch.bfloat16)
    ops = 2.0 * m * n * hidden
    workload = f"QKV op, H3 geometry: q INT8 [{m},{hidden}] x W [{n},{hidden}]^T, 56 heads x 128"
    cfg = {"workload": workload, "tokens": m, "heads": heads, "hidden": hidden,
           "l2": "inputs larger than L2 (D alone is 3*56*M*256 bytes)", "timing": f"median of {args.steps} calls"}
    if args.impl == "reference":
        from oracle import qkv as oqkv
        sample = 256
        bits = lambda t: t.contiguous().view(torch.int16).numpy().view(np.uint16)
        times = []
        for _ in range(max(1, args.steps)):
            t0 = time.perf_counter()
            oqkv.qkv(q_cpu[:sample].numpy(), w_cpu.numpy(), xs_cpu[:sample].numpy(), ws_cpu.numpy(),
                     bits(rope_cpu[:, :sample]).reshape(-1, 192), bits(qw_cpu), bits(kw_cpu), 1e-6, threads=threads)
            times.append(time.perf_counter() - t0)
        cpu_s = statistics.median(times) * m / sample
        value = m / cpu_s
        line = {"metric": "QKV op tokens/s (H3 geometry)", "value": value, "unit": "tokens/s", "n_gpus": 1,
                "steps": args.steps, "warmup": 0, "ms_per_step": cpu_s * 1e3, "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "int8", "data": "synthetic", "config": cfg,
                "impl": "reference",
                "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "port",
                                 "sample": f"{sample} of the {m} rows through the CPU restatement, scaled"},
                "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return 0
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    i8 = int8_peaks(_lib.load(), torch.cuda.current_stream().cuda_stream)
    int8_peak = i8["burst"]
    args_dev = tuple(t.to(dev) for t in (q_cpu, w_cpu, xs_cpu, ws_cpu, rope_cpu, qw_cpu, kw_cpu))
    op = QKV()
    clocks = ClockSampler()
    ms = _median_ms(lambda _: op.run(*args_dev, 1e-6), warmup=max(3, args.warmup), iters=max(3, args.steps))
    q, w, xs, ws = args_dev[:4]
    y = torch.empty((m, n), dtype=torch.bfloat16, device=dev)
    clocks.start()
    gemm_ms = _median_ms(lambda _: gemm.int8_linear(q, w, xs.view(-1), ws.view(-1), out=y),
                         warmup=max(3, args.warmup), iters=max(3, args.steps))
    ms = _median_ms(lambda _: op.run(*args_dev, 1e-6), warmup=1, iters=max(3, args.steps))
    clock = clocks.stop()
    del y
    out = op.run(*args_dev, 1e-6)
    v = out["d"][2]
    lib = _lib.load()
    st = torch.cuda.current_stream().cuda_stream
    vq_ms = _median_ms(lambda _: lib.h3_quant_v(out["vp"].data_ptr(), v.data_ptr(), out["vi"].data_ptr(),
                                                out["vs"].data_ptr(), out["vinv"].data_ptr(), m, heads, st),
                       warmup=3, iters=max(3, args.steps))
    # the QKV GEMM with its head epilogue fused (one launch), timed alone: its
    # tensor roofline, and its cost over the plain dequant GEMM
    fused_ms = _median_ms(lambda _: lib.h3_qkv_quant_kv_ex(
        q.data_ptr(), w.data_ptr(), xs.data_ptr(), ws.data_ptr(), out["d"].data_ptr(), args_dev[4].data_ptr(),
        args_dev[5].data_ptr(), args_dev[6].data_ptr(), ct.c_float(1e-6), out["qi"].data_ptr(),
        out["qs"].data_ptr(), out["vp"].data_ptr(), out["ki"].data_ptr(), out["ks"].data_ptr(),
        out["sk"].data_ptr(), out["anchors"].data_ptr(), m, heads, hidden, None, st),
        warmup=3, iters=max(3, args.steps))
    # end to end: q and the RoPE rows from pinned host memory, the three code
    # tensors and their scales back to pinned host memory, inside the timed region
    pin = lambda t: t.pin_memory()
    q_h, xs_h, rope_h = pin(q_cpu), pin(xs_cpu.float()), pin(rope_cpu)
    res_h = [torch.empty(out[k].shape, dtype=out[k].dtype).pin_memory() for k in ("qi", "ki", "vi", "qs", "ks", "vs")]
    q_d, xs_d, rope_d = torch.empty_like(args_dev[0]), torch.empty_like(args_dev[2]), torch.empty_like(args_dev[4])

    def e2e(_):
        q_d.copy_(q_h, non_blocking=True)
        xs_d.copy_(xs_h, non_blocking=True)
        rope_d.copy_(rope_h, non_blocking=True)
        r = op.run(q_d, w, xs_d, ws, rope_d, args_dev[5], args_dev[6], 1e-6)
        for h_t, k in zip(res_h, ("qi", "ki", "vi", "qs", "ks", "vs")):
            h_t.copy_(r[k], non_blocking=True)
    e2e_ms = _median_ms(e2e, warmup=2, iters=max(3, args.steps))
    h2d = q_cpu.numel() + xs_cpu.numel() * 4 + rope_cpu.numel() * 2
    d2h = sum(t.numel() * t.element_size() for t in res_h)
    # CPU baseline: the restatement on a bounded sample
    from oracle import qkv as oqkv
    sample = 256
    bits = lambda t: t.contiguous().view(torch.int16).numpy().view(np.uint16)
    t0 = time.perf_counter()
    if not args.no_cpu_baseline:
        oqkv.qkv(q_cpu[:sample].numpy(), w_cpu.numpy(), xs_cpu[:sample].numpy(), ws_cpu.numpy(),
                 bits(rope_cpu[:, :sample]).reshape(-1, 192), bits(qw_cpu), bits(kw_cpu), 1e-6, threads=threads)
    cpu_s = (time.perf_counter() - t0) * m / sample
    gemm_tops = ops / (gemm_ms / 1e3) / 1e12
    line = {
        "metric": "QKV op tokens/s (H3 geometry)", "value": m / (ms / 1e3), "unit": "tokens/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int8", "data": "synthetic", "config": cfg,
        "tops": ops / (ms / 1e3) / 1e12,
        "kernels_ms": {"op": ms, "gemm_alone": gemm_ms, "gemm_with_head_epilogue": fused_ms, "v_quant": vq_ms,
                       "samples_and_anchors": ms - fused_ms - vq_ms},
        "roofline": {"bound": "tensor", "kernel": "int8_gemm_persistent (fused QKV head epilogue)",
                     "achieved": ops / (fused_ms / 1e3) / 1e12, "peak": int8_peak, "unit": "TOPS",
                     "frac": ops / (fused_ms / 1e3) / 1e12 / int8_peak, "traffic": None,
                     "peak_source": "burst INT8: " + i8["burst_source"],
                     "gemm_alone_tops": gemm_tops, "head_epilogue_cost": fused_ms / gemm_ms - 1.0},
        "e2e": {"value": m / (e2e_ms / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h},
        "cpu_baseline": None if args.no_cpu_baseline else {
            "value": m / cpu_s, "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"{sample} of the {m} rows through the CPU restatement, scaled"},
        "clocks": clock, "gpu_launches": 8,
    }
    print(json.dumps(line), flush=True)
    return 0


def _attention_operands(m: int, heads: int, dev, seed: int = 4321):
    """Seeded INT8 codes and FP32 scales in the QKV op's output layouts (Q/K
    [1, H, S, 128], V channel-major [H*128, padded S], per-group scales), made
    on the device."""
    import torch
    from h3_speedkit.ops.qkv import PrequantizedInt8Attention
    g = torch.Generator(device=dev).manual_seed(seed)
    parts = (m + 127) // 128
    codes = lambda shape: torch.randint(-127, 128, shape, generator=g, device=dev, dtype=torch.int8)
    rand = lambda shape: torch.rand(shape, generator=g, device=dev)
    return PrequantizedInt8Attention(
        q=codes((1, heads, m, 128)), k=codes((1, heads, m, 128)), v=codes((heads * 128, parts * 128)),
        q_scale=rand((1, heads, parts * 32)) * 0.02 + 0.001, k_scale=rand((1, heads, parts * 4)) * 0.02 + 0.001,
        v_scale=rand((heads * 128,)) * 0.01 + 0.0005, original_head_dim=128, input_dtype=torch.bfloat16,
        attention_scale=128 ** -0.5, cta_k=128, attn_mask=None)


def run_attention(args):
    """The INT8 attention of the H3 block (56 heads x 128, one sequence of
    --attn-tokens tokens attending to itself) on one GPU: h3_dense_launch_window
    on the QKV op's operand layouts, BF16 output stored BSHD.  Median over
    `--steps` launches after `--warmup`; Q, K and V (2.75 GB at 32768 tokens)
    are larger than L2.  `--impl reference` times the reference's own kernel
    (kernels/dense/dense_ring.cu, compiled from its sources into oracle/_ref) on
    the same operands: the reference has no CPU attention to time."""
    if int(os.environ.get("RANK", "0")) != 0:
        return 0
    import ctypes as ct
    import torch

    from h3_speedkit import _lib
    from h3_speedkit.ops.dense import DenseLibrary, allocate_output
    heads, m = args.attn_heads, args.attn_tokens
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    packed = _attention_operands(m, heads, dev)
    ops = 4.0 * m * m * 128 * heads          # Q K^T and P V, 2 ops per multiply-add
    scores = float(m) * m * heads            # one ex2 per score
    cfg = {"workload": f"INT8 attention, H3 geometry: {heads} heads x 128, Sq = Sk = {m}, batch 1",
           "tokens": m, "heads": heads, "head_dim": 128, "layout": "Q/K [1,H,S,128], V [H*128, S], O BSHD",
           "l2": "inputs larger than L2", "timing": f"median of {args.steps} launches"}
    base = {"metric": "INT8 attention TOPS (H3 geometry)", "unit": "TOPS", "n_gpus": 1, "steps": args.steps,
            "warmup": args.warmup, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "int8", "data": "synthetic", "config": cfg}
    st = torch.cuda.current_stream().cuda_stream
    if args.impl == "reference":
        from oracle import ref_gpu
        out = allocate_output(packed, "bshd")
        ra = ref_gpu.dense_args(packed.q, packed.k, packed.v, packed.q_scale, packed.k_scale, packed.v_scale,
                                out, packed.attention_scale)
        fn = ref_gpu._load("ref_dense.so").h3_dense_launch_window
        fn.argtypes = [ct.POINTER(ref_gpu.DenseArgs), ct.c_size_t, ct.c_uint32]
        fn.restype = ct.c_int
        ms = _median_ms(lambda _: fn(ct.byref(ra), st, 0), warmup=max(3, args.warmup), iters=max(3, args.steps))
        value = ops / (ms / 1e3) / 1e12
        line = dict(base, value=value, ms_per_step=ms, impl="reference",
                    cpu_baseline={"value": value, "unit": "TOPS", "cores": 0, "kind": "reference",
                                  "sample": "the reference's GPU kernel on the same operands (no CPU attention "
                                            "exists in the reference)"},
                    e2e={"value": value, "unit": "TOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0})
        print(json.dumps(line), flush=True)
        return 0
    lib = _lib.load()
    dense = DenseLibrary()
    out = allocate_output(packed, "bshd")
    call = dense.bind(packed, out)
    gex2 = ct.c_double(0.0)
    ex2_peak = gex2.value if lib.h3sk_ex2_peak(1 << 14, ct.byref(gex2), st) == 0 else None
    clocks = ClockSampler()
    clocks.start()
    ms = _median_ms(lambda _: call(), warmup=max(3, args.warmup), iters=max(3, args.steps))
    clock = clocks.stop()
    if lib.h3sk_ex2_peak(1 << 14, ct.byref(gex2), st) == 0 and ex2_peak:
        ex2_peak = max(ex2_peak, gex2.value)
    i8 = int8_peaks(lib, st)
    # end to end: codes and scales from pinned host memory, the BF16 output back
    names = ("q", "k", "v", "q_scale", "k_scale", "v_scale")
    host = {k: getattr(packed, k).cpu().pin_memory() for k in names}
    dev_in = {k: torch.empty_like(getattr(packed, k)) for k in names}
    out_h = torch.empty(out.shape, dtype=out.dtype).pin_memory()
    import dataclasses
    staged = dataclasses.replace(packed, **dev_in)
    call_e2e = dense.bind(staged, out)

    def e2e(_):
        for k in names:
            dev_in[k].copy_(host[k], non_blocking=True)
        call_e2e()
        out_h.copy_(out, non_blocking=True)
    e2e_ms = _median_ms(e2e, warmup=1, iters=max(3, min(args.steps, 5)))
    h2d = sum(t.numel() * t.element_size() for t in host.values())
    d2h = out_h.numel() * out_h.element_size()
    achieved = scores / (ms / 1e3) / 1e9
    line = dict(base, value=ops / (ms / 1e3) / 1e12, ms_per_step=ms,
                roofline={"bound": "sfu", "kernel": "attention_kernel (h3_dense_launch_window)",
                          "achieved": achieved, "peak": ex2_peak, "unit": "G ex2/s",
                          "frac": achieved / ex2_peak if ex2_peak else None, "traffic": None,
                          "peak_source": "live ex2.approx throughput probe (h3sk_ex2_peak)",
                          "tensor_frac_of_burst_int8": ops / (ms / 1e3) / 1e12 / i8["burst"]},
                e2e={"value": ops / (e2e_ms / 1e3) / 1e12, "unit": "TOPS", "h2d_bytes_per_step": h2d,
                     "d2h_bytes_per_step": d2h},
                cpu_baseline=None, cpu_baseline_note="no CPU attention: the arithmetic is the GPU's ex2.approx",
                clocks=clock, gpu_launches=1)
    print(json.dumps(line), flush=True)
    return 0


def _block_inputs(m: int, dev):
    """One H3-geometry block (hidden 5376, 56 heads, SwiGLU, two adaLN table rows)
    with seeded synthetic weights, RoPE table, Q/K norm weights and tokens."""
    import torch
    from h3_speedkit import synthetic
    bw = synthetic.h3_block(0, tables=2, device=dev)
    g = torch.Generator(device=dev).manual_seed(77)
    ang = torch.rand((m, 48), generator=g, device=dev) * 6.283
    rope = torch.stack([ang.cos(), -ang.sin(), ang.sin(), ang.cos()], -1).reshape(1, m, 1, 48, 2, 2)
    qw = (torch.rand((128,), generator=g, device=dev) + 0.5).to(torch.bfloat16)
    kw = (torch.rand((128,), generator=g, device=dev) + 0.5).to(torch.bfloat16)
    x = synthetic.cfg5_tokens(m, 5376, device=dev)
    rows = (torch.arange(m, device=dev) % 2).to(torch.int32)
    return bw, rope.to(torch.bfloat16), qw, kw, x, rows


def _block_ns(bw, qw, kw):
    from types import SimpleNamespace as NS

    def linear(w, s):
        return NS(weight=w, weight_int8=w, weight_scale=s)
    return NS(adaln_proj=lambda t: (bw.shift_msa, bw.scale_msa, bw.gate_msa, bw.shift_mlp, bw.scale_mlp,
                                    bw.gate_mlp),
              norm1=NS(weight=bw.norm1, eps=1e-6), norm2=NS(weight=bw.norm2, eps=1e-6),
              attn=NS(qkv_proj=linear(bw.qkv, bw.qkv_s), out_proj=linear(bw.out, bw.out_s),
                      q_norm=NS(weight=qw, eps=1e-6), k_norm=NS(weight=kw, eps=1e-6)),
              mlp=NS(fc1=linear(bw.fc1, bw.fc1_s), fc2=linear(bw.fc2, bw.fc2_s)))


def run_block(args):
    """One whole H3 block (hidden 5376, 56 heads x 128 INT8 attention, SwiGLU MLP
    of width 14336) on --attn-tokens tokens, through runtime.Backend.block with
    attention="int8": prologue, QKV op, INT8 attention, ConvRot, outproj, prologue,
    FC1, SwiGLU quantiser, FC2 -- the reference's runtime.py:126-164.  Median of
    `--steps` blocks after `--warmup` (tokens updated in place, as in the model).
    `--impl reference` times the same block as the chain of the reference's own
    kernels compiled from its sources (its prologue, gather, anchor detector,
    r84_kfourwarp.cu, dense_ring.cu, register ConvRot, gate.cu, fc1.cu and
    Kitchen quantiser), with this library's K-only sample projection and V
    quantiser for the two steps it has no C kernel for."""
    if int(os.environ.get("RANK", "0")) != 0:
        return 0
    import ctypes as ct
    import torch
    m = args.attn_tokens
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    bw, rope, qw, kw, x, rows = _block_inputs(m, dev)
    attn_ops = 4.0 * m * m * 128 * 56
    lin_ops = 2.0 * m * 5376 * (3 * 7168 + 7168 + 2 * 14336 + 14336)
    cfg = {"workload": f"one H3 block with INT8 attention: hidden 5376, 56 heads x 128, SwiGLU 14336, {m} tokens",
           "tokens": m, "hidden": 5376, "heads": 56, "ffn": 14336, "l2": "inputs larger than L2",
           "timing": f"median of {args.steps} blocks"}
    base = {"metric": "H3 block tokens/s (INT8 attention included)", "unit": "tokens/s", "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8", "data": "synthetic", "config": cfg}
    if args.impl == "reference":
        from oracle import ref_gpu
        from h3_speedkit import _lib
        lib = _lib.load()
        st = torch.cuda.current_stream().cuda_stream
        parts = (m + 127) // 128

        def ref_block(_):
            q, qs = ref_gpu.norm_quant(x, bw.norm1, bw.shift_msa, bw.scale_msa, rows, 1e-6)
            sq, sx, sr = ref_gpu.sample_gather(q, qs, rope.view(m, 192))
            sd = torch.empty((3, 56, 9, 128), dtype=torch.bfloat16, device=dev)
            lib.h3_sample_konly_ex(sq.data_ptr(), bw.qkv.data_ptr(), sx.data_ptr(), bw.qkv_s.data_ptr(),
                                   sd.data_ptr(), sr.data_ptr(), qw.data_ptr(), kw.data_ptr(), ct.c_float(1e-6),
                                   9, 56, 5376, None, st)
            sk = sd[1].contiguous()
            t = ref_gpu.qkv_quant_kv(q, bw.qkv, qs, bw.qkv_s, rope, qw, kw, 1e-6, sk, ref_gpu.sample_anchor(sk))
            vi = torch.empty((56 * 128, parts * 128), dtype=torch.int8, device=dev)
            vs = torch.empty((56 * 128,), dtype=torch.float32, device=dev)
            lib.h3_quant_v(t["vp"].data_ptr(), t["d"][2].data_ptr(), vi.data_ptr(), vs.data_ptr(),
                           torch.empty_like(vs).data_ptr(), m, 56, st)
            o = ref_gpu.dense(t["qi"].view(1, 56, m, 128), t["ki"].view(1, 56, m, 128), vi,
                              t["qs"].view(1, 56, parts * 32), t["ks"].view(1, 56, parts * 4), vs, 128 ** -0.5)
            aq, asc, _ = ref_gpu.convrot_register(o.transpose(1, 2).reshape(m, 7168), 0)
            ref_gpu.int8_gate(aq, bw.out, asc.view(-1), bw.out_s, bw.gate_msa, rows, x, out=x)
            q, qs = ref_gpu.norm_quant(x, bw.norm2, bw.shift_mlp, bw.scale_mlp, rows, 1e-6)
            h = ref_gpu.int8(q, bw.fc1, qs.view(-1), bw.fc1_s)
            hq, hs = ref_gpu.kitchen_quant(h, 2)
            ref_gpu.int8_gate(hq, bw.fc2, hs.view(-1), bw.fc2_s, bw.gate_mlp, rows, x, out=x)
        ms = _median_ms(ref_block, warmup=max(3, args.warmup), iters=max(3, args.steps))
        value = m / (ms / 1e3)
        line = dict(base, value=value, ms_per_step=ms, impl="reference",
                    cpu_baseline={"value": value, "unit": "tokens/s", "cores": 0, "kind": "reference",
                                  "sample": "the reference's GPU kernels chained as its runtime.py block"},
                    e2e={"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0})
        print(json.dumps(line), flush=True)
        return 0
    from h3_speedkit.runtime import Backend
    backend = Backend()
    block = _block_ns(bw, qw, kw)

    def ours(_):
        backend.block(block, x, None, None, rope, rows=rows, attention="int8", mlp_act="swiglu")
    clocks = ClockSampler()
    clocks.start()
    ms = _median_ms(ours, warmup=max(3, args.warmup), iters=max(3, args.steps))
    clock = clocks.stop()
    # end to end: the tokens from pinned host memory and back, around the block
    x_h = x.cpu().pin_memory()
    out_h = torch.empty_like(x_h).pin_memory()

    def e2e(_):
        x.copy_(x_h, non_blocking=True)
        backend.block(block, x, None, None, rope, rows=rows, attention="int8", mlp_act="swiglu")
        out_h.copy_(x, non_blocking=True)
    e2e_ms = _median_ms(e2e, warmup=1, iters=max(3, min(args.steps, 5)))
    nbytes = x_h.numel() * x_h.element_size()
    line = dict(base, value=m / (ms / 1e3), ms_per_step=ms, tops=(attn_ops + lin_ops) / (ms / 1e3) / 1e12,
                ops_split={"attention_tops_per_block": attn_ops / 1e12, "linear_tops_per_block": lin_ops / 1e12},
                e2e={"value": m / (e2e_ms / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": nbytes,
                     "d2h_bytes_per_step": nbytes},
                cpu_baseline=None, cpu_baseline_note="no CPU attention: the arithmetic is the GPU's ex2.approx",
                clocks=clock, gpu_launches=16)
    print(json.dumps(line), flush=True)
    return 0


def main():
    global D, ATTN, FFN, SWIGLU
    args = parse_args()
    D, ATTN, FFN, SWIGLU = GEOMETRIES[args.geometry]
    if args.op == "qkv":
        return run_qkv(args)
    if args.op == "attention":
        return run_attention(args)
    if args.op == "block":
        return run_block(args)
    if args.impl == "reference":
        return run_reference(args)
    if args.config != 5:
        return run_config(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
