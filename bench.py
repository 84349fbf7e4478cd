"""Benchmark of the B200 paged-KV attention path (one JSON line on rank 0).

Default workload (``--workload decode``, the BASELINE config 2 the headline
metric is quoted on): per GPU, 64 requests whose context after this step's
token is drawn uniformly from 1024..8192, Qwen3-4B attention heads (32 query /
8 KV, head_dim 128), bf16, 128-token pages with seeded shuffled page tables,
inputs N(0,1) with QK-norm and RoPE theta 1e6. One step = scatter the step's
new K/V into the pool (kernel a) + split-KV decode attention (kernel c) for
one layer. The KV read per step (about 1.2 GB) is far larger than the 126 MB
L2, so no flush is needed between steps.

``--workload prefill`` times config 3 (8 requests x 512-token chunk on a
prefix U[0, 4096]); ``--workload longdecode`` times config 5 (512 requests x
32768-token context in groups of 16 sharing a 4096-token prefix, split across
ranks by group); ``--workload engine`` times config 4 (hayate's own engine and
random-init Qwen3-4B from baseline/_ref, with this repo's KV manager, or with
the reference's under ``--impl reference``).

Multi-GPU: one process per GPU (torchrun), each rank owns its own pool and
requests; there is no collective on the data path. Timing is by CUDA events,
max over ranks (NCCL all_reduce of the elapsed times only). The headline's K
timed steps are replayed from one CUDA graph captured from the same calls (no
host launch inside the timed region); the same K steps launched one by one are
timed beside it (`eager`), with per-launch events for the roofline.

``--workload normrope`` times the fused QK-norm + RoPE + KV scatter kernel
(``PagedKVBatch.prepare_layer``) on config 3's chunk.

The default run adds, beside the config-2 headline: config 3 (and the same shape
on longer prefixes), the fused QK-norm + RoPE + scatter on config 3's chunk,
config 5 at every N (its own 128 steps, with each rank's
kernel time, host time and barrier wait), config 4's engine at N=1, the e2e
number through the public API with host buffers, the CPU baseline, and at N=1
the reference's own GPU attention (its torch.compile'd FlexAttention from
baseline/_ref) timed on the same inputs beside configs 2 and 3.

``--impl reference`` times hayate's OWN CPU attention path (its unmodified
``PagedKVCacheManager``/``PagedKVBatch`` from ``baseline/_ref``, fp32, eager
FlexAttention) with every host thread, on a bounded sample of config 2 (and
config 1 exactly beside it); the NumPy restatement stands in only where the
reference cannot be imported.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "hayate-exp_b200"))
sys.path.insert(0, ROOT)

PEAKS_PATH = os.path.join(ROOT, "MEASURED_PEAKS.json")
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None,
                    help="timed steps (default 2000; config 5's 128 for --workload longdecode)")
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["decode", "prefill", "longdecode", "engine", "normrope"],
                    default="decode")
    ap.add_argument("--split-tokens", type=int, default=0)
    ap.add_argument("--requests", type=int, default=64, help="decode requests per GPU (64 = config 2)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true", help="headline workload only")
    ap.add_argument("--no-engine", action="store_true", help="skip the config-4 engine leg of the default run")
    ap.add_argument("--long-groups", type=int, default=32,
                    help="config 5: prefix groups of 16 requests in the job (32 = config 5; 4 = one "
                         "rank's share at 8 GPUs)")
    ap.add_argument("--no-prefill-plan", action="store_true",
                    help="prefill on the default grid instead of the planned schedule")
    ap.add_argument("--prefix-max", type=int, default=4096,
                    help="prefill workload: prefixes drawn from U[0, prefix-max] (config 3: 4096)")
    ap.add_argument("--reference-gpu", action="store_true",
                    help="time the reference's compiled FlexAttention path on the GPU at any N (by default "
                         "only at N=1; needs baseline/_ref)")
    ap.add_argument("--no-reference-gpu", action="store_true",
                    help="skip the reference's GPU path (timed beside ours by default at N=1)")
    args = ap.parse_args()
    if args.steps is None:
        args.steps = {"longdecode": 128, "normrope": 200}.get(args.workload, 2000)
    return args


def wants_reference_gpu(args, world: int, rank: int) -> bool:
    """The reference's own GPU attention (its torch.compile'd FlexAttention) is timed beside
    ours on rank 0 of a 1-GPU run unless --no-reference-gpu, or at any N with --reference-gpu."""
    if rank != 0 or args.no_reference_gpu:
        return False
    return args.reference_gpu or world == 1


def load_peaks():
    try:
        with open(PEAKS_PATH) as f:
            peaks = json.load(f)
        return peaks, "measured"
    except (OSError, ValueError):
        return FALLBACK_PEAKS, "fallback"


# ---------------------------------------------------------------------------- workloads
def decode_lengths(seed: int, batch: int = 64, lo: int = 1024, hi: int = 8192):
    """Context lengths after the step's token; the cached history is one less."""
    rng = np.random.RandomState(seed)
    return [int(n) for n in rng.randint(lo, hi + 1, size=batch)]


# DRAM bytes per launch of the dominant kernel (dram__bytes_read.sum + dram__bytes_write.sum)
# from one ncu capture each at full size: config 2's fused decode launch (1.1938 GB read +
# 7.37 MB written, 1.013 x the algorithmic bytes) and config 3's prefill launch.
DECODE_CFG2_TRAFFIC = 1.2012e9
PREFILL_CFG3_TRAFFIC = 145.36e6


def attention_flops(cache_lens, query_len: int, num_q_heads: int, head_dim: int) -> int:
    """Causal-valid attention FLOPs of a prefill step: 4 * H_q * D per visible (query, key)
    pair (QK^T and PV, 2 FLOPs per multiply-add), padded tile work not counted."""
    pairs = sum(int(n) * query_len + query_len * (query_len + 1) // 2 for n in cache_lens)
    return pairs * 4 * num_q_heads * head_dim


def prefill_prefixes(seed: int, batch: int = 8, hi: int = 4096):
    rng = np.random.RandomState(seed)
    return [int(n) for n in rng.randint(0, hi + 1, size=batch)]


class ClockSampler:
    """SM clock and clock-event reasons sampled in the background while a leg runs
    (read-only NVML queries every 10 ms; nvidia-smi if NVML is unavailable).

    Samples are kept from ``__enter__`` to ``__exit__``. A leg's timed region can be a few
    milliseconds (20 decode steps take ~4 ms), shorter than any sampling period, so each
    leg calls ``hold(step)`` after its timed loop: the same step keeps the GPU busy for at
    least ``min_s`` more seconds inside the window (untimed), and ``summary()`` reports
    the samples of the whole window.
    """

    REASONS = (("hw_slowdown", 0x8), ("sw_thermal_slowdown", 0x20), ("hw_thermal_slowdown", 0x40),
               ("hw_power_brake_slowdown", 0x80), ("sw_power_cap", 0x4))
    SMI_FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
                  "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                  "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int, period_ms: int = 10):
        self.gpu_index = gpu_index
        self.period_s = period_ms / 1e3
        self.samples: list[tuple[float, set]] = []
        self.max_mhz = None
        self.source = None
        self.held_s = 0.0
        self._stop = threading.Event()
        self._thread = None
        self._proc = None

    def _nvml_handle(self):
        import pynvml
        import torch

        pynvml.nvmlInit()
        try:  # the CUDA device's PCI address: NVML's index order can differ from CUDA's
            props = torch.cuda.get_device_properties(self.gpu_index)
            bus = "%08x:%02x:%02x.0" % (props.pci_domain_id, props.pci_bus_id, props.pci_device_id)
            return pynvml.nvmlDeviceGetHandleByPciBusId(bus.encode())
        except Exception:
            return pynvml.nvmlDeviceGetHandleByIndex(self.gpu_index)

    def _poll_nvml(self, handle):
        import pynvml

        while not self._stop.is_set():
            try:
                mhz = float(pynvml.nvmlDeviceGetClockInfo(handle, pynvml.NVML_CLOCK_SM))
                bits = int(pynvml.nvmlDeviceGetCurrentClocksEventReasons(handle))
            except Exception:
                break
            self.samples.append((mhz, {name for name, bit in self.REASONS if bits & bit}))
            self._stop.wait(self.period_s)

    def _read_smi(self):
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self._proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                mhz, self.max_mhz = float(parts[1]), float(parts[2])
            except ValueError:
                continue
            self.samples.append((mhz, {n for n, f in zip(names, parts[5:9]) if f.lower().startswith("active")}))

    def __enter__(self):
        try:
            import pynvml

            handle = self._nvml_handle()
            self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(handle, pynvml.NVML_CLOCK_SM))
            self.source = "nvml"
            self._thread = threading.Thread(target=self._poll_nvml, args=(handle,), daemon=True)
        except Exception:
            try:
                self._proc = subprocess.Popen(
                    ["nvidia-smi", f"--query-gpu={self.SMI_FIELDS}", "--format=csv,noheader,nounits",
                     "-i", str(self.gpu_index), "-lms", "20"],
                    stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
                self.source = "nvidia-smi"
                self._thread = threading.Thread(target=self._read_smi, daemon=True)
            except OSError:
                return self
        self._thread.start()
        return self

    def hold(self, step, min_s: float = 0.5) -> None:
        """Run ``step()`` (untimed) until at least ``min_s`` seconds of GPU work have passed,
        so the window holds samples taken under the leg's load."""
        import torch

        t0 = time.perf_counter()
        while time.perf_counter() - t0 < min_s:
            for _ in range(8):
                step()
            torch.cuda.synchronize()
        self.held_s = time.perf_counter() - t0

    def __exit__(self, *exc):
        self._stop.set()
        if self._proc is not None:
            self._proc.terminate()
            try:
                self._proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self._proc.kill()
        if self._thread is not None:
            self._thread.join(timeout=2)

    def summary(self):
        sm = [mhz for mhz, _ in self.samples]
        reasons = set().union(*[r for _, r in self.samples]) if self.samples else set()
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": self.max_mhz,
                "reasons": sorted(reasons), "samples": len(sm), "source": self.source,
                "window": "timed region + %.2f s of the same steps right after it" % self.held_s}


# ---------------------------------------------------------------------------- distributed
def dist_setup(args):
    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def _reduce(value: float, op_name: str) -> float:
    import torch
    import torch.distributed as dist

    # NCCL reduces device tensors; gloo (the CPU tests of this logic) host tensors
    device = "cuda" if dist.get_backend() == "nccl" else "cpu"
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=getattr(dist.ReduceOp, op_name))
    return float(t.item())


def max_over_ranks(value: float, world: int) -> float:
    """The slowest rank's time (the job's time): every rank gets the same number."""
    return value if world == 1 else _reduce(value, "MAX")


def sum_over_ranks(value: float, world: int) -> float:
    """Whole-job work (bytes, FLOPs, tokens) from each rank's share."""
    return value if world == 1 else _reduce(value, "SUM")


def gather_over_ranks(value: float, world: int) -> list:
    """Every rank's value, in rank order (e.g. each rank's output checksum)."""
    if world == 1:
        return [value]
    import torch
    import torch.distributed as dist

    device = "cuda" if dist.get_backend() == "nccl" else "cpu"
    mine = torch.tensor([value], dtype=torch.float64, device=device)
    parts = [torch.empty_like(mine) for _ in range(world)]
    dist.all_gather(parts, mine)
    return [float(t.item()) for t in parts]


# ---------------------------------------------------------------------------- decode (cfg 2)
def build_decode(rank: int, split_tokens: int, requests: int = 64):
    import torch

    from hayate_b200 import PagedKVCacheManager
    from hayate_b200 import workloads as W

    ctx = decode_lengths(1000 + rank, batch=requests)
    hist = [n - 1 for n in ctx]
    pages = sum(math.ceil(n / 128) for n in ctx) + 8
    manager = PagedKVCacheManager(1, 8, 128, pages * 128, 128, len(ctx), torch.bfloat16, "cuda")
    manager.split_tokens = split_tokens
    W.shuffle_free_pages(manager, 1000 + rank)
    gen = torch.Generator(device="cuda").manual_seed(1000 + rank)
    handles = [manager.allocate() for _ in ctx]
    for h, n in zip(handles, hist):
        W.fill_history(manager, h, n, gen)
    q, k, v = W.step_inputs(manager, handles, 1, 32, gen)
    return manager, handles, ctx, q, k, v


def run_decode(args, world, rank, local, peaks, peak_kind):
    import torch

    from hayate_b200 import ops

    manager, handles, ctx, q, k, v = build_decode(rank, args.split_tokens, args.requests)
    kv_bytes = sum(ctx) * 8 * 128 * 2 * 2           # K and V rows read by attention
    scatter_bytes = 2 * 2 * len(ctx) * 8 * 128 * 2    # read + write of the new K and V rows
    q_out_bytes = 2 * len(ctx) * 32 * 128 * 2
    step_bytes = kv_bytes + scatter_bytes + q_out_bytes
    batch = manager.begin_batch(handles, 1)
    out = torch.empty((len(ctx), 1, 32, 128), dtype=q.dtype, device="cuda").transpose(1, 2)
    ws = manager.workspace_for(len(ctx), 1, 32, batch.max_kv_len)

    def step(events=None):
        """One decode step: the new K/V rows are written and attended by one launch of the
        decode kernel (PagedKVBatch.write_attend_layer's path)."""
        if events is not None:
            events[0].record()
        ops.paged_attention_scatter(q, k, v, manager.k_cache, manager.v_cache, 0, batch.page_table,
                                    batch.cache_lens_i32, 128, batch.max_kv_len, out=out,
                                    workspace=ws, error_word=manager.error_word,
                                    split_tokens=args.split_tokens)
        if events is not None:
            events[1].record()

    def unfused_step(attn_events=None):
        """The same step as two launches: the scatter kernel, then the decode kernel."""
        ops.kv_scatter(k, v, manager.k_cache, manager.v_cache, 0, batch.page_table,
                       batch.cache_lens_i32, 128, error_word=manager.error_word)
        if attn_events is not None:
            attn_events[0].record()
        ops.paged_attention(q, manager.k_cache, manager.v_cache, 0, batch.page_table,
                            batch.cache_lens_i32, 128, batch.max_kv_len, out=out, workspace=ws,
                            error_word=manager.error_word, split_tokens=args.split_tokens)
        if attn_events is not None:
            attn_events[1].record()

    for _ in range(args.warmup):
        step()
        unfused_step()
    torch.cuda.synchronize()
    manager.check_device_errors()

    # The timed region replays the K steps from one CUDA graph captured from the same calls
    # (what a serving loop does with its decode steps): no host launch inside it, so eight
    # ranks sharing one host's cores cannot leave their GPUs idle between steps. The same K
    # steps launched one by one from Python run right before it: their per-launch events
    # give the kernel time the roofline uses, and the device idle time between launches.
    graph, graph_note = capture_steps(step, args.steps)
    kern = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            for _ in range(args.steps)]
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        barrier(world)
        torch.cuda.synchronize()
        e0.record()
        t_host = time.perf_counter()
        for i in range(args.steps):
            step(kern[i])
        e1.record()
        host_ms = (time.perf_counter() - t_host) * 1e3
        torch.cuda.synchronize()
        barrier(world)
        torch.cuda.synchronize()
        start.record()
        if graph is not None:
            graph.replay()
        else:
            for i in range(args.steps):
                step()
        end.record()
        torch.cuda.synchronize()
        barrier(world)
        clocks.hold(step)
    ms_local = start.elapsed_time(end)
    eager_local = e0.elapsed_time(e1)
    kernel_ms = sum(a.elapsed_time(b) for a, b in kern) / args.steps
    # device idle inside the eager loop: before the first launch, and between launches
    first_gap = e0.elapsed_time(kern[0][0])
    between = sum(kern[i][1].elapsed_time(kern[i + 1][0]) for i in range(args.steps - 1))
    manager.check_device_errors()
    checksums = gather_over_ranks(float(out.double().sum().item()), world)
    per_rank = {
        "elapsed_ms_per_step": [round(x / args.steps, 4) for x in gather_over_ranks(ms_local, world)],
        "eager_elapsed_ms_per_step": [round(x / args.steps, 4) for x in gather_over_ranks(eager_local, world)],
        "kernel_ms": [round(x, 4) for x in gather_over_ranks(kernel_ms, world)],
        "eager_gap_before_first_launch_ms": [round(x, 4) for x in gather_over_ranks(first_gap, world)],
        "eager_gaps_between_launches_ms": [round(x, 4) for x in gather_over_ranks(between, world)],
        "eager_host_enqueue_ms_per_step": [round(x / args.steps, 4) for x in gather_over_ranks(host_ms, world)],
    }
    ms_total = max_over_ranks(ms_local, world)
    eager_total = max_over_ranks(eager_local, world)
    total_bytes = sum_over_ranks(float(step_bytes), world)
    value = total_bytes * args.steps / (ms_total / 1e3) / 1e9
    del graph
    # the roofline's launch duration: the timed region holds only the K launches of the decode
    # kernel, so its length / K is their average (back to back, as in a graph-replayed serving
    # step); with the eager fallback, the per-launch events
    launch_ms = ms_local / args.steps if graph_note.startswith(f"{args.steps} steps replayed") else kernel_ms
    achieved = step_bytes / (launch_ms / 1e3) / 1e9
    peak = peaks["hbm_gbs"]

    # the two-launch step beside it (outside the timed region): scatter, then attention alone
    n_unfused = max(1, args.steps // 4)
    attn = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            for _ in range(n_unfused)]
    u0, u1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize()
    u0.record()
    for i in range(n_unfused):
        unfused_step(attn[i])
    u1.record()
    torch.cuda.synchronize()
    barrier(world)
    unfused_ms = max_over_ranks(u0.elapsed_time(u1), world) / n_unfused
    attn_ms = sum(a.elapsed_time(b) for a, b in attn) / n_unfused
    attn_gbs = kv_bytes / (attn_ms / 1e3) / 1e9
    manager.check_device_errors()
    read_ceiling = plain_read_ceiling(kv_bytes, world)

    result = {
        "metric": "decode attn HBM GB/s (% of peak)",
        "value": round(value, 1),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_total / args.steps, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic: seeded N(0,1) q/k/v, QK-norm + RoPE theta 1e6 at true positions, shuffled page tables",
        "config": {
            "workload": "config 2: bf16 paged decode sweep (scatter + split-KV decode attention, 1 layer; the decode kernel writes the new K/V rows itself)",
            "requests_per_gpu": len(ctx), "kv_len": "U[1024, 8192]", "mean_kv_len": round(float(np.mean(ctx)), 1),
            "query_heads": 32, "kv_heads": 8, "head_dim": 128, "page_size": 128,
            "l2": "inputs larger than L2 (KV read per step ~%.2f GB > 126 MB)" % (kv_bytes / 1e9),
            "parallelism": f"request-parallel x{world} (own pool per GPU, no data-path collective)",
            "split_tokens": args.split_tokens or "auto",
        },
        "step_bytes_per_gpu": step_bytes,
        "unfused": {"step_ms": round(unfused_ms, 4), "step_GB_s": round(step_bytes / (unfused_ms / 1e3) / 1e9, 1),
                    "attention_ms": round(attn_ms, 4), "attention_GB_s": round(attn_gbs, 1),
                    "attention_frac_of_peak": round(attn_gbs / peak, 4),
                    "what": "kv_scatter launch + decode launch (no fused rows), same inputs, %d steps" % n_unfused},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured" else "fallback 6.65 TB/s",
                     "nominal_frac_8TBs": round(achieved / 8000.0, 4),
                     "traffic": DECODE_CFG2_TRAFFIC if len(ctx) == 64 else None,
                     "traffic_unit": "bytes per launch (ncu dram__bytes_read.sum + write.sum)",
                     "bytes_per_launch": step_bytes,
                     "launch_ms": round(launch_ms, 4),
                     "eager_launch_ms": round(kernel_ms, 4),
                     "launch_timing": "timed-region length / K launches (graph-replayed, back to back); "
                                      "eager_launch_ms: events around each launch of the eager loop, which "
                                      "add the launch latency",
                     "kernel": "decode_attention_kernel (split-KV decode with the fused row scatter)"},
        "read_ceiling": read_ceiling,
        "timing": graph_note,
        "eager": {"value": round(total_bytes * args.steps / (eager_total / 1e3) / 1e9, 1),
                  "ms_per_step": round(eager_total / args.steps, 4),
                  "what": "the same K steps launched one by one from Python (max over ranks)"},
        "per_rank": per_rank,
        "gpu_launches": args.steps,
        "clocks": clocks.summary(),
        "output_checksums": [round(c, 6) for c in checksums],
    }
    result["roofline"]["frac_of_read_ceiling"] = round(achieved / read_ceiling["GB_s"], 4)
    if wants_reference_gpu(args, world, rank):
        ref_gpu = reference_gpu_compare(manager, handles, q, k, v, out, kv_bytes / 1e9, "GB_s")
        if "ms" in ref_gpu:
            ref_gpu["ours_attention_ms"] = round(attn_ms, 4)
            ref_gpu["speedup"] = round(ref_gpu["ms"] / attn_ms, 1)
        result["reference_gpu"] = ref_gpu
    if not args.no_e2e:
        result["e2e"] = decode_e2e(args, world, manager, handles, ctx, q, k, v, step_bytes)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        result["cpu_baseline"] = cpu_baseline_decode(manager, batch, q, ctx)
    return result


def capture_steps(step, n: int):
    """The n steps captured into one CUDA graph (replayed as the timed region), or None and
    the reason when capture is not possible (the eager loop is timed instead)."""
    import torch

    try:
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for _ in range(n):
                step()
        torch.cuda.synchronize()
        return graph, f"{n} steps replayed from one CUDA graph captured from the same calls; CUDA events around the replay"
    except Exception as exc:  # pragma: no cover - depends on the box
        return None, f"eager loop ({type(exc).__name__} in graph capture: {str(exc).splitlines()[0][:120]})"


def plain_read_ceiling(nbytes: int, world: int, repeats: int = 20):
    """HBM read ceiling on this GPU: the library's plain streaming-read kernel
    (``hyt_read_probe``, 16-byte loads, 4 in flight per thread) over a contiguous buffer of
    the decode step's KV size (> L2, so every launch reads HBM), best and mean of
    ``repeats`` CUDA-event-timed launches, at the CTA count that reads fastest of a few."""
    import torch

    from hayate_b200 import ops

    sms = torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count
    buf = torch.ones(nbytes // 16 * 16, dtype=torch.uint8, device="cuda")
    best = {}
    for per_sm in (2, 4, 8):
        sink = torch.zeros(sms * per_sm, dtype=torch.int32, device="cuda")
        for _ in range(3):
            ops.read_probe(buf, sink)
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(repeats)]
        for a, b in evs:
            a.record()
            ops.read_probe(buf, sink)
            b.record()
        torch.cuda.synchronize()
        ms = [a.elapsed_time(b) for a, b in evs]
        best[per_sm] = (min(ms), sum(ms) / len(ms))
    per_sm = min(best, key=lambda c: best[c][1])
    ms_min, ms_mean = best[per_sm]
    del buf
    return {"GB_s": round(buf_gbs(nbytes, ms_mean), 1), "best_GB_s": round(buf_gbs(nbytes, ms_min), 1),
            "bytes": nbytes // 16 * 16, "ctas": sms * per_sm,
            "kernel": "read_probe_kernel (hyt_read_probe): contiguous 16-byte streaming loads, no writes",
            "timing": f"mean (and best) of {repeats} launches, CUDA events, buffer > L2"}


def buf_gbs(nbytes: int, ms: float) -> float:
    return nbytes / (ms / 1e3) / 1e9


def decode_e2e(args, world, manager, handles, ctx, q, k, v, step_bytes):
    """Same step through the public API with host buffers: each step copies its inputs
    host -> device and its output device -> host (pinned memory), inside the timed region.

    Measured twice: serial (copy in, compute, copy out, one stream) and pipelined the way a
    serving loop feeds the engine (a copy stream brings step i+1's inputs in and takes step
    i's output out while step i+1 / i computes; double-buffered device inputs). ``value`` is
    the pipelined figure; both are reported."""
    import torch

    B = len(ctx)
    # the step's q, k and v packed in one pinned host buffer: one H2D copy per step
    parts = [t.detach().contiguous() for t in (q, k, v)]
    sizes = [t.numel() for t in parts]
    host_in = torch.empty(sum(sizes), dtype=q.dtype).pin_memory()
    off = 0
    for t, n in zip(parts, sizes):
        host_in[off: off + n].copy_(t.reshape(-1).cpu())
        off += n
    out_h = [torch.empty((B, 32, 1, 128), dtype=q.dtype).pin_memory() for _ in range(2)]
    dev_in = [torch.empty_like(host_in, device="cuda") for _ in range(2)]

    def views(buf):  # q, k, v as [B, H, 1, D] views of one device buffer
        out, off = [], 0
        for t, n in zip(parts, sizes):
            out.append(buf[off: off + n].view(t.shape))
            off += n
        return tuple(out)

    dev = [views(buf) for buf in dev_in]
    meta_bytes = (3 * B + B * max(len(h.pages) for h in handles)) * 4
    total = sum_over_ranks(float(step_bytes), world)

    def serial_step():
        batch = manager.begin_batch(handles, 1)               # H2D: page table + lengths
        dev_in[0].copy_(host_in, non_blocking=True)           # H2D: q, k, v
        qd, kd, vd = dev[0]
        o = batch.write_attend_layer(0, kd, vd, qd)
        out_h[0].copy_(o, non_blocking=True)                  # D2H of the step's result

    compute = torch.cuda.current_stream()
    copier = torch.cuda.Stream()
    inputs_ready = [torch.cuda.Event() for _ in range(2)]
    inputs_free = [torch.cuda.Event() for _ in range(2)]
    output_ready = [torch.cuda.Event() for _ in range(2)]

    def copy_in(i):
        s = i & 1
        with torch.cuda.stream(copier):
            copier.wait_event(inputs_free[s])
            dev_in[s].copy_(host_in, non_blocking=True)
            inputs_ready[s].record(copier)

    def pipelined(steps):
        for s in range(2):
            inputs_free[s].record(compute)
        copy_in(0)
        for i in range(steps):
            s = i & 1
            if i + 1 < steps:
                copy_in(i + 1)
            compute.wait_event(inputs_ready[s])
            batch = manager.begin_batch(handles, 1)
            qd, kd, vd = dev[s]
            o = batch.write_attend_layer(0, kd, vd, qd)
            inputs_free[s].record(compute)
            output_ready[s].record(compute)
            with torch.cuda.stream(copier):
                copier.wait_stream(compute)
                out_h[s].copy_(o, non_blocking=True)
        compute.wait_stream(copier)

    def timed(fn):
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier(world)
        torch.cuda.synchronize()
        start.record()
        fn()
        end.record()
        torch.cuda.synchronize()
        barrier(world)
        return max_over_ranks(start.elapsed_time(end), world)

    for _ in range(max(3, args.warmup)):
        serial_step()
    pipelined(max(3, args.warmup))
    torch.cuda.synchronize()
    ms_serial = timed(lambda: [serial_step() for _ in range(args.steps)])
    ms_pipe = timed(lambda: pipelined(args.steps))
    manager.check_device_errors()
    return {"value": round(total * args.steps / (ms_pipe / 1e3) / 1e9, 1), "unit": "GB/s",
            "ms_per_step": round(ms_pipe / args.steps, 4),
            "serial": {"value": round(total * args.steps / (ms_serial / 1e3) / 1e9, 1),
                       "ms_per_step": round(ms_serial / args.steps, 4)},
            "h2d_bytes_per_step": int(host_in.numel() * host_in.element_size() + meta_bytes),
            "d2h_bytes_per_step": int(out_h[0].numel() * 2),
            "path": "PagedKVCacheManager.begin_batch -> PagedKVBatch.write_attend_layer (write_layer + "
                    "attend_layer in one launch), q/k/v in one pinned host buffer (one H2D copy), the "
                    "output back to pinned memory; copies on a second stream overlap the "
                    "neighbouring steps"}


def cpu_threads() -> int:
    return len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()


def import_reference():
    """hayate's own modules from the offline install in ``baseline/_ref``, or the reason they
    cannot be imported."""
    if not os.path.isdir(os.path.join(REF_DIR, "hayate")):
        return None, "the reference is not installed in baseline/_ref"
    if REF_DIR not in sys.path:
        sys.path.insert(0, REF_DIR)
    try:
        import hayate.engine.paged_cache as paged_cache
        from hayate.model.cache import Cache
        from hayate.model.rope import apply_rope_vectorized, compute_rope_params

        return (paged_cache, Cache, compute_rope_params, apply_rope_vectorized), None
    except Exception as exc:  # pragma: no cover - depends on the box
        return None, f"{type(exc).__name__}: {str(exc).splitlines()[0][:200]}"


# The reference's CPU attention path on two workloads (fp32, its own manager and batch):
# config 1 exactly, and a bounded sample of config 2 (its first 4 requests).
REF_CPU_WORKLOADS = {
    "config1": {"history": [511] * 4, "pool": 16384,
                "what": "config 1: 4 requests x 512-token context (511 cached + 1 new), pool of 16384 "
                        "slots in 128-token pages, fp32"},
    "config2_sample": {"history": [n - 1 for n in decode_lengths(1000)[:4]], "pool": None,
                       "what": "bounded sample of config 2: its first 4 requests (kv %s), pool sized to "
                               "them plus 8 pages, fp32" % decode_lengths(1000)[:4]},
}


def reference_cpu_path(which: str, steps: int, warmup: int, budget_s: float | None = None):
    """Time hayate's OWN paged attention path on the host cores: ``PagedKVCacheManager
    .begin_batch -> PagedKVBatch.write_layer -> attend_layer`` (``hayate/engine/
    paged_cache.py:202-293,44-71``), unmodified, in fp32 on the CPU. Its module-level
    ``torch.compile(flex_attention)`` does not lower on the CPU (Inductor
    LoweringException), so it is swapped for the eager ``flex_attention`` it wraps; the
    attention math and masks are the reference's. Inputs: N(0,1), RMSNorm (QK-norm) and
    the reference's own RoPE (theta 1e6) at true positions, seeded shuffled free pages.

    One step is one layer's write + attention for the whole sample. ``value`` is GB/s of the
    K/V rows attended, counted in fp32 (4 bytes per element, the dtype the reference runs
    in). Timing stops early once ``budget_s`` seconds of steps are done."""
    mods, why = import_reference()
    if mods is None:
        return {"unavailable": why}
    paged_cache, Cache, compute_rope_params, apply_rope = mods
    from torch.nn.attention.flex_attention import flex_attention

    # the swap lasts for this call only: the GPU comparisons later in the same process time
    # the reference's compiled wrapper
    compiled = paged_cache._compiled_flex_attention
    paged_cache._compiled_flex_attention = flex_attention
    try:
        return _reference_cpu_steps(which, steps, warmup, budget_s, paged_cache, Cache,
                                    compute_rope_params, apply_rope)
    finally:
        paged_cache._compiled_flex_attention = compiled


def _reference_cpu_steps(which, steps, warmup, budget_s, paged_cache, Cache, compute_rope_params,
                         apply_rope):
    """The timed loop of ``reference_cpu_path`` (eager FlexAttention already in place)."""
    import random

    import torch

    threads = cpu_threads()
    torch.set_num_threads(threads)
    spec = REF_CPU_WORKLOADS[which]
    hist = spec["history"]
    B, HQ, HKV, D, P = len(hist), 32, 8, 128, 128
    pool = spec["pool"] or (sum(math.ceil((n + 1) / P) for n in hist) + 8) * P
    gen = torch.Generator().manual_seed(1)
    cos, sin = compute_rope_params(D, 1_000_000, max(hist) + 2)

    def qk(shape, pos):
        x = torch.nn.functional.rms_norm(torch.randn(shape, generator=gen), (D,), eps=1e-6)
        return apply_rope(x, cos, sin, pos)

    import warnings

    warnings.filterwarnings("ignore", message="flex_attention called without torch.compile")
    with torch.inference_mode():
        m = paged_cache.PagedKVCacheManager(1, HKV, D, pool, P, B, torch.float32, "cpu")
        m.k_cache.zero_()
        m.v_cache.zero_()
        random.Random(0).shuffle(m._free_pages)
        handles = []
        for n in hist:
            pos = torch.arange(n)[None]
            k = qk((1, HKV, n, D), pos)
            v = torch.randn((1, HKV, n, D), generator=gen)
            handles.append(m.allocate_for_request(Cache.from_tensors(k, v)))  # [layers=1, H_kv, n, D]
        pos = torch.tensor(hist)[:, None]
        q, kn, vn = qk((B, HQ, 1, D), pos), qk((B, HKV, 1, D), pos), torch.randn((B, HKV, 1, D), generator=gen)
        times = []
        t_start = time.perf_counter()
        for i in range(warmup + steps):
            t0 = time.perf_counter()
            batch = m.begin_batch(handles, 1)
            batch.write_layer(0, kn, vn)
            out = batch.attend_layer(q, 0)
            dt = time.perf_counter() - t0
            if i >= warmup:
                times.append(dt)
            if budget_s is not None and times and time.perf_counter() - t_start > budget_s:
                break
    kv_bytes = sum(n + 1 for n in hist) * HKV * D * 4 * 2
    secs = sum(times)
    return {"value": round(kv_bytes * len(times) / secs / 1e9, 4), "unit": "GB/s",
            "ms_per_step": round(secs / len(times) * 1e3, 2), "steps_timed": len(times),
            "cores": threads, "kind": "reference",
            "sample": spec["what"] + "; one step = begin_batch + write_layer + attend_layer",
            "path": "hayate PagedKVCacheManager.begin_batch -> PagedKVBatch.write_layer -> attend_layer "
                    "(baseline/_ref, unmodified; eager flex_attention in place of its torch.compile "
                    "wrapper, which does not lower on the CPU)",
            "checksum": round(float(out.double().sum()), 6)}


def cpu_port_decode(manager, batch, q, ctx, budget_s: float = 5.0):
    """The oracle (NumPy restatement of the reference path) on a bounded sample of requests."""
    import oracle
    from threadpoolctl import threadpool_limits

    threads = cpu_threads()
    kp = manager.k_cache.float().cpu().numpy()
    vp = manager.v_cache.float().cpu().numpy()
    table = batch.page_table.cpu().numpy().astype(np.int64)
    lens = batch.cache_lens.cpu().numpy()
    qn = q.float().cpu().numpy()
    done, nbytes = 0, 0
    t0 = time.perf_counter()
    with threadpool_limits(limits=threads):
        while time.perf_counter() - t0 < budget_s:
            r = done % len(ctx)
            oracle.paged_attention(qn, kp, vp, 0, table, lens, 128, requests=[r])
            nbytes += ctx[r] * 8 * 128 * 2 * 2
            done += 1
    secs = time.perf_counter() - t0
    return {"value": round(nbytes / secs / 1e9, 3), "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"{done} request-attentions cycling over the {len(ctx)}-request config-2 batch "
                      f"(fp32 NumPy oracle gathering only the attended keys, bf16 bytes counted), {secs:.1f} s"}


def cpu_baseline_decode(manager, batch, q, ctx):
    """The reference's own CPU path timed on the host cores (~10 s on a config-2 sample, ~6 s
    on config 1), with the NumPy restatement's speed beside it."""
    base = reference_cpu_path("config2_sample", steps=1000, warmup=2, budget_s=10.0)
    if "unavailable" in base:  # no reference on this box: the restatement stands in
        port = cpu_port_decode(manager, batch, q, ctx, budget_s=10.0)
        port["reason"] = "reference not importable: " + base["unavailable"]
        return port
    base["config1"] = reference_cpu_path("config1", steps=1000, warmup=2, budget_s=6.0)
    base["port"] = cpu_port_decode(manager, batch, q, ctx)
    return base


# ---------------------------------------------------------------------------- prefill (cfg 3)
def run_prefill(args, world, rank, local, peaks, peak_kind, steps=None, warmup=None, prefix_max=None):
    """8 requests x 512-token chunk on prefixes U[0, prefix_max] (config 3: 4096); scatter +
    tcgen05 prefill attention."""
    import torch

    from hayate_b200 import PagedKVCacheManager, ops
    from hayate_b200 import workloads as W

    steps = args.steps if steps is None else steps
    warmup = args.warmup if warmup is None else warmup
    T = 512
    prefix_max = args.prefix_max if prefix_max is None else prefix_max
    prefixes = prefill_prefixes(2000 + rank, hi=prefix_max)
    pages = sum(math.ceil((n + T) / 128) for n in prefixes) + 8
    manager = PagedKVCacheManager(1, 8, 128, pages * 128, 128, len(prefixes), torch.bfloat16, "cuda")
    W.shuffle_free_pages(manager, 2000 + rank)
    gen = torch.Generator(device="cuda").manual_seed(2000 + rank)
    handles = [manager.allocate() for _ in prefixes]
    for h, n in zip(handles, prefixes):
        W.fill_history(manager, h, n, gen)
    q, k, v = W.step_inputs(manager, handles, T, 32, gen)
    manager.prefill_plan = not args.no_prefill_plan
    batch = manager.begin_batch(handles, T)
    flops = attention_flops(prefixes, T, 32, 128)
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device="cuda")  # > 126 MB L2

    def step(ev=None):
        """write_layer + attend_layer of one layer through the public API."""
        batch.write_layer(0, k, v)
        if ev is not None:
            ev[1].record()
        return batch.attend_layer(q, 0)

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    manager.check_device_errors()
    evs = [tuple(torch.cuda.Event(enable_timing=True) for _ in range(3)) for _ in range(steps)]
    with ClockSampler(local) as clocks:
        barrier(world)
        torch.cuda.synchronize()
        for i in range(steps):
            flush.fill_(i & 0xFF)  # evict the step's inputs from L2 (outside the timed events)
            evs[i][0].record()
            step(evs[i])
            evs[i][2].record()
        torch.cuda.synchronize()
        barrier(world)
        clocks.hold(step)
    manager.check_device_errors()
    out = step()  # the rows (compared with the reference's GPU path's)
    plan = batch.prefill_schedule(q)
    schedule = ("default grid" if plan is None else
                f"planned: {plan[0].shape[0]} CTAs, {plan[1]} items cut in two (longest first)")
    step_ms = sum(a.elapsed_time(c) for a, _, c in evs) / steps
    attn_ms = sum(b.elapsed_time(c) for _, b, c in evs) / steps
    step_ms = max_over_ranks(step_ms, world)
    total_flops = sum_over_ranks(float(flops), world)
    achieved = flops / (attn_ms / 1e3) / 1e12
    ref_gpu = None
    if wants_reference_gpu(args, world, rank):
        ref_gpu = reference_gpu_compare(manager, handles, q, k, v, out, flops / 1e12, "TFLOP_s")
        if "ms" in ref_gpu:
            ref_gpu["ours_attention_ms"] = round(attn_ms, 4)
            ref_gpu["speedup"] = round(ref_gpu["ms"] / attn_ms, 1)
    return {
        "reference_gpu": ref_gpu,
        "workload": f"{'config 3' if prefix_max == 4096 else 'config 3 shape, longer prefixes'}: bf16 chunked "
                    f"prefill, 8 requests x 512-token chunk on prefixes U[0, {prefix_max}]",
        "prefixes": prefixes, "value": round(total_flops / (step_ms / 1e3) / 1e12, 1), "unit": "TFLOP/s",
        "ms_per_step": round(step_ms, 4), "flops_per_step": flops,
        "attention_only": {"ms": round(attn_ms, 4), "TFLOP_s": round(achieved, 1)},
        "roofline": {"bound": "tensor", "achieved": round(achieved, 1), "peak": peaks["bf16_tflops"],
                     "unit": "TFLOP/s", "frac": round(achieved / peaks["bf16_tflops"], 4),
                     "frac_of_sustained": round(achieved / peaks["bf16_tflops_sustained"], 4),
                     "nominal_frac_2250": round(achieved / 2250.0, 4),
                     "peak_source": f"{peak_kind} bf16_tflops (burst)",
                     "traffic": PREFILL_CFG3_TRAFFIC if prefix_max == 4096 else None,
                     "traffic_unit": "bytes per launch (ncu dram__bytes_read.sum + write.sum)",
                     "kernel": "prefill_attention_kernel (tcgen05 + TMEM)"},
        "l2": "256 MB buffer written between timed steps (L2 flush); events bracket each step",
        "schedule": schedule,
        "gpu_launches": 2 * steps,
        "clocks": clocks.summary(),
    }


def run_norm_rope(args, world, rank, local, peaks, peak_kind, steps: int = 50, warmup: int = 5):
    """The fused QK-norm + RoPE + scatter kernel (``PagedKVBatch.prepare_layer``) on config
    3's chunk: 8 requests x 512 new tokens on prefixes U[0, 4096]; q/k/v are the raw
    projections ``[B, T, H, 128]`` the kernel normalises, rotates at their positions and
    writes (q transposed, k/v into their pool pages). HBM-bound: per token it reads q, k, v
    and that position's cos/sin rows and writes q, k, v once."""
    import torch

    from hayate_b200 import PagedKVCacheManager
    from hayate_b200 import workloads as W

    T = 512
    prefixes = prefill_prefixes(2000 + rank, hi=4096)
    pages = sum(math.ceil((n + T) / 128) for n in prefixes) + 8
    manager = PagedKVCacheManager(1, 8, 128, pages * 128, 128, len(prefixes), torch.bfloat16, "cuda")
    W.shuffle_free_pages(manager, 2000 + rank)
    handles = []
    for n in prefixes:
        h = manager.allocate()
        manager.reserve(h, n)
        h.length = n
        handles.append(h)
    gen = torch.Generator(device="cuda").manual_seed(3000 + rank)
    B = len(prefixes)
    q = torch.randn(B, T, 32, 128, generator=gen, device="cuda").to(torch.bfloat16)
    k = torch.randn(B, T, 8, 128, generator=gen, device="cuda").to(torch.bfloat16)
    v = torch.randn(B, T, 8, 128, generator=gen, device="cuda").to(torch.bfloat16)
    wq = (1 + 0.1 * torch.randn(128, generator=gen, device="cuda")).to(torch.bfloat16)
    wk = (1 + 0.1 * torch.randn(128, generator=gen, device="cuda")).to(torch.bfloat16)
    cos, sin = W.rope_angles(torch.arange(max(prefixes) + T, device="cuda"), 128)
    cos, sin = cos.contiguous(), sin.contiguous()
    batch = manager.begin_batch(handles, T)
    tokens = B * T
    # bytes per launch: q read + written (32 heads), k and v read + written (8 heads each),
    # each token's cos and sin rows (fp32) read once
    step_bytes = tokens * (2 * 32 * 128 * 2 + 4 * 8 * 128 * 2 + 2 * 128 * 4)
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device="cuda")  # > 126 MB L2

    def step():
        return batch.prepare_layer(0, q, k, v, wq, wk, cos, sin)

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    manager.check_device_errors()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    with ClockSampler(local) as clocks:
        barrier(world)
        torch.cuda.synchronize()
        for i in range(steps):
            flush.fill_(i & 0xFF)  # evict the step's inputs from L2 (outside the timed events)
            evs[i][0].record()
            step()
            evs[i][1].record()
        torch.cuda.synchronize()
        barrier(world)
        clocks.hold(step)
    manager.check_device_errors()
    ms = max_over_ranks(sum(a.elapsed_time(b) for a, b in evs) / steps, world)
    achieved = step_bytes / (ms / 1e3) / 1e9
    return {
        "workload": "config 3's chunk (8 requests x 512 tokens on prefixes U[0, 4096]): fused QK-norm + "
                    "RoPE + KV scatter of one layer (PagedKVBatch.prepare_layer)",
        "value": round(achieved * world, 1), "unit": "GB/s", "ms_per_launch": round(ms, 4),
        "bytes_per_launch": step_bytes,
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": round(achieved / peaks["hbm_gbs"], 4),
                     "peak_source": f"{peak_kind} hbm_gbs", "kernel": "norm_rope_scatter_kernel"},
        "l2": "256 MB buffer written between timed launches (L2 flush); events bracket each launch",
        "gpu_launches": steps,
        "clocks": clocks.summary(),
    }


# ---------------------------------------------------------------------------- long decode (cfg 5)
LONG_GROUPS, LONG_PER_GROUP, LONG_PREFIX, LONG_CONTEXT, LONG_STEPS = 32, 16, 4096, 32768, 128


def long_groups(rank: int, world: int, groups: int = LONG_GROUPS) -> list[int]:
    """Prefix groups of config 5 this rank serves: whole groups, round robin, so every
    shared prefix stays on one GPU and no data crosses between ranks. ``groups`` < 32 runs
    a share of config 5 (e.g. 4 groups: one rank's share at N=8) on fewer GPUs."""
    return [g for g in range(groups) if g % world == rank]


def run_longdecode(args, world, rank, local, peaks, peak_kind, steps=None, warmup=None):
    """512 requests x 32768-token context, groups of 16 alias a 4096-token prefix (shared
    pages); every request decodes one token per step. Groups are split across ranks.

    Besides tok/s (whole job, max over ranks) the leg reports, per rank and gathered in rank
    order, what bounds the 1 -> N curve: the rank's decode-kernel time per step and its GB/s
    of unique bytes, the host time of ``begin_batch`` (alone, and inside the loop where it
    also blocks on the upload ring once the host is 4 steps ahead), the rank's own elapsed
    time and how long it waited at the closing barrier for the slowest rank."""
    import torch

    from hayate_b200 import PagedKVCacheManager
    from hayate_b200 import workloads as W

    steps = args.steps if steps is None else steps
    warmup = args.warmup if warmup is None else warmup
    t_setup = time.perf_counter()
    groups = long_groups(rank, world, args.long_groups)
    n_req = len(groups) * LONG_PER_GROUP
    own = LONG_CONTEXT - LONG_PREFIX
    unique = len(groups) * (LONG_PREFIX + LONG_PER_GROUP * own)
    pages = unique // 128 + n_req * (steps // 128 + 1) + 8
    manager = PagedKVCacheManager(1, 8, 128, pages * 128, 128, n_req + len(groups),
                                  torch.bfloat16, "cuda")
    W.shuffle_free_pages(manager, 5000 + rank)
    gen = torch.Generator(device="cuda").manual_seed(5000 + rank)
    handles = []
    for _ in groups:
        root = manager.allocate()
        W.fill_history(manager, root, LONG_PREFIX, gen)
        for _ in range(LONG_PER_GROUP):
            h = manager.share(root, LONG_PREFIX)              # prefix pages aliased, not copied
            W.fill_history(manager, h, LONG_CONTEXT, gen, start=LONG_PREFIX)
            handles.append(h)
        manager.release(root)                                 # the 16 sharers keep the pages
    inputs = [W.step_inputs(manager, handles, 1, 32, gen, lengths=[LONG_CONTEXT + s] * n_req)
              for s in range(steps + warmup)]
    torch.cuda.synchronize()
    setup_s = time.perf_counter() - t_setup

    last = [None, None]
    host_ms = [0.0]

    def step(s, ev=None):
        t0 = time.perf_counter()
        batch = manager.begin_batch(handles, 1)
        host_ms[0] += (time.perf_counter() - t0) * 1e3
        q, k, v = inputs[s]
        if ev is not None:
            ev[0].record()
        last[0] = batch.write_attend_layer(0, k, v, q)  # one launch: the decode kernel writes the rows
        last[1] = (batch, k, v, q)
        if ev is not None:
            ev[1].record()
        manager.commit_batch(handles, 1)

    for s in range(warmup):
        step(steps + s)
    torch.cuda.synchronize()
    for h in handles:  # undo the warm-up appends so the timed steps start at 32768
        manager.truncate(h, LONG_CONTEXT)
    host_ms[0] = 0.0
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        barrier(world)
        torch.cuda.synchronize()
        start.record()
        for s in range(steps):
            step(s, evs[s])
        end.record()
        torch.cuda.synchronize()
        t_done = time.perf_counter()
        barrier(world)
        waited_ms = (time.perf_counter() - t_done) * 1e3   # this rank idle at the barrier
        b, k, v, q = last[1]
        clocks.hold(lambda: b.write_attend_layer(0, k, v, q))  # the last step again (same rows)
    manager.check_device_errors()
    # begin_batch's own host time, with the GPU idle (inside the timed loop it also blocks
    # on the upload ring whenever the host runs 4 steps ahead of the GPU)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(10):
        manager.begin_batch(handles, 1)
    host_only_ms = (time.perf_counter() - t0) * 1e3 / 10
    ms_local = start.elapsed_time(end)
    ms = max_over_ranks(ms_local, world)
    attn_ms = sum(a.elapsed_time(b) for a, b in evs) / steps
    checksums = gather_over_ranks(float(last[0].double().sum().item()), world)
    row = 8 * 128 * 2 * 2  # K + V bytes per token
    unique_per_step = sum(len(groups) * (LONG_PREFIX + LONG_PER_GROUP * (own + s + 1)) for s in range(steps)) * row / steps
    logical_per_step = sum(n_req * (LONG_CONTEXT + s + 1) for s in range(steps)) * row / steps
    achieved = unique_per_step / (attn_ms / 1e3) / 1e9
    tokens = sum_over_ranks(float(n_req * steps), world)
    per_rank = {
        "elapsed_ms_per_step": [round(x / steps, 4) for x in gather_over_ranks(ms_local, world)],
        "kernel_ms_per_step": [round(x, 4) for x in gather_over_ranks(attn_ms, world)],
        "kernel_unique_GB_s": [round(x, 1) for x in gather_over_ranks(achieved, world)],
        "begin_batch_host_ms": [round(x, 4) for x in gather_over_ranks(host_only_ms, world)],
        "begin_batch_in_loop_ms_per_step": [round(x / steps, 4) for x in gather_over_ranks(host_ms[0], world)],
        "barrier_wait_ms": [round(x, 3) for x in gather_over_ranks(waited_ms, world)],
        "requests": [int(x) for x in gather_over_ranks(float(n_req), world)],
    }
    return {
        "metric": "long-context decode tok/s (config 5)", "value": round(tokens / (ms / 1e3), 1),
        "unit": "tok/s", "n_gpus": world, "steps": steps, "warmup": warmup,
        "ms_per_step": round(ms / steps, 4), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: seeded N(0,1), QK-norm + RoPE theta 1e6, shuffled pages",
        "config": {"workload": ("config 5: 512 requests x 32768 context, groups of 16 share a 4096-token prefix, 1 layer"
                                if args.long_groups == LONG_GROUPS else
                                f"config 5's shapes, {args.long_groups} of its 32 prefix groups "
                                f"({args.long_groups * LONG_PER_GROUP} requests)"),
                   "requests_this_rank": n_req, "groups_this_rank": len(groups),
                   "parallelism": f"request-parallel by prefix group x{world}",
                   "l2": "KV read per step tens of GB >> 126 MB L2"},
        "unique_GB_per_step_this_rank": round(unique_per_step / 1e9, 2),
        "logical_GB_per_step_this_rank": round(logical_per_step / 1e9, 2),
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": round(achieved / peaks["hbm_gbs"], 4), "bytes": "unique (shared prefix pages once)",
                     "logical_GB_s": round(logical_per_step / (attn_ms / 1e3) / 1e9, 1), "traffic": None,
                     "kernel": "decode_attention_kernel"},
        "attention_ms_per_step": round(attn_ms, 4),
        "per_rank": per_rank,
        "setup_s_rank0": round(setup_s, 1),
        "gpu_launches": steps,
        "clocks": clocks.summary(),
        "output_checksums": [round(c, 6) for c in checksums],
    }


# ---------------------------------------------------------------------------- reference GPU path
def reference_gpu_compare(manager, handles, q, k, v, ours_out, per_step_units, unit, repeats=10):
    """Time the reference's own paged attention on the GPU (torch.compile'd FlexAttention,
    installed from the reference into baseline/_ref) on the same K/V and q, and compare its
    output with ours. The reference pools are zeroed first: it allocates them with
    torch.empty, and FlexAttention multiplies masked-out (zero-weight) keys' V rows too,
    so uninitialised NaN bytes in the pool turn into NaN outputs."""
    import torch

    if not os.path.isdir(os.path.join(REF_DIR, "hayate")):
        return {"unavailable": "the reference is not installed in baseline/_ref"}
    if REF_DIR not in sys.path:
        sys.path.insert(0, REF_DIR)
    try:
        import hayate.engine.paged_cache as ref
        from hayate.model.cache import Cache

        # compile afresh for this shape: with dynamic=True a kernel compiled for an earlier
        # comparison's shape (decode, T=1) would otherwise be reused for a prefill chunk
        torch._dynamo.reset()
        torch.cuda.empty_cache()
        T = q.shape[2]
        rm = ref.PagedKVCacheManager(1, manager.num_kv_heads, manager.head_dim, manager.capacity_tokens,
                                     manager.page_size, len(handles), torch.bfloat16, "cuda")
        rm.k_cache.zero_()
        rm.v_cache.zero_()
        rhs = []
        for h in handles:
            snap = manager.snapshot(h)
            rhs.append(rm.allocate_for_request(Cache.from_tensors(snap.k, snap.v) if h.length else None))
        rb = rm.begin_batch(rhs, T)
        with torch.inference_mode():
            rb.write_layer(0, k.contiguous(), v.contiguous())
            for _ in range(3):
                out = rb.attend_layer(q.contiguous(), 0)
            torch.cuda.synchronize()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            for _ in range(repeats):
                out = rb.attend_layer(q.contiguous(), 0)
            b.record()
            torch.cuda.synchronize()
        ms = a.elapsed_time(b) / repeats
        return {"ms": round(ms, 4), unit: round(per_step_units / (ms / 1e3), 3),
                "max_abs_vs_ours": float((out.float() - ours_out.float()).abs().max().item()),
                "path": "reference PagedKVBatch.attend_layer (torch.compile FlexAttention), same inputs"}
    except Exception as exc:
        return {"unavailable": f"{type(exc).__name__}: {str(exc).splitlines()[0][:200]}"}


# ---------------------------------------------------------------------------- engine (cfg 4)
REF_DIR = os.path.join(ROOT, "baseline", "_ref")
ENGINE_REQUESTS, ENGINE_OUTPUT, ENGINE_POOL, ENGINE_BATCH = 256, 256, 262144, 48


def engine_prompt_lengths(seed: int = 4, n: int = ENGINE_REQUESTS):
    rng = np.random.RandomState(seed)
    return np.clip(np.round(rng.lognormal(np.log(1024), 1.0, size=n)), 1, 8192).astype(int).tolist()


class _StubTokenizer:
    """The engine only decodes finished requests for display; ids are enough here."""

    def decode(self, tokens, skip_special_tokens=True):
        return ""


def run_engine(args, world, rank, impl: str, step: str = "reference"):
    """hayate's own Engine and random-init Qwen3-4B (installed from the
    reference into baseline/_ref), with only the paged KV manager swapped: this repo's
    (impl "ours") or the reference's compiled-FlexAttention one (impl "reference").
    ``step`` "reference" ticks with ``Engine.generate``; "mixed" (ours only) with
    ``hayate_b200.mixed_step.mixed_generate``: one packed forward pass per group of
    prompt chunks, decodes included, instead of one per chunk length plus one for decode."""
    import torch

    if not os.path.isdir(os.path.join(REF_DIR, "hayate")):
        return {"impl": impl, "workload": "engine",
                "unavailable": "the reference engine is not installed in baseline/_ref"}
    sys.path.insert(0, REF_DIR)
    from hayate.engine import engine as ref_engine
    from hayate.engine.request import Request
    from hayate.engine.sampler import Sampler
    from hayate.engine.scheduler import Scheduler
    from hayate.model import Qwen3Model

    if impl == "ours":
        from hayate_b200 import PagedKVCacheManager as Manager
    else:
        from hayate.engine.paged_cache import PagedKVCacheManager as Manager

    torch.manual_seed(0)
    with torch.device("cuda"):
        model = Qwen3Model()
    model.initialize_rope("cuda")
    model.eval()
    eng = ref_engine.Engine.__new__(ref_engine.Engine)
    eng.prefill_chunk_size = 512
    eng.model = model
    eng.num_layers, eng.num_kv_groups, eng.head_dim = model.num_layers, model.num_kv_groups, model.head_dim
    eng.max_position_embeddings = model.max_position_embeddings
    eng.tokenizer = _StubTokenizer()
    eng.stop_token_ids = set()  # fixed-length generation (stop tokens disabled)
    eng.scheduler = Scheduler(max_batch_size=ENGINE_BATCH)
    eng.prefix_cache = None
    eng.sampler = Sampler(eng.tokenizer, set())
    eng.paged_cache = Manager(num_layers=eng.num_layers, num_kv_heads=eng.num_kv_groups,
                              head_dim=eng.head_dim, max_cache_tokens=ENGINE_POOL, page_size=128,
                              max_requests=ENGINE_BATCH, dtype=torch.bfloat16, device="cuda")
    rng = np.random.RandomState(1234)

    def submit(lengths, out_tokens):
        reqs = []
        for i, n in enumerate(lengths):
            r = Request(id=i, prompt_tokens=rng.randint(0, 151936, size=n).tolist(), max_tokens=out_tokens)
            eng._prepare_request(r)
            eng.scheduler.add(r)
            reqs.append(r)
        return reqs

    if step in ("mixed", "graphs"):
        from hayate_b200.mixed_step import DecodeGraphs, mixed_generate

        graphs = DecodeGraphs(eng) if step == "graphs" else None
        tick = lambda: mixed_generate(eng, graphs)  # noqa: E731
    else:
        tick = eng.generate
    with torch.inference_mode():
        # warm-up: library load / FlexAttention compilation on a few shapes
        for _ in range(max(1, args.warmup)):
            submit([700, 33, 1500, 129, 512, 1], 8)
            while tick():
                pass
        lengths = engine_prompt_lengths()
        reqs = submit(lengths, ENGINE_OUTPUT)
        torch.cuda.synchronize()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0 = time.perf_counter()
        start.record()
        while tick():
            pass
        end.record()
        torch.cuda.synchronize()
        wall = time.perf_counter() - t0
    secs = start.elapsed_time(end) / 1e3
    out_tokens = sum(len(r.tokens) for r in reqs)
    prompt_tokens = int(sum(lengths))
    return {
        "impl": impl, "metric": "engine output tok/s (config 4)", "value": round(out_tokens / secs, 1),
        "unit": "tok/s", "n_gpus": 1, "steps": 1, "warmup": args.warmup, "higher_is_better": True,
        "total_tok_s": round((out_tokens + prompt_tokens) / secs, 1), "seconds": round(secs, 3),
        "wall_seconds": round(wall, 3), "dtype": "bf16",
        "data": "random-init Qwen3-4B weights, uniform random token ids, lognormal prompt lengths",
        "config": {"workload": "config 4: hayate Engine, 256 requests, prompts lognormal(median 1024, max 8192), "
                               "256 greedy tokens each, chunk 512, pool 262144 tokens",
                   "max_batch": ENGINE_BATCH, "prompt_tokens": prompt_tokens, "output_tokens": out_tokens,
                   "kv_manager": "hayate_b200" if impl == "ours" else "reference (torch.compile FlexAttention)",
                   "engine_tick": {"mixed": "hayate_b200 mixed_generate (packed prefill + decode passes)",
                                   "graphs": "hayate_b200 mixed_generate, decode-only ticks replayed from "
                                             "CUDA graphs (DecodeGraphs)"}.get(step, "hayate Engine.generate")},
    }


def engine_leg(args):
    """Config 4 beside the headline (N=1): this repository's engine tick (packed prefill +
    decode passes, decode-only ticks replayed from CUDA graphs) and hayate's own tick
    (``Engine.generate``), both on this repository's KV manager and the same random-init
    Qwen3-4B; output tok/s of each. Needs hayate's model and engine from baseline/_ref."""
    import argparse as _ap

    import torch

    quick = _ap.Namespace(**{**vars(args), "warmup": 1})
    try:
        ours = run_engine(quick, 1, 0, "ours", step="graphs")
        if "unavailable" in ours:
            return ours
        torch.cuda.empty_cache()
        theirs = run_engine(quick, 1, 0, "ours", step="reference")
    except Exception as exc:
        return {"unavailable": f"{type(exc).__name__}: {str(exc).splitlines()[0][:200]}"}
    return {"metric": ours["metric"], "value": ours["value"], "unit": "tok/s",
            "total_tok_s": ours["total_tok_s"], "seconds": ours["seconds"], "config": ours["config"],
            "hayate_tick": {k: theirs[k] for k in ("value", "total_tok_s", "seconds")},
            "speedup_vs_hayate_tick": round(ours["value"] / theirs["value"], 3),
            "what": "the same engine, model, requests and KV kernels; only the tick differs (hayate's "
                    "Engine.generate runs one forward pass per distinct prompt-chunk length plus one "
                    "for decode)"}


# ---------------------------------------------------------------------------- reference arm
def run_reference(args, world, rank):
    """The reference arm: hayate's own CPU attention path on the host cores (rank 0 only),
    on this arm's metric and unit. Each step is a bounded sample of config 2 (its first 4
    requests: begin_batch + write_layer + attend_layer, fp32); config 1 exactly is reported
    beside it. Where the reference cannot be imported, the NumPy restatement stands in
    (``kind`` "port", with the reason)."""
    if rank != 0:
        return None
    threads = cpu_threads()
    common = {"impl": "reference", "metric": "decode attn HBM GB/s (% of peak)", "unit": "GB/s",
              "n_gpus": world, "warmup": args.warmup, "higher_is_better": True, "scaling": "weak",
              "vs_baseline": None, "dtype": "f32",
              "data": "synthetic N(0,1), QK-norm + RoPE theta 1e6 (the reference's rope.py), shuffled pages"}
    ref = reference_cpu_path("config2_sample", steps=args.steps, warmup=args.warmup, budget_s=240.0)
    if "unavailable" not in ref:
        value = ref["value"]
        cfg1 = reference_cpu_path("config1", steps=max(3, min(args.steps, 20)), warmup=1, budget_s=30.0)
        return {**common, "value": value, "steps": ref["steps_timed"], "ms_per_step": ref["ms_per_step"],
                "config": {"workload": ref["sample"],
                           "query_heads": 32, "kv_heads": 8, "head_dim": 128, "page_size": 128},
                "cpu_baseline": {k: ref[k] for k in ("value", "unit", "cores", "kind", "sample", "path")},
                "config1": cfg1,
                "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    # fallback: the restatement on one config-2 request per step
    import oracle
    from threadpoolctl import threadpool_limits

    ctx = decode_lengths(1000)
    rng = np.random.RandomState(7)
    sample = list(range(8))
    pools = {}
    for r in sample:
        pages = math.ceil(ctx[r] / 128)
        pools[r] = (rng.standard_normal((1, 1, 8, pages * 128, 128)).astype(np.float32),
                    rng.standard_normal((1, 1, 8, pages * 128, 128)).astype(np.float32),
                    rng.permutation(pages)[None].astype(np.int64),
                    rng.standard_normal((1, 32, 1, 128)).astype(np.float32),
                    rng.standard_normal((1, 8, 1, 128)).astype(np.float32))
    t_total, b_total = 0.0, 0
    with threadpool_limits(limits=threads):
        for i in range(args.warmup + args.steps):
            r = sample[i % len(sample)]
            n = ctx[r]
            kp, vp, table, qn, kn = pools[r]
            t0 = time.perf_counter()
            oracle.kv_scatter(kp, vp, 0, kn, kn, table, np.array([n - 1]), 128)
            oracle.paged_attention(qn, kp, vp, 0, table, np.array([n - 1]), 128)
            dt = time.perf_counter() - t0
            if i >= args.warmup:
                t_total += dt
                b_total += n * 8 * 128 * 2 * 2
    value = b_total / t_total / 1e9
    return {**common, "value": round(value, 3), "steps": args.steps,
            "ms_per_step": round(t_total / args.steps * 1e3, 3),
            "config": {"workload": "config 2: paged decode sweep; each step = one request of the 64-request batch",
                       "query_heads": 32, "kv_heads": 8, "head_dim": 128, "page_size": 128},
            "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                             "sample": "one request per step, rotating over 8 requests of the config-2 batch",
                             "reason": "reference not importable: " + ref["unavailable"]},
            "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


# ---------------------------------------------------------------------------- main
def main():
    args = parse_args()
    if args.workload == "engine":
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        if rank == 0:
            try:
                if args.impl == "ours":
                    # this repo's engine step (packed passes, graph-replayed decode ticks);
                    # beside it the packed step without graphs and hayate's own tick, both
                    # on this repo's KV manager
                    result = run_engine(args, world, rank, "ours", step="graphs")
                    for name, step in (("packed_tick", "mixed"), ("reference_tick", "reference")):
                        torch_mod = sys.modules.get("torch")
                        if torch_mod is not None:
                            torch_mod.cuda.empty_cache()
                        other = run_engine(args, world, rank, "ours", step=step)
                        result[name] = {k: other[k] for k in ("value", "total_tok_s", "seconds")}
                else:
                    result = run_engine(args, world, rank, args.impl)
            except Exception as exc:  # the reference's torch.compile(flex_attention) path
                if args.impl != "reference":
                    raise
                result = {"impl": "reference", "workload": "engine",
                          "unavailable": f"reference GPU path failed: {type(exc).__name__}: "
                                         f"{str(exc).splitlines()[0][:200]}"}
            print(json.dumps(result), flush=True)
        return
    if args.impl == "reference":
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        result = run_reference(args, world, rank)
        if result is not None:
            print(json.dumps(result), flush=True)
        return
    import torch

    world, rank, local = dist_setup(args)
    peaks, peak_kind = load_peaks()
    if args.workload == "decode":
        result = run_decode(args, world, rank, local, peaks, peak_kind)
        if not args.no_extras:
            # config 3 beside the headline (short: 50 timed steps)
            result["prefill"] = run_prefill(args, world, rank, local, peaks, peak_kind, steps=50, warmup=5,
                                            prefix_max=4096)
            # the config-3 launch is short (~0.2 ms, 3.5 CTA waves); the same shape on longer
            # prefixes shows the kernel on long items (there the planned schedule cuts the
            # heaviest in two)
            result["prefill_long_prefix"] = run_prefill(args, world, rank, local, peaks, peak_kind,
                                                        steps=20, warmup=3, prefix_max=32768)
            # the fused QK-norm + RoPE + scatter kernel (the caller's side of the path) on
            # config 3's chunk
            result["norm_rope"] = run_norm_rope(args, world, rank, local, peaks, peak_kind)
            # config 5 at every N: the request-partitioned long-context decode the 1/2/4/8-GPU
            # tok/s is quoted on (its own 128 steps, whatever --steps says)
            torch.cuda.empty_cache()
            result["longdecode"] = run_longdecode(args, world, rank, local, peaks, peak_kind,
                                                  steps=LONG_STEPS, warmup=3)
            if world == 1 and not args.no_engine:
                torch.cuda.empty_cache()
                result["engine"] = engine_leg(args)
    elif args.workload == "prefill":
        result = run_prefill(args, world, rank, local, peaks, peak_kind)
    elif args.workload == "normrope":
        result = run_norm_rope(args, world, rank, local, peaks, peak_kind, steps=args.steps,
                               warmup=args.warmup)
    else:
        result = run_longdecode(args, world, rank, local, peaks, peak_kind)
    if rank == 0:
        print(json.dumps(result), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()
    del torch


if __name__ == "__main__":
    main()
